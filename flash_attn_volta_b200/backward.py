"""Attention backward entry point (drop-in for flash_attn_volta/triton_fa_bwd.py:587-700).

`flash_attn_backward(do, q, k, v, o, lse, causal, sm_scale) -> (dq, dk, dv)`
keeps the reference's signature, AssertionError checks (triton_fa_bwd.py:609-614,
:646) and default scale.  delta = rowsum(O*dO), the five backward GEMMs and
the dQ conversion all run on the GPU behind fa_sm100_bwd_ex, reached through
the torch.ops.fav.bwd operator (csrc/torch_ops.cpp); the fp32 workspace it
needs comes from the torch caching allocator and is released on return.
"""
from __future__ import annotations

import math

import torch

from . import _lib, ops
from .forward import _kv_heads


def flash_attn_backward(
    do: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    o: torch.Tensor,
    lse: torch.Tensor,
    causal: bool = False,
    sm_scale: float | None = None,
    *,
    deterministic: bool | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """FlashAttention backward on B200 — fp16 (or bf16) in/out, fp32 accumulation.

    Args:
        do: (B, N, H, D) gradient w.r.t. output, q's dtype (fp16 or bf16).
        q, k, v, o: (B, N, H, D) fp16 forward inputs and output (k, v may have
            H_kv heads, H % H_kv == 0, and N_k rows, as in the forward).
        lse: (B, H, N) fp32 log-sum-exp from the forward (+inf on fully masked rows).
        causal, sm_scale: must match the forward call.
        deterministic: dQ from a separate kernel that sums each query row's key
            blocks in a fixed order (bit-reproducible, like the reference's
            atomics-free dQ kernel) instead of L2 reductions into an fp32
            accumulator.  None = the package default (deterministic_default()).

    Returns:
        (dq, dk, dv), fp16, shaped like q, k and v (dk, dv sum over the query
        heads that share each K/V head).
    """
    assert q.is_cuda and k.is_cuda and v.is_cuda and o.is_cuda and do.is_cuda
    assert q.dtype in (torch.float16, torch.bfloat16)
    assert q.dtype == k.dtype == v.dtype == o.dtype == do.dtype
    assert lse.dtype == torch.float32
    assert q.device == k.device == v.device == o.device == do.device == lse.device, \
        "all tensors must be on the same device"
    assert q.shape == o.shape == do.shape
    Hkv = _kv_heads(q, k, v)
    B, N, H, D = q.shape
    assert D in (16, 32, 64, 128), f"unsupported head_dim {D}"
    assert lse.shape == (B, H, N), f"lse shape {lse.shape} expected ({B},{H},{N})"

    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)

    ops.load()
    ops.note_device(q.device.index)
    if deterministic is None:
        deterministic = _lib.deterministic_default()
    dq, dk, dv = torch.ops.fav.bwd(do, q, k, v, o, lse, bool(causal), float(sm_scale),
                                   bool(deterministic))
    if _lib.debug_sync():
        _lib.check_status(q.device)
    return dq, dk, dv
