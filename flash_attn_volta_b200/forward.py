"""Attention forward entry point (drop-in for flash_attn_volta/triton_fa.py:291-401).

`flash_attn_forward` keeps the reference's signature, its AssertionError input
checks (triton_fa.py:313-317), default scale (:319-320) and return convention
(out, or (out, lse) with lse (B, H, N) fp32 natural log, +inf on fully masked
rows).  The work runs in the sm_100a kernel behind fa_sm100_fwd_ex, reached
through the torch.ops.fav.fwd operator (csrc/torch_ops.cpp); there is no
padding of small head dims and no permute copy: the kernel reads the
(B, N, H, D) tensors directly.
"""
from __future__ import annotations

import math

import torch

from . import _lib, ops


def _kv_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> int:
    """K/V head count: q's (multi-head) or a divisor of it (grouped-query /
    multi-query attention: k and v are (B, N_k, H_kv, D), N_k may differ from
    q's N).  Anything else raises the reference's AssertionError."""
    ok = (k.shape == v.shape and q.dim() == 4 and k.dim() == 4 and q.shape[0] == k.shape[0]
          and q.shape[3] == k.shape[3] and k.shape[2] > 0
          and q.shape[2] % k.shape[2] == 0)
    assert ok, f"qkv shape mismatch {q.shape} {k.shape} {v.shape}"
    return k.shape[2]


def _stream_ptr(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    return _lib.stream_ptr(idx)


def flash_attn_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    causal: bool = False,
    sm_scale: float | None = None,
    return_softmax_lse: bool = False,
):
    """FlashAttention forward on B200: fp16 (or bf16) in/out, fp32 accumulation.

    Args:
        q, k, v: (B, N, H, D) fp16 on CUDA (bf16 also accepted: all three the
                 same dtype, output in it). D in {16, 32, 64, 128}.  k and v
                 may also have H_kv heads with H % H_kv == 0 (grouped-query or
                 multi-query attention: query head h uses K/V head h // (H // H_kv)),
                 and N_k rows instead of N (KV-cache prefill and the like).
        causal:  if True apply the top-left lower-triangular mask (for N_k != N
                 aligned to the bottom-right: query i sees keys j <= i + N_k - N;
                 a query row that sees no key gets out 0 and lse +inf).
        sm_scale: softmax scale (default 1/sqrt(D)).
        return_softmax_lse: if True also return the per-row log-sum-exp.

    Returns:
        out: (B, N, H, D) contiguous, q's dtype; with return_softmax_lse also
        lse: (B, H, N) fp32, natural log, +inf for fully masked rows.
    """
    assert q.is_cuda and k.is_cuda and v.is_cuda, "tensors must be on CUDA"
    assert q.dtype in (torch.float16, torch.bfloat16) and q.dtype == k.dtype == v.dtype, \
        "fp16 (or bf16) only, the same for q, k, v"
    Hkv = _kv_heads(q, k, v)
    B, N, H, D = q.shape
    assert D in (16, 32, 64, 128), f"unsupported head_dim {D} (allowed: 16,32,64,128)"
    assert q.device == k.device == v.device, "q, k, v must be on the same device"

    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)

    ops.load()
    ops.note_device(q.device.index)
    out, lse = torch.ops.fav.fwd(q, k, v, bool(causal), float(sm_scale))
    if _lib.debug_sync():
        _lib.check_status(q.device)
    if return_softmax_lse:
        return out, lse
    return out


# Public alias kept from the reference (triton_fa.py:401)
flash_attn_volta = flash_attn_forward
