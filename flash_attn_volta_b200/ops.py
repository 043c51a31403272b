"""torch.ops.fav: the PyTorch operators over the C ABI.

Loads libfa_torch_ops.so (built in-tree next to this file, see build.py), which
registers the CUDA kernels of ``fav::fwd`` and ``fav::bwd``, and registers here
what torch needs besides: the shape functions used for FakeTensor / meta
tracing (torch.compile, torch.export) and the autograd formula of ``fav::fwd``.

There is no fallback: without the library every call raises RuntimeError.
"""
from __future__ import annotations

import os
import threading

import torch

from .build import ops_path

_lock = threading.Lock()
_loaded = False
_status_devices: set[int] = set()  # devices whose status word exists


def load() -> None:
    """Load libfa_torch_ops.so once (raises RuntimeError when it is missing)."""
    global _loaded
    if _loaded:
        return
    with _lock:
        if _loaded:
            return
        path = os.environ.get("FA_SM100_OPS_LIB") or ops_path()
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with `python -m flash_attn_volta_b200.build` "
                "(the CUDA kernels have no fallback)")
        torch.ops.load_library(path)
        _register_python_parts()
        _loaded = True


def _expect(t, shape, name):
    if tuple(t.shape) != tuple(shape):
        raise RuntimeError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")


def _check_qkv(q, k, v):
    """The shape rules the CUDA operators enforce (csrc/torch_ops.cpp), for
    the shape functions, so a traced call fails where an eager one would."""
    if q.dim() != 4 or k.dim() != 4:
        raise RuntimeError("q, k, v must be (batch, seqlen, heads, head_dim)")
    _expect(k, (q.shape[0], k.shape[1], k.shape[2], q.shape[3]), "k")
    _expect(v, k.shape, "v")
    if k.shape[2] == 0 or q.shape[2] % k.shape[2]:
        raise RuntimeError("the query heads must be a multiple of the key/value heads")


def _register_python_parts() -> None:
    @torch.library.register_fake("fav::fwd")
    def _fwd_fake(q, k, v, causal, sm_scale):
        _check_qkv(q, k, v)
        B, S, H, _ = q.shape
        return q.new_empty(q.shape), q.new_empty((B, H, S), dtype=torch.float32)

    @torch.library.register_fake("fav::bwd")
    def _bwd_fake(dout, q, k, v, out, lse, causal, sm_scale, deterministic=False):
        _check_qkv(q, k, v)
        _expect(dout, q.shape, "dout")
        _expect(out, q.shape, "out")
        _expect(lse, (q.shape[0], q.shape[2], q.shape[1]), "lse")
        return q.new_empty(q.shape), k.new_empty(k.shape), v.new_empty(v.shape)

    @torch.library.register_fake("fav::merge_")
    def _merge_fake(acc_o, acc_lse, o, lse, first):
        _expect(acc_o, o.shape, "acc_o")
        _expect(lse, (o.shape[0], o.shape[2], o.shape[1]), "lse")
        _expect(acc_lse, lse.shape, "acc_lse")
        return None

    def _setup(ctx, inputs, output):
        q, k, v, causal, sm_scale = inputs
        out, lse = output
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal = causal
        ctx.sm_scale = sm_scale
        ctx.mark_non_differentiable(lse)

    def _backward(ctx, dout, dlse):
        q, k, v, out, lse = ctx.saved_tensors
        dout = dout.contiguous()
        if dout.dtype != q.dtype:
            dout = dout.to(q.dtype)
        from ._lib import deterministic_default
        dq, dk, dv = torch.ops.fav.bwd(dout, q, k, v, out, lse, ctx.causal, ctx.sm_scale,
                                       deterministic_default())
        return dq, dk, dv, None, None

    torch.library.register_autograd("fav::fwd", _backward, setup_context=_setup)


def status_word(index: int) -> torch.Tensor:
    """The int32 status word of CUDA device `index` that the operators pass to
    the kernels (bit 0: an on-device wait timed out; bit 1: a row term was
    clamped)."""
    load()
    _status_devices.add(index)
    return torch.ops.fav.status(index)


def note_device(index: int) -> None:
    """Record that the operators ran on CUDA device `index` (they create its
    status word), so that check_status() without a device looks there.  Not
    recorded inside torch.compile tracing (a side effect dynamo refuses); the
    word still exists and check_status(device) finds it."""
    if not torch.compiler.is_compiling():
        _status_devices.add(index)


def status_devices() -> list[int]:
    """CUDA devices whose status word has been created."""
    return sorted(_status_devices)
