"""Autograd-aware entry point (drop-in for flash_attn_volta/autograd.py:19-59).

`_FlashAttnFn.forward` runs the forward with LSE and saves (q, k, v, out, lse)
plus causal / sm_scale; `backward` makes dO contiguous, casts it to q's dtype
(autograd.py:37-39) and runs the backward.
"""
from __future__ import annotations

import math

import torch

from .backward import flash_attn_backward
from .forward import flash_attn_forward


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal: bool, sm_scale: float | None,
                deterministic: bool | None = None):
        if sm_scale is None:
            sm_scale = 1.0 / math.sqrt(q.shape[-1])
        out, lse = flash_attn_forward(q, k, v, causal=causal, sm_scale=sm_scale,
                                      return_softmax_lse=True)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.causal = causal
        ctx.sm_scale = sm_scale
        ctx.deterministic = deterministic
        return out

    @staticmethod
    def backward(ctx, do):
        q, k, v, out, lse = ctx.saved_tensors
        do = do.contiguous()
        if do.dtype != q.dtype:
            do = do.to(q.dtype)
        dq, dk, dv = flash_attn_backward(do, q, k, v, out, lse, causal=ctx.causal,
                                         sm_scale=ctx.sm_scale,
                                         deterministic=ctx.deterministic)
        return dq, dk, dv, None, None, None


def flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
               causal: bool = False, sm_scale: float | None = None, *,
               deterministic: bool | None = None) -> torch.Tensor:
    """Attention with gradients: the B200 forward, and the B200 backward when
    autograd reaches it.

    q, k, v are (batch, seqlen, heads, head_dim) CUDA tensors in fp16 (or bf16),
    head_dim one of 16, 32, 64, 128.  With ``causal`` each query attends only
    to keys at or before its own position.  ``sm_scale`` multiplies the scores
    before the softmax and defaults to head_dim ** -0.5.  The result has q's
    shape and dtype.  ``deterministic`` selects the backward's dQ mode (see
    flash_attn_backward).
    """
    return _FlashAttnFn.apply(q, k, v, causal, sm_scale, deterministic)
