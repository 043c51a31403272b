"""flash_attn_volta_b200 — FlashAttention forward + backward for NVIDIA B200 (sm_100a).

Drop-in for the public API of flash_attn_volta (flash_attn_volta/__init__.py:14-24):

    flash_attn_forward(q, k, v, causal=False, sm_scale=None,
                       return_softmax_lse=False)         -> out [, lse]
    flash_attn_volta  (alias of flash_attn_forward)
    flash_attn(q, k, v, causal=False, sm_scale=None)     -> out  (autograd-aware)
    flash_attn_backward(do, q, k, v, o, lse,
                        causal=False, sm_scale=None)     -> (dq, dk, dv)

Tensors are (batch, seq, n_heads, head_dim) fp16 with head_dim in
{16, 32, 64, 128}; LSE is (B, H, N) fp32.  The kernels are hand-written
tcgen05/TMA CUDA in libfa_sm100.so, reached through its C ABI
(include/fa_sm100.h).
"""

from .forward import flash_attn_forward, flash_attn_volta
from .backward import flash_attn_backward
from .autograd import flash_attn
from ._lib import check_status

__all__ = [
    "flash_attn_forward",
    "flash_attn_volta",
    "flash_attn_backward",
    "flash_attn",
]
__version__ = "0.2.0"
