"""CPU oracle for the attention forward/backward path — TEST INFRASTRUCTURE ONLY.

This module is a checker.  Only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference arm may import it.  The product path
(flash_attn_volta_b200) never calls it and has no CPU fallback.

It restates, in plain torch-on-CPU arithmetic, what the reference computes:

* `attention_fwd`   — flash_attn_volta/ref.py:9-36 (fp32 eager softmax(QK^T*scale)V,
  top-left causal mask built with triu(-inf, diagonal=1), ref.py:27-32) plus the
  log-sum-exp the reference's forward kernel stores: natural log, layout
  (B, H, S) fp32, +inf for rows whose every key is masked
  (flash_attn_volta/triton_fa.py:152-159).
* `attention_bwd`   — the Algorithm-4 backward of flash_attn_volta/triton_fa_bwd.py:
  delta = rowsum(O*dO) (:650), P = exp(S - LSE) (:165), dP = dO V^T (:169),
  dS = P (dP - delta) (:172), dQ = scale dS K (:176-178),
  dV = P^T dO (:415), dK = scale dS^T Q (:426-429), evaluated exactly (no
  tiling) in float64 by default.
* `attention_fwd_tiled` — the online-softmax recurrence of the reference's
  forward kernel (triton_fa.py:117-150: running max with the -inf guard of
  :129, alpha rescale of l and acc, final acc/l), on 64-wide key blocks.  It
  exists to show the recurrence and the exact formula agree.
* `attention_rows`  — exact attention for a subset of query rows, used at sizes
  where the full S x S score matrix does not fit (config 4, long context).

Parity of this oracle with the reference is pinned by tests/test_oracle.py
against tests/golden/*.npz, which tests/golden/make_golden.py produced by
running the reference's own Triton kernels (interpreter mode) and ref.py.
"""
from __future__ import annotations

import math

import torch

__all__ = [
    "attention_fwd",
    "attention_bwd",
    "attention_fwd_tiled",
    "attention_rows",
    "attention_bwd_given_lse",
    "flops_fwd",
    "flops_fwdbwd",
]


def _scores(q, k, causal, scale, dtype, causal_offset=0):
    """(B,S,H,D) inputs -> (B,H,Sq,Sk) scaled, masked scores (ref.py:22-32).

    The causal mask keeps key j for query i when j <= i + causal_offset; the
    reference's square attention is causal_offset = 0 (top-left).  The kernels'
    Sq != Sk extension uses causal_offset = Sk - Sq (bottom-right alignment)."""
    qh = q.permute(0, 2, 1, 3).to(dtype)
    kh = k.permute(0, 2, 1, 3).to(dtype)
    s = torch.einsum("bhnd,bhmd->bhnm", qh, kh) * scale
    if causal:
        n, m = s.shape[-2], s.shape[-1]
        mask = torch.triu(torch.full((n, m), float("-inf"), dtype=dtype),
                          diagonal=1 + causal_offset)
        s = s + mask
    return s


def attention_fwd(q, k, v, causal=False, scale=None, dtype=torch.float32, *, causal_offset=0):
    """Exact forward. Returns (o (B,S,H,D) in `dtype`, lse (B,H,S) in `dtype`).

    Follows ref.py:9-36; the LSE convention follows triton_fa.py:152-159.
    """
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = _scores(q, k, causal, scale, dtype, causal_offset)
    lse = torch.logsumexp(s, dim=-1)
    # a row with every key masked: l == 0 -> the reference stores +inf
    lse = torch.where(torch.isneginf(lse), torch.full_like(lse, float("inf")), lse)
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    vh = v.permute(0, 2, 1, 3).to(dtype)
    o = torch.einsum("bhnm,bhmd->bhnd", p, vh).permute(0, 2, 1, 3).contiguous()
    return o, lse


def attention_bwd(do, q, k, v, causal=False, scale=None, dtype=torch.float64, *,
                  causal_offset=0):
    """Exact backward. Returns (dq, dk, dv), each (B,S,H,D) in `dtype`.

    Restates triton_fa_bwd.py's algorithm (see module docstring) without tiling
    and without the fp16 roundings of P and dS the kernels make.
    """
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = _scores(q, k, causal, scale, dtype, causal_offset)
    p = torch.nan_to_num(torch.softmax(s, dim=-1), nan=0.0)
    vh = v.permute(0, 2, 1, 3).to(dtype)
    qh = q.permute(0, 2, 1, 3).to(dtype)
    kh = k.permute(0, 2, 1, 3).to(dtype)
    doh = do.permute(0, 2, 1, 3).to(dtype)
    oh = torch.einsum("bhnm,bhmd->bhnd", p, vh)
    delta = (oh * doh).sum(-1, keepdim=True)                 # triton_fa_bwd.py:650
    dv = torch.einsum("bhnm,bhnd->bhmd", p, doh)              # P^T dO
    dp = torch.einsum("bhnd,bhmd->bhnm", doh, vh)             # dO V^T
    ds = p * (dp - delta)
    dq = torch.einsum("bhnm,bhmd->bhnd", ds, kh) * scale
    dk = torch.einsum("bhnm,bhnd->bhmd", ds, qh) * scale
    back = lambda t: t.permute(0, 2, 1, 3).contiguous()
    return back(dq), back(dk), back(dv)


def attention_bwd_given_lse(do, q, k, v, o, lse, causal=False, scale=None,
                            dtype=torch.float64):
    """Backward of one (query block, key block) pair given the *global* output O
    and log-sum-exp: P = exp(S - LSE) (triton_fa_bwd.py:165), delta =
    rowsum(O*dO) (:650), dS = P (dP - delta) (:172), dQ = scale dS K,
    dK = scale dS^T Q, dV = P^T dO.  With O and LSE of the block alone this is
    the ordinary backward; with those of a longer key range it is that block's
    share of the gradients.  Returns (dq, dk, dv) like `attention_bwd`.
    """
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    s = _scores(q, k, causal, scale, dtype)
    p = torch.exp(s - lse.to(dtype)[..., None])
    p = torch.nan_to_num(p, nan=0.0)
    vh = v.permute(0, 2, 1, 3).to(dtype)
    qh = q.permute(0, 2, 1, 3).to(dtype)
    kh = k.permute(0, 2, 1, 3).to(dtype)
    doh = do.permute(0, 2, 1, 3).to(dtype)
    oh = o.permute(0, 2, 1, 3).to(dtype)
    delta = (oh * doh).sum(-1, keepdim=True)
    dv = torch.einsum("bhnm,bhnd->bhmd", p, doh)
    dp = torch.einsum("bhnd,bhmd->bhnm", doh, vh)
    ds = p * (dp - delta)
    dq = torch.einsum("bhnm,bhmd->bhnd", ds, kh) * scale
    dk = torch.einsum("bhnm,bhnd->bhmd", ds, qh) * scale
    back = lambda t: t.permute(0, 2, 1, 3).contiguous()
    return back(dq), back(dk), back(dv)


def attention_fwd_tiled(q, k, v, causal=False, scale=None, block_n=64):
    """Online-softmax forward on key blocks (triton_fa.py:117-159), fp32.

    Returns (o, lse) like `attention_fwd`.
    """
    B, S, H, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    qh = q.permute(0, 2, 1, 3).float() * scale
    kh = k.permute(0, 2, 1, 3).float()
    vh = v.permute(0, 2, 1, 3).float()
    m = torch.full((B, H, S), float("-inf"))
    l = torch.zeros((B, H, S))
    acc = torch.zeros((B, H, S, D))
    rows = torch.arange(S)
    for n0 in range(0, S, block_n):
        cols = torch.arange(n0, min(n0 + block_n, S))
        s = torch.einsum("bhnd,bhmd->bhnm", qh, kh[:, :, cols])
        if causal:
            s = s.masked_fill(rows[:, None] < cols[None, :], float("-inf"))
        m_cur = torch.maximum(s.amax(-1), m)
        m_safe = torch.where(torch.isneginf(m_cur), torch.zeros_like(m_cur), m_cur)
        alpha = torch.exp(m - m_safe)
        p = torch.exp(s - m_safe[..., None])
        l = l * alpha + p.sum(-1)
        acc = acc * alpha[..., None] + torch.einsum("bhnm,bhmd->bhnd", p, vh[:, :, cols])
        m = m_safe
    safe_l = torch.where(l > 0, l, torch.ones_like(l))
    o = (acc / safe_l[..., None]).permute(0, 2, 1, 3).contiguous()
    lse = torch.where(l > 0, m + torch.log(safe_l), torch.full_like(l, float("inf")))
    return o, lse


def attention_rows(q, k, v, b, h, rows, causal=False, scale=None, do=None,
                   dtype=torch.float64):
    """Exact forward for query rows `rows` of head (b, h), full key span.

    Returns (o_rows (R,D), lse_rows (R,)) and, when `do` is given, the exact
    dq for those rows (R,D) as a third value.  Used to check large
    configurations on a sample of rows.
    """
    D = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    rows = torch.as_tensor(rows)
    qr = q[b, rows, h].to(dtype)
    kk = k[b, :, h].to(dtype)
    vv = v[b, :, h].to(dtype)
    s = (qr @ kk.T) * scale
    if causal:
        cols = torch.arange(kk.shape[0])
        s = s.masked_fill(rows[:, None] < cols[None, :], float("-inf"))
    lse = torch.logsumexp(s, -1)
    p = torch.exp(s - lse[:, None])
    o = p @ vv
    if do is None:
        return o, lse
    dor = do[b, rows, h].to(dtype)
    dp = dor @ vv.T
    delta = (o * dor).sum(-1, keepdim=True)
    ds = p * (dp - delta)
    dq = (ds @ kk) * scale
    return o, lse, dq


def flops_fwd(B, S, H, D, causal):
    """Forward FLOPs in the convention of the benchmark: 4*B*H*S^2*D, halved if causal."""
    f = 4.0 * B * H * S * S * D
    return f * 0.5 if causal else f


def flops_fwdbwd(B, S, H, D, causal):
    """Forward+backward FLOPs: 2.5x the forward count."""
    return 2.5 * flops_fwd(B, S, H, D, causal)
