"""The two launch shapes of the main kernels give the same results.

Both main kernels walk a list of tiles: with at most 16 tiles per SM (8 for
causal sequences longer than 4096; this test's are 4096 long) the grid is
one persistent CTA per SM (several rounds of tiles per CTA), otherwise one CTA
per tile.  A tile's arithmetic does not depend on which CTA runs it, so O, LSE,
dK and dV of a head must be bit-identical whether the head is computed among
many heads (one CTA per tile) or alone / in a small slice (persistent grid).
dQ is accumulated with fp32 atomics in an order that depends on timing, so it
is compared within the gradient tolerance.

A second case runs the persistent grid over several rounds with grouped-query
attention and query tiles that see no key (Sq > Sk, causal) in the middle of
the tile list, against the exact oracle.
"""
import math

import pytest
import torch

from oracle.attention_oracle import attention_bwd, attention_fwd
from tests.helpers import TOL_GRAD, TOL_LSE, TOL_O, maxdiff

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _fwd_bwd(q, k, v, do, causal):
    from flash_attn_volta_b200 import check_status, flash_attn, flash_attn_forward
    qd, kd, vd = (t.clone().requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=causal)
    out.backward(do)
    _, lse = flash_attn_forward(q, k, v, causal=causal, return_softmax_lse=True)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    return out.detach(), lse, qd.grad, kd.grad, vd.grad


def test_one_cta_per_tile_matches_persistent_grid():
    # 80 x 32 = 2560 tiles (more than 16 per SM on 148 SMs): one CTA per tile
    B, S, H, D = 1, 4096, 80, 128
    g = torch.Generator().manual_seed(77)
    q, k, v, do = [(torch.randn((B, S, H, D), generator=g) * 0.5).half().to(DEV)
                   for _ in range(4)]
    full = _fwd_bwd(q, k, v, do, True)
    # an 8-head slice (256 tiles: two persistent rounds) and one head (32 tiles)
    for lo, hi in ((8, 16), (79, 80)):
        part = _fwd_bwd(*(t[:, :, lo:hi].contiguous() for t in (q, k, v, do)), True)
        o_f, lse_f, dq_f, dk_f, dv_f = full
        o_p, lse_p, dq_p, dk_p, dv_p = part
        assert torch.equal(o_f[:, :, lo:hi], o_p)
        assert torch.equal(lse_f[:, lo:hi], lse_p)
        assert torch.equal(dk_f[:, :, lo:hi], dk_p)
        assert torch.equal(dv_f[:, :, lo:hi], dv_p)
        assert maxdiff(dq_f[:, :, lo:hi].cpu(), dq_p.cpu()) <= TOL_GRAD


def test_persistent_rounds_with_empty_query_tiles_and_gqa():
    # 32 query heads x 16 query tiles = 512 forward tiles (4 rounds on 148
    # SMs); Sq > Sk with a causal mask, so query tiles 0..7 see no key
    B, Sq, Sk, H, Hkv, D = 1, 2048, 1024, 32, 8, 64
    grp = H // Hkv
    g = torch.Generator().manual_seed(78)
    q = torch.randn((B, Sq, H, D), generator=g).half()
    k = torch.randn((B, Sk, Hkv, D), generator=g).half()
    v = torch.randn((B, Sk, Hkv, D), generator=g).half()
    do = torch.randn((B, Sq, H, D), generator=g).half()
    out, lse, dq, dk, dv = _fwd_bwd(*(t.to(DEV) for t in (q, k, v, do)), True)
    scale = 1.0 / math.sqrt(D)
    off = Sk - Sq
    kh = 3  # K/V head 3 and its query heads 12..15
    hs = slice(kh * grp, (kh + 1) * grp)
    qs, dos = q[:, :, hs], do[:, :, hs]
    ke = k[:, :, kh:kh + 1].repeat_interleave(grp, dim=2)
    ve = v[:, :, kh:kh + 1].repeat_interleave(grp, dim=2)
    o_ref, lse_ref = attention_fwd(qs, ke, ve, True, scale, dtype=torch.float64,
                                   causal_offset=off)
    dq_ref, dk_ref, dv_ref = attention_bwd(dos, qs, ke, ve, True, scale, causal_offset=off)
    lse_c = lse[:, hs].cpu().double()
    inf_ref = torch.isinf(lse_ref)
    assert torch.equal(torch.isinf(lse_c), inf_ref)
    assert maxdiff(lse_c[~inf_ref], lse_ref[~inf_ref]) <= TOL_LSE
    assert maxdiff(out[:, :, hs].cpu(), o_ref) <= TOL_O
    assert maxdiff(dq[:, :, hs].cpu(), dq_ref) <= TOL_GRAD
    assert maxdiff(dk[:, :, kh:kh + 1].cpu(), dk_ref.sum(2, keepdim=True)) <= TOL_GRAD
    assert maxdiff(dv[:, :, kh:kh + 1].cpu(), dv_ref.sum(2, keepdim=True)) <= TOL_GRAD
