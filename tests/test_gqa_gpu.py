"""Grouped-query / multi-query attention (K/V with fewer heads than Q) on the
GPU against the exact oracle: the oracle sees K/V expanded to the query heads
(what the reference's HF patches did with repeat_kv, patch_hf.py:187-188), and
dK / dV of the expanded heads summed over each K/V head's group.

Tolerances as for multi-head attention: O and LSE <= 2e-3, dQ / dK / dV <= 5e-3
max-abs (dK / dV of a group are sums of `group` heads' gradients, each within
the multi-head tolerance of its own exact value; the shapes below keep the sum
inside the same bound).
"""
import math

import pytest
import torch

from tests.helpers import TOL_GRAD, TOL_LSE, TOL_O, make_inputs, maxdiff, oracle_heads

pytestmark = pytest.mark.gpu

DEV = "cuda"

# (B, S, H, H_kv, D, causal)
SHAPES = [
    (2, 300, 8, 2, 64, True),     # ragged S, group 4
    (1, 512, 8, 1, 128, False),   # multi-query
    (1, 1024, 16, 4, 128, True),  # group 4, several key tiles per head
    (2, 256, 6, 3, 32, True),     # group 2, small head dim
    (1, 130, 4, 2, 16, False),
]


def _id(s):
    B, S, H, Hkv, D, c = s
    return f"B{B}_S{S}_H{H}_Hkv{Hkv}_D{D}_{'c' if c else 'nc'}"


@pytest.mark.parametrize("shape", SHAPES, ids=_id)
def test_gqa_fwd_bwd_vs_oracle(shape):
    from flash_attn_volta_b200 import check_status, flash_attn, flash_attn_forward
    B, S, H, Hkv, D, causal = shape
    g = H // Hkv
    q, do = make_inputs(B, S, H, D, seed=11 * S + H, n=2)
    k, v = make_inputs(B, S, Hkv, D, seed=13 * S + Hkv, n=2)
    scale = 1.0 / math.sqrt(D)

    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=causal)
    out.backward(do.to(DEV))
    _, lse = flash_attn_forward(qd.detach(), kd.detach(), vd.detach(), causal=causal,
                                return_softmax_lse=True)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    assert kd.grad.shape == k.shape and vd.grad.shape == v.shape

    ke, ve = k.repeat_interleave(g, dim=2), v.repeat_interleave(g, dim=2)
    ref = oracle_heads(q, ke, ve, do, causal, scale)
    n = B * H
    o_ref = ref["o"].reshape(B, H, S, D).permute(0, 2, 1, 3)
    lse_ref = ref["lse"].reshape(B, H, S)
    dq_ref = ref["dq"].reshape(B, H, S, D).permute(0, 2, 1, 3)
    dk_ref = ref["dk"].reshape(B, Hkv, g, S, D).sum(2).permute(0, 2, 1, 3)
    dv_ref = ref["dv"].reshape(B, Hkv, g, S, D).sum(2).permute(0, 2, 1, 3)
    assert ref["o"].shape[0] == n
    assert maxdiff(out.detach().cpu(), o_ref) <= TOL_O
    assert maxdiff(lse.cpu(), lse_ref) <= TOL_LSE
    assert maxdiff(qd.grad.cpu(), dq_ref) <= TOL_GRAD
    assert maxdiff(kd.grad.cpu(), dk_ref) <= TOL_GRAD
    assert maxdiff(vd.grad.cpu(), dv_ref) <= TOL_GRAD


def test_gqa_matches_expanded_kernel_run():
    """The grouped call and the same attention with K/V expanded to every query
    head (multi-head kernel path) agree; dK / dV are the group sums."""
    from flash_attn_volta_b200 import flash_attn
    B, S, H, Hkv, D = 2, 1000, 8, 2, 128
    g = H // Hkv
    q, do = (t.to(DEV) for t in make_inputs(B, S, H, D, seed=5, n=2))
    k, v = (t.to(DEV) for t in make_inputs(B, S, Hkv, D, seed=6, n=2))
    a = [t.clone().requires_grad_() for t in (q, k, v)]
    oa = flash_attn(*a, causal=True)
    oa.backward(do)
    ke = k.repeat_interleave(g, dim=2).detach().requires_grad_()
    ve = v.repeat_interleave(g, dim=2).detach().requires_grad_()
    qe = q.clone().requires_grad_()
    ob = flash_attn(qe, ke, ve, causal=True)
    ob.backward(do)
    torch.cuda.synchronize()
    assert maxdiff(oa.detach(), ob.detach()) == 0.0  # same arithmetic per query head
    assert maxdiff(a[0].grad, qe.grad) <= 1e-3
    dk_sum = ke.grad.float().reshape(B, S, Hkv, g, D).sum(3)
    dv_sum = ve.grad.float().reshape(B, S, Hkv, g, D).sum(3)
    assert maxdiff(a[1].grad, dk_sum) <= TOL_GRAD
    assert maxdiff(a[2].grad, dv_sum) <= TOL_GRAD
