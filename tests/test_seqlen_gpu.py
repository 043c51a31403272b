"""Query and key sequences of different lengths (Sq != Sk) on the GPU against
the exact oracle.  The reference is square-only; the extension aligns the
causal mask to the bottom-right (query i sees keys j <= i + Sk - Sq, the
reference's top-left mask when Sq == Sk); a query row that sees no key gets
O = 0 and LSE = +inf, the reference's convention for fully masked rows.

Tolerances as for square attention: O and LSE <= 2e-3, dQ / dK / dV <= 5e-3
max-abs (fp16).
"""
import math

import pytest
import torch

from oracle.attention_oracle import attention_bwd, attention_fwd
from tests.helpers import TOL_GRAD, TOL_LSE, TOL_O, maxdiff

pytestmark = pytest.mark.gpu

DEV = "cuda"

# (B, Sq, Sk, H, H_kv, D, causal)
SHAPES = [
    (1, 256, 1024, 4, 4, 128, True),   # prefill after 768 cached keys
    (2, 300, 170, 4, 2, 64, True),     # Sq > Sk: the first 130 rows see no key
    (1, 100, 600, 2, 2, 32, False),
    (1, 1, 513, 4, 1, 128, True),      # one decode row, multi-query
    (1, 700, 200, 2, 2, 16, True),     # whole query tiles without a visible key
]


def _id(s):
    B, Sq, Sk, H, Hkv, D, c = s
    return f"B{B}_Sq{Sq}_Sk{Sk}_H{H}_Hkv{Hkv}_D{D}_{'c' if c else 'nc'}"


@pytest.mark.parametrize("shape", SHAPES, ids=_id)
def test_sq_ne_sk_vs_oracle(shape):
    from flash_attn_volta_b200 import check_status, flash_attn, flash_attn_forward
    B, Sq, Sk, H, Hkv, D, causal = shape
    grp = H // Hkv
    g = torch.Generator().manual_seed(Sq * 7 + Sk)
    q = torch.randn((B, Sq, H, D), generator=g).half()
    k = torch.randn((B, Sk, Hkv, D), generator=g).half()
    v = torch.randn((B, Sk, Hkv, D), generator=g).half()
    do = torch.randn((B, Sq, H, D), generator=g).half()
    scale = 1.0 / math.sqrt(D)
    off = Sk - Sq

    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=causal)
    out.backward(do.to(DEV))
    _, lse = flash_attn_forward(qd.detach(), kd.detach(), vd.detach(), causal=causal,
                                return_softmax_lse=True)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    assert out.shape == q.shape and lse.shape == (B, H, Sq)
    assert kd.grad.shape == k.shape and vd.grad.shape == v.shape

    ke, ve = k.repeat_interleave(grp, dim=2), v.repeat_interleave(grp, dim=2)
    o_ref, lse_ref = attention_fwd(q, ke, ve, causal, scale, dtype=torch.float64,
                                   causal_offset=off)
    dq_ref, dk_ref, dv_ref = attention_bwd(do, q, ke, ve, causal, scale, causal_offset=off)
    dk_ref = dk_ref.reshape(B, Sk, Hkv, grp, D).sum(3)
    dv_ref = dv_ref.reshape(B, Sk, Hkv, grp, D).sum(3)

    lse_c = lse.cpu().double()
    inf_ref = torch.isinf(lse_ref)
    assert torch.equal(torch.isinf(lse_c), inf_ref)
    assert maxdiff(lse_c[~inf_ref], lse_ref[~inf_ref]) <= TOL_LSE if (~inf_ref).any() else True
    assert maxdiff(out.detach().cpu(), o_ref) <= TOL_O
    assert maxdiff(qd.grad.cpu(), dq_ref) <= TOL_GRAD
    assert maxdiff(kd.grad.cpu(), dk_ref) <= TOL_GRAD
    assert maxdiff(vd.grad.cpu(), dv_ref) <= TOL_GRAD
