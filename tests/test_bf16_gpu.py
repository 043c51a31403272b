"""bf16 inputs and outputs on the GPU against the exact oracle evaluated on the
same bf16-rounded inputs.

bf16 keeps 8 mantissa bits (fp16: 11), so rounding P, dS and the outputs costs
about 4x the fp16 error.  Tolerances: O 1e-2 and LSE 2e-3 max-abs (the LSE comes
from fp32 scores); dQ / dK / dV |err| <= 2e-2 + |ref| / 128 element-wise, the
relative part being two bf16 units of the output (grouped-query dK / dV are sums
over the group and larger).  The reference is fp16-only; bf16 is an extension
of the same API.
"""
import math

import pytest
import torch

from tests.helpers import maxdiff, oracle_heads

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL_O_BF16, TOL_LSE_BF16, TOL_GRAD_BF16, RTOL_GRAD_BF16 = 1e-2, 2e-3, 2e-2, 1.0 / 128


def excess(got, ref):
    """max of |got - ref| - |ref| / 128: the gradient error beyond bf16's relative part."""
    got, ref = got.double(), ref.double()
    return float(((got - ref).abs() - RTOL_GRAD_BF16 * ref.abs()).max())

# (B, S, H, H_kv, D, causal)
SHAPES = [
    (1, 1024, 8, 8, 128, True),
    (2, 300, 4, 4, 64, False),
    (1, 512, 8, 2, 128, True),   # grouped-query, bf16
    (1, 256, 2, 2, 32, True),
    (1, 130, 2, 2, 16, False),
]


def _id(s):
    B, S, H, Hkv, D, c = s
    return f"B{B}_S{S}_H{H}_Hkv{Hkv}_D{D}_{'c' if c else 'nc'}"


def _inputs(B, S, H, Hkv, D, seed):
    g = torch.Generator().manual_seed(seed)
    mk = lambda h: torch.randn((B, S, h, D), generator=g).to(torch.bfloat16)  # noqa: E731
    return mk(H), mk(Hkv), mk(Hkv), mk(H)


@pytest.mark.parametrize("shape", SHAPES, ids=_id)
def test_bf16_fwd_bwd_vs_oracle(shape):
    from flash_attn_volta_b200 import check_status, flash_attn, flash_attn_forward
    B, S, H, Hkv, D, causal = shape
    grp = H // Hkv
    q, k, v, do = _inputs(B, S, H, Hkv, D, seed=3 * S + D)
    scale = 1.0 / math.sqrt(D)
    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=causal)
    assert out.dtype == torch.bfloat16
    out.backward(do.to(DEV))
    _, lse = flash_attn_forward(qd.detach(), kd.detach(), vd.detach(), causal=causal,
                                return_softmax_lse=True)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    assert qd.grad.dtype == kd.grad.dtype == torch.bfloat16

    ke, ve = k.repeat_interleave(grp, dim=2), v.repeat_interleave(grp, dim=2)
    ref = oracle_heads(q.float(), ke.float(), ve.float(), do.float(), causal, scale)
    o_ref = ref["o"].reshape(B, H, S, D).permute(0, 2, 1, 3)
    dq_ref = ref["dq"].reshape(B, H, S, D).permute(0, 2, 1, 3)
    dk_ref = ref["dk"].reshape(B, Hkv, grp, S, D).sum(2).permute(0, 2, 1, 3)
    dv_ref = ref["dv"].reshape(B, Hkv, grp, S, D).sum(2).permute(0, 2, 1, 3)
    errs = {
        "o": maxdiff(out.detach().cpu(), o_ref),
        "lse": maxdiff(lse.cpu(), ref["lse"].reshape(B, H, S)),
        "dq": excess(qd.grad.cpu(), dq_ref),
        "dk": excess(kd.grad.cpu(), dk_ref),
        "dv": excess(vd.grad.cpu(), dv_ref),
    }
    assert errs["o"] <= TOL_O_BF16, errs
    assert errs["lse"] <= TOL_LSE_BF16, errs
    assert max(errs["dq"], errs["dk"], errs["dv"]) <= TOL_GRAD_BF16, errs


def test_bf16_and_fp16_paths_agree():
    """Inputs exactly representable in both formats: the two element types give
    the same attention up to their output rounding."""
    from flash_attn_volta_b200 import flash_attn_forward
    g = torch.Generator().manual_seed(9)
    # multiples of 1/64 in [-2, 2]: exact in fp16 and bf16
    q, k, v = ((torch.randint(-128, 129, (1, 512, 4, 64), generator=g) / 64.0) for _ in range(3))
    o16, l16 = flash_attn_forward(*(t.to(DEV, torch.float16) for t in (q, k, v)), causal=True,
                                  return_softmax_lse=True)
    ob, lb = flash_attn_forward(*(t.to(DEV, torch.bfloat16) for t in (q, k, v)), causal=True,
                                return_softmax_lse=True)
    torch.cuda.synchronize()
    assert maxdiff(o16.float(), ob.float()) <= TOL_O_BF16
    assert maxdiff(l16, lb) <= 1e-4
