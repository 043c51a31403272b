"""CPU tests of the oracle: pinned to the reference through tests/golden/*.npz."""
import math

import pytest
import torch

from oracle.attention_oracle import (attention_bwd, attention_fwd, attention_fwd_tiled,
                                     attention_rows, flops_fwd, flops_fwdbwd)
from tests.helpers import golden_cases, load_golden, make_inputs, maxdiff

CASES = golden_cases()


def test_golden_fixtures_present():
    assert len(CASES) >= 8


@pytest.mark.parametrize("path", CASES, ids=lambda p: p.split("/")[-1][:-4])
def test_oracle_matches_reference_eager(path):
    """Oracle forward == ref.py attention_ref (fp32) on the reference's own output."""
    g = load_golden(path)
    o, _ = attention_fwd(g["q"], g["k"], g["v"], g["causal"], g["scale"])
    assert maxdiff(o, g["o_eager"]) < 2e-6


@pytest.mark.parametrize("path", CASES, ids=lambda p: p.split("/")[-1][:-4])
def test_oracle_matches_reference_kernels(path):
    """Oracle vs the reference's Triton kernels (run in interpreter mode).

    The reference rounds Q*scale to fp16 and P / dS to fp16, so the bound is
    its own published accuracy (fwd <= 1.95e-3, grads <= 3.06e-3 vs fp64),
    not bit equality.
    """
    g = load_golden(path)
    o, lse = attention_fwd(g["q"], g["k"], g["v"], g["causal"], g["scale"], dtype=torch.float64)
    assert maxdiff(o, g["o_ref"].float()) < 2e-3
    assert maxdiff(lse, g["lse_ref"]) < 2e-3
    dq, dk, dv = attention_bwd(g["do"], g["q"], g["k"], g["v"], g["causal"], g["scale"])
    assert maxdiff(dq, g["dq_ref"].float()) < 5e-3
    assert maxdiff(dk, g["dk_ref"].float()) < 5e-3
    assert maxdiff(dv, g["dv_ref"].float()) < 5e-3


@pytest.mark.parametrize("causal", [False, True])
def test_tiled_recurrence_equals_exact(causal):
    q, k, v = make_inputs(2, 150, 3, 32, seed=3, n=3)
    o1, l1 = attention_fwd(q, k, v, causal)
    o2, l2 = attention_fwd_tiled(q, k, v, causal, block_n=64)
    assert maxdiff(o1, o2) < 1e-5
    assert maxdiff(l1, l2) < 1e-5


@pytest.mark.parametrize("causal", [False, True])
def test_analytic_backward_equals_autograd(causal):
    q, k, v, do = make_inputs(1, 40, 2, 16, seed=4)
    leaves = [t.double().requires_grad_() for t in (q, k, v)]
    o, _ = attention_fwd(*leaves, causal=causal, dtype=torch.float64)
    o.backward(do.double())
    dq, dk, dv = attention_bwd(do, q, k, v, causal)
    for a, b in zip((dq, dk, dv), leaves):
        assert maxdiff(a, b.grad) < 1e-10


def test_fully_masked_row_lse_is_inf():
    # With a bottom-right causal mask and fewer keys than queries
    # (causal_offset = Sk - Sq < 0) the first Sq - Sk query rows see no key:
    # the reference's convention (triton_fa.py:152-159) is O = 0, LSE = +inf.
    q, _, _ = make_inputs(1, 8, 2, 16, seed=5, n=3)
    _, k, v = make_inputs(1, 5, 2, 16, seed=6, n=3)
    o, lse = attention_fwd(q, k, v, causal=True, causal_offset=5 - 8, dtype=torch.float64)
    assert torch.isposinf(lse[:, :, :3]).all()
    assert torch.isfinite(lse[:, :, 3:]).all()
    assert (o[:, :3] == 0).all()
    # an empty sequence gives an empty LSE in the tiled recurrence
    _, lse_t = attention_fwd_tiled(q[:, :0], k[:, :0], v[:, :0])
    assert lse_t.numel() == 0


def test_rows_oracle_matches_full():
    q, k, v, do = make_inputs(1, 96, 2, 32, seed=6)
    rows = [0, 5, 50, 95]
    o, lse = attention_fwd(q, k, v, True, dtype=torch.float64)
    dq, _, _ = attention_bwd(do, q, k, v, True)
    o_r, lse_r, dq_r = attention_rows(q, k, v, 0, 1, rows, causal=True, do=do)
    assert maxdiff(o_r, o[0, rows, 1]) < 1e-12
    assert maxdiff(lse_r, lse[0, 1, rows]) < 1e-12
    assert maxdiff(dq_r, dq[0, rows, 1]) < 1e-12


def test_flop_formulas():
    # values of the benchmark convention: 4*B*H*S^2*D, /2 causal, fwd+bwd = 2.5x
    assert flops_fwd(2, 1024, 8, 64, False) == pytest.approx(4.295e9, rel=1e-3)
    assert flops_fwdbwd(1, 4096, 8, 128, True) == pytest.approx(8.590e10, rel=1e-3)
    assert flops_fwdbwd(8, 8192, 32, 128, True) == pytest.approx(1.100e13, rel=1e-3)
