"""The deterministic backward (FA_BWD_DETERMINISTIC / deterministic=True).

dQ comes from its own kernel that sums every query row's key blocks in a fixed
order in tensor memory, as the reference's atomics-free dQ kernel does
(flash_attn_volta/triton_fa_bwd.py:73-180), so dQ is bit-reproducible.  These
tests check it against the exact oracle (O/LSE <= 2e-3, dQ/dK/dV <= 5e-3
max-abs; bf16 with its own documented tolerance), and the two properties the
reference's tests rely on at a size with many key blocks: repeated runs give
identical bits, and the causal-leak test (tests/test_backward.py:194-234 of
the reference) holds bit for bit.
"""
import math

import pytest
import torch

from tests.helpers import TOL_GRAD, TOL_O, make_inputs, maxdiff, oracle_heads, pick_heads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)

SHAPES = [
    # (B, S, H, D, causal, amp, heads or None)
    (2, 1024, 8, 64, False, 1.0, [(0, 0), (1, 7)]),
    (4, 512, 4, 32, True, 1.0, None),
    (1, 64, 2, 64, True, 1.0, None),
    (1, 2048, 16, 128, True, 1.0, [(0, 1), (0, 15)]),
    (1, 4096, 8, 128, True, 0.5, [(0, 2), (0, 7)]),
    (2, 300, 3, 128, True, 1.0, None),
    (3, 77, 2, 32, True, 1.0, None),
    (1, 16, 2, 16, True, 1.0, None),
    (2, 130, 2, 16, False, 1.0, None),
]


def _run(q, k, v, do, causal, dtype=torch.float16):
    from flash_attn_volta_b200 import check_status, flash_attn
    qd, kd, vd = (t.to(DEV, dtype).requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=causal, deterministic=True)
    out.backward(do.to(DEV, dtype))
    torch.cuda.synchronize(DEV)
    check_status(DEV)
    return out.detach().cpu(), qd.grad.cpu(), kd.grad.cpu(), vd.grad.cpu()


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "B{}_S{}_H{}_D{}_{}".format(
    s[0], s[1], s[2], s[3], "c" if s[4] else "nc"))
def test_deterministic_fwd_bwd_vs_oracle(shape):
    B, S, H, D, causal, amp, heads = shape
    q, k, v, do = make_inputs(B, S, H, D, amp, seed=3 * S + D)
    heads = heads or [(b, h) for b in range(B) for h in range(H)]
    out, dq, dk, dv = _run(q, k, v, do, causal)
    ref = oracle_heads(q, k, v, do, causal, 1.0 / math.sqrt(D), heads)
    assert maxdiff(pick_heads(out, heads), ref["o"]) <= TOL_O
    for name, g in (("dq", dq), ("dk", dk), ("dv", dv)):
        assert maxdiff(pick_heads(g, heads), ref[name]) <= TOL_GRAD, name


def test_deterministic_gqa_bf16_and_ragged_lengths():
    """Grouped-query K/V (H=8, H_kv=2), Sq != Sk with the bottom-right mask,
    bf16: against the oracle with the bf16 tolerance (gradients 2e-2 + |ref|/128)."""
    from flash_attn_volta_b200 import check_status, flash_attn
    from oracle.attention_oracle import attention_bwd, attention_fwd
    B, Sq, Sk, H, Hkv, D = 2, 200, 333, 8, 2, 64
    g = torch.Generator().manual_seed(11)
    q = torch.randn((B, Sq, H, D), generator=g).to(torch.bfloat16)
    k = torch.randn((B, Sk, Hkv, D), generator=g).to(torch.bfloat16)
    v = torch.randn((B, Sk, Hkv, D), generator=g).to(torch.bfloat16)
    do = torch.randn((B, Sq, H, D), generator=g).to(torch.bfloat16)
    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=True, deterministic=True)
    out.backward(do.to(DEV))
    torch.cuda.synchronize(DEV)
    check_status(DEV)
    rep = H // Hkv
    ke, ve = k.repeat_interleave(rep, dim=2), v.repeat_interleave(rep, dim=2)
    o_ref, _ = attention_fwd(q, ke, ve, True, dtype=torch.float64, causal_offset=Sk - Sq)
    dq, dke, dve = attention_bwd(do, q, ke, ve, True, causal_offset=Sk - Sq)
    dk_ref = dke.view(B, Sk, Hkv, rep, D).sum(3)
    dv_ref = dve.view(B, Sk, Hkv, rep, D).sum(3)
    assert maxdiff(out.detach().cpu(), o_ref) <= 1e-2
    for got, ref in ((qd.grad, dq), (kd.grad, dk_ref), (vd.grad, dv_ref)):
        err = (got.cpu().double() - ref).abs()
        assert (err <= 2e-2 + ref.abs() / 128).all()


def test_deterministic_matches_default_mode():
    from flash_attn_volta_b200 import flash_attn
    q, k, v, do = [t.to(DEV) for t in make_inputs(2, 1000, 4, 128, seed=12)]
    res = []
    for det in (False, True):
        qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
        flash_attn(qq, kk, vv, causal=True, deterministic=det).backward(do)
        res.append((qq.grad, kk.grad, vv.grad))
    assert torch.equal(res[0][1], res[1][1]) and torch.equal(res[0][2], res[1][2])
    assert maxdiff(res[0][0], res[1][0]) <= 1e-3


def test_deterministic_repeated_runs_bit_identical():
    """dQ included: 16 key blocks per query row at S=2048."""
    from flash_attn_volta_b200 import flash_attn
    q, k, v, do = [t.to(DEV) for t in make_inputs(2, 2048, 8, 128, seed=31)]
    ref = None
    for _ in range(6):
        qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
        flash_attn(qq, kk, vv, causal=True, deterministic=True).backward(do)
        cur = (qq.grad, kk.grad, vv.grad)
        if ref is None:
            ref = cur
        else:
            for a, b in zip(ref, cur):
                assert torch.equal(a, b)


def test_deterministic_causal_no_leak_bit_identical_many_blocks():
    """The reference's causal-leak test at N=1024, H=4, D=128 (eight key blocks
    of 128 rows): dQ of rows < N/2 must not change, bit for bit, when the K / V
    rows >= N/2 are perturbed."""
    from flash_attn_volta_b200 import flash_attn
    B, N, H, D = 1, 1024, 4, 128
    q, k, v, do = make_inputs(B, N, H, D, seed=0)
    g = torch.Generator().manual_seed(1)
    j = N // 2
    kp, vp = k.clone(), v.clone()
    kp[:, j:] += (torch.randn(kp[:, j:].shape, generator=g) * 0.5).half()
    vp[:, j:] += (torch.randn(vp[:, j:].shape, generator=g) * 0.5).half()
    grads = []
    for kk, vv in ((k, v), (kp, vp)):
        qd = q.to(DEV).requires_grad_()
        out = flash_attn(qd, kk.to(DEV).requires_grad_(), vv.to(DEV).requires_grad_(),
                         causal=True, deterministic=True)
        out.backward(do.to(DEV))
        grads.append(qd.grad.cpu())
    assert (grads[0][:, :j] - grads[1][:, :j]).abs().max().item() == 0.0
    assert (grads[0][:, j:] - grads[1][:, j:]).abs().max().item() > 1e-3


def test_deterministic_fully_masked_rows():
    """Sq > Sk with the bottom-right causal mask: the first Sq - Sk query rows see
    no key (O = 0, LSE = +inf, dQ = 0), whole 128-row query tiles among them
    (the dQ kernel writes those tiles' zeros without any key block)."""
    from flash_attn_volta_b200 import check_status, flash_attn
    from oracle.attention_oracle import attention_bwd, attention_fwd
    B, Sq, Sk, H, D = 1, 700, 200, 2, 64
    g = torch.Generator().manual_seed(13)
    q = torch.randn((B, Sq, H, D), generator=g).half()
    k = torch.randn((B, Sk, H, D), generator=g).half()
    v = torch.randn((B, Sk, H, D), generator=g).half()
    do = torch.randn((B, Sq, H, D), generator=g).half()
    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=True, deterministic=True)
    out.backward(do.to(DEV))
    torch.cuda.synchronize(DEV)
    check_status(DEV)
    o_ref, _ = attention_fwd(q, k, v, True, dtype=torch.float64, causal_offset=Sk - Sq)
    dq, dk, dv = attention_bwd(do, q, k, v, True, causal_offset=Sk - Sq)
    assert (qd.grad[:, :Sq - Sk] == 0).all() and (out[:, :Sq - Sk] == 0).all()
    assert maxdiff(out.detach().cpu(), o_ref) <= TOL_O
    for got, ref in ((qd.grad, dq), (kd.grad, dk), (vd.grad, dv)):
        assert maxdiff(got.cpu(), ref) <= TOL_GRAD
