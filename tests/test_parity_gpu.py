"""GPU parity of the sm_100a kernels with the CPU oracle (and the golden
fixtures made by the reference itself).

Tolerances (max-abs, against the exact oracle in fp64):
  O and LSE <= 2e-3, dQ / dK / dV <= 5e-3.
Inputs are generated on the CPU generator so the oracle and the GPU see the
same fp16 tensors.
"""
import math

import pytest
import torch

from tests.helpers import (TOL_GRAD, TOL_LSE, TOL_O, golden_cases, load_golden, make_inputs,
                           maxdiff, oracle_heads, pick_heads)

pytestmark = pytest.mark.gpu

DEV = "cuda"

# (B, S, H, D, causal, amp, heads-to-check or None = all)
SHAPES = [
    (2, 1024, 8, 64, False, 1.0, [(0, 0), (1, 7), (1, 3)]),     # config 1
    (4, 512, 4, 32, False, 1.0, None),                         # config 2
    (4, 512, 4, 32, True, 1.0, None),                          # config 2
    (1, 64, 2, 64, False, 1.0, None),
    (1, 64, 2, 64, True, 1.0, None),
    (1, 2048, 16, 128, False, 1.0, [(0, 0), (0, 9)]),
    (1, 2048, 16, 128, True, 1.0, [(0, 1), (0, 15)]),
    (1, 4096, 16, 64, True, 0.5, [(0, 0), (0, 11)]),            # config 3a
    (1, 4096, 8, 128, True, 0.5, [(0, 2), (0, 7)]),             # config 3b
    (2, 300, 3, 128, True, 1.0, None),                          # ragged S
    (1, 200, 2, 64, False, 1.0, None),
    (3, 77, 2, 32, True, 1.0, None),
    (1, 16, 2, 16, True, 1.0, None),
    (2, 130, 2, 16, False, 1.0, None),
]


def _id(s):
    B, S, H, D, c, a, _ = s
    return f"B{B}_S{S}_H{H}_D{D}_{'c' if c else 'nc'}"


def _run(q, k, v, do, causal):
    from flash_attn_volta_b200 import flash_attn, check_status
    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=causal)
    out.backward(do.to(DEV))
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    return out.detach().cpu(), qd.grad.cpu(), kd.grad.cpu(), vd.grad.cpu()


@pytest.mark.parametrize("shape", SHAPES, ids=_id)
def test_fwd_lse_vs_oracle(shape):
    from flash_attn_volta_b200 import flash_attn_forward, check_status
    B, S, H, D, causal, amp, heads = shape
    q, k, v = make_inputs(B, S, H, D, amp, seed=S + D, n=3)
    heads = heads or [(b, h) for b in range(B) for h in range(H)]
    out, lse = flash_attn_forward(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal,
                                  return_softmax_lse=True)
    torch.cuda.synchronize()
    check_status(torch.device(DEV))
    assert out.shape == (B, S, H, D) and out.dtype == torch.float16 and out.is_contiguous()
    assert lse.shape == (B, H, S) and lse.dtype == torch.float32
    ref = oracle_heads(q, k, v, None, causal, 1.0 / math.sqrt(D), heads, grads=False)
    assert maxdiff(pick_heads(out.cpu(), heads), ref["o"]) <= TOL_O
    assert maxdiff(pick_heads(lse.cpu(), heads), ref["lse"]) <= TOL_LSE


@pytest.mark.parametrize("shape", SHAPES, ids=_id)
def test_fwd_bwd_vs_oracle(shape):
    B, S, H, D, causal, amp, heads = shape
    q, k, v, do = make_inputs(B, S, H, D, amp, seed=7 * S + D)
    heads = heads or [(b, h) for b in range(B) for h in range(H)]
    out, dq, dk, dv = _run(q, k, v, do, causal)
    ref = oracle_heads(q, k, v, do, causal, 1.0 / math.sqrt(D), heads)
    errs = {
        "o": maxdiff(pick_heads(out, heads), ref["o"]),
        "dq": maxdiff(pick_heads(dq, heads), ref["dq"]),
        "dk": maxdiff(pick_heads(dk, heads), ref["dk"]),
        "dv": maxdiff(pick_heads(dv, heads), ref["dv"]),
    }
    assert errs["o"] <= TOL_O, errs
    assert errs["dq"] <= TOL_GRAD, errs
    assert errs["dk"] <= TOL_GRAD, errs
    assert errs["dv"] <= TOL_GRAD, errs


@pytest.mark.parametrize("path", golden_cases(), ids=lambda p: p.split("/")[-1][:-4])
def test_golden_reference_fixtures(path):
    """Same inputs the reference's own kernels saw: we must be at least as close
    to the exact answer as the tolerance, and close to the reference's output."""
    g = load_golden(path)
    out, dq, dk, dv = _run(g["q"], g["k"], g["v"], g["do"], g["causal"])
    from flash_attn_volta_b200 import flash_attn_forward
    _, lse = flash_attn_forward(g["q"].to(DEV), g["k"].to(DEV), g["v"].to(DEV),
                                causal=g["causal"], return_softmax_lse=True)
    assert maxdiff(out, g["o_eager"]) <= TOL_O
    assert maxdiff(out, g["o_ref"]) <= 2 * TOL_O
    assert maxdiff(lse.cpu(), g["lse_ref"]) <= TOL_LSE
    assert maxdiff(dq, g["dq_ref"]) <= 2 * TOL_GRAD
    assert maxdiff(dk, g["dk_ref"]) <= 2 * TOL_GRAD
    assert maxdiff(dv, g["dv_ref"]) <= 2 * TOL_GRAD


def test_causal_no_leak_bit_identical():
    """tests/test_backward.py:194-234 of the reference: dQ of rows < N/2 must not
    change (bit for bit) when K, V rows >= N/2 are perturbed."""
    from flash_attn_volta_b200 import flash_attn
    B, N, H, D = 1, 64, 2, 64
    q, k, v, do = make_inputs(B, N, H, D, seed=0)
    g = torch.Generator().manual_seed(1)
    j = N // 2
    kp, vp = k.clone(), v.clone()
    kp[:, j:] += (torch.randn(kp[:, j:].shape, generator=g) * 0.5).half()
    vp[:, j:] += (torch.randn(vp[:, j:].shape, generator=g) * 0.5).half()
    grads = []
    for kk, vv in ((k, v), (kp, vp)):
        qd = q.to(DEV).requires_grad_()
        out = flash_attn(qd, kk.to(DEV).requires_grad_(), vv.to(DEV).requires_grad_(), causal=True)
        out.backward(do.to(DEV))
        grads.append(qd.grad.cpu())
    assert (grads[0][:, :j] - grads[1][:, :j]).abs().max().item() == 0.0
    assert (grads[0][:, j:] - grads[1][:, j:]).abs().max().item() > 1e-3


def test_finite_difference_gradcheck():
    """tests/test_backward.py:96-191 of the reference: central differences of an
    fp64 loss vs the kernel's analytical gradient on 8 coordinates per tensor."""
    from flash_attn_volta_b200 import flash_attn
    from oracle.attention_oracle import attention_fwd
    B, N, H, D = 1, 16, 2, 32
    q, k, v, gt = make_inputs(B, N, H, D, seed=2)
    qd, kd, vd = (t.to(DEV).requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=True)
    (out.float() * gt.to(DEV).float()).sum().backward()
    ana = [t.grad.cpu().double() for t in (qd, kd, vd)]
    base = [t.double() for t in (q, k, v)]
    h = 1e-4

    def loss(ts):
        o, _ = attention_fwd(*ts, causal=True, dtype=torch.float64)
        return float((o * gt.double()).sum())

    g = torch.Generator().manual_seed(42)
    worst = 0.0
    for i in range(3):
        for idx in torch.randperm(base[i].numel(), generator=g)[:8].tolist():
            tp = [t.clone() for t in base]
            tm = [t.clone() for t in base]
            tp[i].view(-1)[idx] += h
            tm[i].view(-1)[idx] -= h
            fd = (loss(tp) - loss(tm)) / (2 * h)
            worst = max(worst, abs(fd - float(ana[i].view(-1)[idx])))
    assert worst < 5e-3


@pytest.mark.parametrize("shape,causal", [((1, 4096, 16, 64), False), ((1, 4096, 16, 64), True),
                                          ((1, 4096, 8, 128), False), ((1, 8192, 4, 64), False),
                                          ((1, 8192, 4, 64), True)])
def test_stability_no_nan_inf(shape, causal):
    """bench/stability.py:16-31 of the reference: 0.5-scaled inputs, no NaN/Inf."""
    from flash_attn_volta_b200 import flash_attn
    q, k, v, do = [t.to(DEV) for t in make_inputs(*shape, amp=0.5, seed=9)]
    q.requires_grad_(); k.requires_grad_(); v.requires_grad_()
    out = flash_attn(q, k, v, causal=causal)
    out.backward(do)
    for t in (out, q.grad, k.grad, v.grad):
        assert torch.isfinite(t).all()


def test_forward_deterministic():
    from flash_attn_volta_b200 import flash_attn_forward
    q, k, v = [t.to(DEV) for t in make_inputs(2, 777, 4, 64, seed=5, n=3)]
    o1, l1 = flash_attn_forward(q, k, v, causal=True, return_softmax_lse=True)
    o2, l2 = flash_attn_forward(q, k, v, causal=True, return_softmax_lse=True)
    assert torch.equal(o1, o2) and torch.equal(l1, l2)


def test_noncontiguous_and_dtype_cast_inputs():
    """Views are made contiguous by the shim; a float32 upstream grad is cast
    to fp16 like autograd.py:37-39 of the reference."""
    from flash_attn_volta_b200 import flash_attn
    B, S, H, D = 2, 128, 4, 64
    q, k, v, do = make_inputs(B, S, H, D, seed=8)
    qt = q.permute(0, 2, 1, 3).contiguous().to(DEV).permute(0, 2, 1, 3).requires_grad_()
    out = flash_attn(qt, k.to(DEV), v.to(DEV))
    out.backward(do.to(DEV).float())
    ref = oracle_heads(q, k, v, do, False, 1 / 8.0, [(0, 0), (1, 3)])
    assert maxdiff(pick_heads(out.detach().cpu(), [(0, 0), (1, 3)]), ref["o"]) <= TOL_O
    assert maxdiff(pick_heads(qt.grad.cpu(), [(0, 0), (1, 3)]), ref["dq"]) <= TOL_GRAD


def test_empty_sequence():
    from flash_attn_volta_b200 import flash_attn_forward, flash_attn_backward
    q = torch.zeros(2, 0, 3, 64, dtype=torch.float16, device=DEV)
    o, lse = flash_attn_forward(q, q, q, return_softmax_lse=True)
    assert o.shape == q.shape and lse.shape == (2, 3, 0)
    dq, dk, dv = flash_attn_backward(q, q, q, q, o, lse)
    assert dq.shape == q.shape


@pytest.mark.parametrize("deterministic", [False, True])
def test_empty_batch_and_no_keys(deterministic):
    """B = 0 gives empty outputs; N_k = 0 keys with N_q > 0 queries makes every
    row fully masked: O = 0, LSE = +inf (the reference's convention) and zero
    gradients, without a kernel launch reading empty tensors."""
    from flash_attn_volta_b200 import flash_attn, flash_attn_backward, flash_attn_forward
    q0 = torch.zeros(0, 64, 2, 64, dtype=torch.float16, device=DEV)
    o0, lse0 = flash_attn_forward(q0, q0, q0, causal=True, return_softmax_lse=True)
    assert o0.shape == q0.shape and lse0.shape == (0, 2, 64)
    g = flash_attn_backward(q0, q0, q0, q0, o0, lse0, causal=True, deterministic=deterministic)
    assert all(t.shape == q0.shape for t in g)
    q = torch.randn(2, 40, 4, 32, dtype=torch.float16, device=DEV).requires_grad_()
    kv = torch.zeros(2, 0, 2, 32, dtype=torch.float16, device=DEV)
    k, v = kv.clone().requires_grad_(), kv.clone().requires_grad_()
    o, lse = flash_attn_forward(q.detach(), kv, kv, return_softmax_lse=True)
    assert (o == 0).all() and torch.isposinf(lse).all()
    out = flash_attn(q, k, v, deterministic=deterministic)
    out.backward(torch.ones_like(out))
    torch.cuda.synchronize(DEV)
    assert (out == 0).all() and (q.grad == 0).all()
    assert k.grad.shape == kv.shape and v.grad.shape == kv.shape


def test_largest_batch_times_heads():
    """B * H = 65535, the most the library accepts (a grid dimension of the
    backward's prep / conversion kernels): fwd + bwd against the oracle on
    sampled (b, h); one more raises instead of launching."""
    from flash_attn_volta_b200 import flash_attn
    B, S, H, D = 13107, 24, 5, 16  # 13107 * 5 = 65535
    q, k, v, do = make_inputs(B, S, H, D, seed=8)
    leaves = [t.to(DEV).requires_grad_() for t in (q, k, v)]
    out = flash_attn(*leaves, causal=True)
    out.backward(do.to(DEV))
    torch.cuda.synchronize(DEV)
    heads = [(0, 0), (6553, 2), (B - 1, H - 1)]
    ref = oracle_heads(q, k, v, do, True, 1 / math.sqrt(D), heads)
    assert maxdiff(pick_heads(out.detach().cpu(), heads), ref["o"]) <= TOL_O
    for g, n in zip(leaves, ("dq", "dk", "dv")):
        assert maxdiff(pick_heads(g.grad.cpu(), heads), ref[n]) <= TOL_GRAD
    big = torch.zeros(65536, 8, 1, 16, dtype=torch.float16, device=DEV)
    with pytest.raises(RuntimeError):
        flash_attn(big, big, big)


@pytest.mark.parametrize("causal", [False, True])
def test_repeated_runs_bit_identical(causal):
    """Intermittent ordering bugs show up as run-to-run differences: the forward
    (O, LSE) and dK / dV (no atomics) must be bit-identical across runs."""
    from flash_attn_volta_b200 import flash_attn, flash_attn_forward
    q, k, v, do = [t.to(DEV) for t in make_inputs(2, 1024, 8, 64, seed=31)]
    ref = None
    for _ in range(8):
        o, lse = flash_attn_forward(q, k, v, causal=causal, return_softmax_lse=True)
        kk, vv = k.clone().requires_grad_(), v.clone().requires_grad_()
        flash_attn(q, kk, vv, causal=causal).backward(do)
        cur = (o, lse, kk.grad, vv.grad)
        if ref is None:
            ref = cur
        else:
            for a, b in zip(ref, cur):
                assert torch.equal(a, b)
