"""Parity at the benchmark's own workload (config 4: B=8, S=8192, H=32, D=128,
causal, fp16, q/k/v/dO ~ N(0,1)), and bit-equality of batch shards.

At this size both main kernels launch one CTA per tile (the grid `bench.py`
times), which the smaller parity shapes never reach.  The oracle is exact
(fp64) and runs one (batch, head) pair at a time on the host; eight pairs are
checked: the first and last batch crossed with the first and last head, plus
four in between.  Tolerances as everywhere: O and LSE <= 2e-3, dQ / dK / dV
<= 5e-3 max-abs.

The deterministic backward is checked at this size too (sampled heads against
the oracle, two runs bit-identical including dQ).

Batch shards: `bench.py --gpus N` gives rank r the batches [r*B/N, (r+1)*B/N)
and runs the same kernels on that slice.  O, LSE, dK and dV of a shard must
equal, bit for bit, the same batches of the single-GPU run (dQ is summed with
L2 reductions whose order varies, so it is compared within tolerance).
"""
import math

import pytest
import torch

from tests.helpers import TOL_GRAD, TOL_LSE, TOL_O, maxdiff, oracle_heads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
B, S, H, D = 8, 8192, 32, 128
HEADS = [(0, 0), (0, 31), (7, 0), (7, 31), (2, 5), (3, 17), (5, 11), (6, 26)]


def _inputs():
    """q, k, v, dO (B, S, H, D) fp16 on the GPU, per-batch seeds (bench.py's gen_shard)."""
    outs = [torch.empty((B, S, H, D), dtype=torch.float16, device=DEV) for _ in range(4)]
    for b in range(B):
        g = torch.Generator(device=DEV).manual_seed(1234 + b)
        for t in outs:
            t[b].normal_(0.0, 1.0, generator=g)
    return outs


def _fwd_bwd(q, k, v, do):
    from flash_attn_volta_b200 import check_status, flash_attn, flash_attn_forward
    qd, kd, vd = (t.detach().clone().requires_grad_() for t in (q, k, v))
    out = flash_attn(qd, kd, vd, causal=True)
    out.backward(do)
    with torch.no_grad():
        _, lse = flash_attn_forward(q, k, v, causal=True, return_softmax_lse=True)
    torch.cuda.synchronize(DEV)
    check_status(DEV)
    return out.detach(), lse, qd.grad, kd.grad, vd.grad


@pytest.fixture(scope="module")
def c4_run():
    q, k, v, do = _inputs()
    res = _fwd_bwd(q, k, v, do)
    yield (q, k, v, do), res
    del q, k, v, do, res
    torch.cuda.empty_cache()


def test_c4_sampled_heads_vs_oracle(c4_run):
    (q, k, v, do), (o, lse, dq, dk, dv) = c4_run
    scale = 1.0 / math.sqrt(D)
    worst = {"o": 0.0, "lse": 0.0, "dq": 0.0, "dk": 0.0, "dv": 0.0}
    for b, h in HEADS:
        sl = lambda t: t[b:b + 1, :, h:h + 1, :].cpu()  # noqa: E731
        ref = oracle_heads(sl(q), sl(k), sl(v), sl(do), True, scale, [(0, 0)])
        worst["o"] = max(worst["o"], maxdiff(o[b, :, h].cpu(), ref["o"][0]))
        worst["lse"] = max(worst["lse"], maxdiff(lse[b, h].cpu(), ref["lse"][0]))
        worst["dq"] = max(worst["dq"], maxdiff(dq[b, :, h].cpu(), ref["dq"][0]))
        worst["dk"] = max(worst["dk"], maxdiff(dk[b, :, h].cpu(), ref["dk"][0]))
        worst["dv"] = max(worst["dv"], maxdiff(dv[b, :, h].cpu(), ref["dv"][0]))
    assert worst["o"] <= TOL_O, worst
    assert worst["lse"] <= TOL_LSE, worst
    assert max(worst["dq"], worst["dk"], worst["dv"]) <= TOL_GRAD, worst


@pytest.mark.parametrize("n_ranks,rank", [(4, 1), (8, 7)])
def test_c4_batch_shard_bit_identical(c4_run, n_ranks, rank):
    (q, k, v, do), (o, lse, dq, dk, dv) = c4_run
    b0, b1 = rank * B // n_ranks, (rank + 1) * B // n_ranks
    sl = lambda t: t[b0:b1].contiguous()  # noqa: E731
    so, slse, sdq, sdk, sdv = _fwd_bwd(sl(q), sl(k), sl(v), sl(do))
    assert torch.equal(so, o[b0:b1])
    assert torch.equal(slse, lse[b0:b1])
    assert torch.equal(sdk, dk[b0:b1])
    assert torch.equal(sdv, dv[b0:b1])
    assert maxdiff(sdq, dq[b0:b1]) <= 1e-3


def test_c4_deterministic_vs_oracle_and_bit_identical(c4_run):
    """The deterministic backward at the benchmark size: sampled heads against
    the exact oracle, and dQ / dK / dV bit-identical over two runs (64 key
    blocks per causal query row at S=8192)."""
    from flash_attn_volta_b200 import check_status, flash_attn
    (q, k, v, do), (o, lse, dq, dk, dv) = c4_run
    runs = []
    for _ in range(2):
        qd, kd, vd = (t.detach().clone().requires_grad_() for t in (q, k, v))
        flash_attn(qd, kd, vd, causal=True, deterministic=True).backward(do)
        torch.cuda.synchronize(DEV)
        check_status(DEV)
        runs.append((qd.grad, kd.grad, vd.grad))
        del qd, kd, vd
    for a, b in zip(*runs):
        assert torch.equal(a, b)
    gq, gk, gv = runs[0]
    assert torch.equal(gk, dk) and torch.equal(gv, dv)  # dK / dV: same kernel arithmetic
    scale = 1.0 / math.sqrt(D)
    worst = 0.0
    for b, h in HEADS[:4]:
        sl = lambda t: t[b:b + 1, :, h:h + 1, :].cpu()  # noqa: E731
        ref = oracle_heads(sl(q), sl(k), sl(v), sl(do), True, scale, [(0, 0)])
        worst = max(worst, maxdiff(gq[b, :, h].cpu(), ref["dq"][0]))
    assert worst <= TOL_GRAD, worst
