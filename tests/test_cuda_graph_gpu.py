"""Capture of forward + backward in a CUDA graph.

The operators are capturable: their TMA tensor maps travel as kernel
parameters (copied into the graph at capture), the backward's workspace comes
from torch's caching allocator (the graph's private pool during capture), and
the status word exists before capture (created by the warm-up call).  The
replayed graph must give exactly the eager results, on new inputs copied into
the captured (static) tensors, several times in a row.
"""
import pytest
import torch

from tests.helpers import make_inputs

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("deterministic", [False, True])
def test_graph_replay_matches_eager(deterministic):
    from flash_attn_volta_b200 import check_status, flash_attn
    B, S, H, D = 2, 640, 4, 64
    static = [t.to(DEV) for t in make_inputs(B, S, H, D, seed=40)]
    q, k, v = (t.requires_grad_() for t in static[:3])
    do = static[3]

    def step():
        out = flash_attn(q, k, v, causal=True, deterministic=deterministic)
        out.backward(do)
        return out

    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        for _ in range(3):
            q.grad = k.grad = v.grad = None
            step()
    torch.cuda.current_stream(DEV).wait_stream(side)
    q.grad = k.grad = v.grad = None

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        static_out = step()
    for seed in (41, 42, 43):
        new = [t.to(DEV) for t in make_inputs(B, S, H, D, seed=seed)]
        with torch.no_grad():
            for dst, src in zip((q, k, v, do), new):
                dst.copy_(src)
        g.replay()
        torch.cuda.synchronize(DEV)
        check_status(DEV)
        qe, ke, ve = (t.clone().requires_grad_() for t in new[:3])
        oe = flash_attn(qe, ke, ve, causal=True, deterministic=deterministic)
        oe.backward(new[3])
        assert torch.equal(static_out, oe.detach())
        assert torch.equal(k.grad, ke.grad) and torch.equal(v.grad, ve.grad)
        if deterministic:
            assert torch.equal(q.grad, qe.grad)
        else:
            assert float((q.grad.float() - qe.grad.float()).abs().max()) <= 1e-3
