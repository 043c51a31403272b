"""Ring context-parallel attention with the real kernels.

One GPU: a ring of one rank still splits the sequence into two zigzag chunks
and merges three blocks (two causal, one full) — compared with the unsharded
kernel and the oracle.  Two GPUs (when present): NCCL ranks as child
processes, compared with the unsharded oracle.
"""
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_attn_volta_b200 import flash_attn, ring
from tests.helpers import TOL_GRAD, TOL_O, make_inputs, maxdiff, oracle_heads, pick_heads

pytestmark = pytest.mark.gpu


def test_ring_one_rank_matches_kernel_and_oracle():
    dev = torch.device("cuda", 0)
    B, S, H, D = 1, 2048, 4, 128
    q, k, v, do = make_inputs(B, S, H, D, seed=11)
    leaves = [t.to(dev).requires_grad_() for t in (q, k, v)]
    o = ring.ring_flash_attn(*leaves, causal=True)
    o.backward(do.to(dev))
    heads = [(0, 0), (0, 3)]
    ref = oracle_heads(q, k, v, do, True, 1 / math.sqrt(D), heads)
    assert maxdiff(pick_heads(o.detach().cpu(), heads), ref["o"]) <= TOL_O
    for g, n in zip(leaves, ("dq", "dk", "dv")):
        assert maxdiff(pick_heads(g.grad.cpu(), heads), ref[n]) <= TOL_GRAD
    full = flash_attn(*(t.to(dev) for t in (q, k, v)), causal=True)
    assert maxdiff(o.detach(), full) <= TOL_O


@pytest.mark.parametrize("hkv,dtype", [(2, torch.float16), (1, torch.bfloat16), (8, torch.bfloat16)])
def test_ring_one_rank_gqa_and_bf16(hkv, dtype):
    """Grouped-query (H_kv=2) and multi-query (H_kv=1) K/V and bf16 through the
    ring, against the unsharded kernel on the same tensors (gradients of K/V
    summed over each group by the kernels)."""
    dev = torch.device("cuda", 0)
    B, S, H, D = 2, 1536, 8, 64
    g = torch.Generator(device=dev).manual_seed(30 + hkv)
    q, do = (torch.randn((B, S, H, D), device=dev, generator=g).to(dtype) for _ in range(2))
    k, v = (torch.randn((B, S, hkv, D), device=dev, generator=g).to(dtype) for _ in range(2))
    # fp16: the parity tolerances; bf16 (8 mantissa bits, both sides rounded on
    # different paths): 1e-2 on O, 2e-2 + |x|/64 on the gradients
    bf16 = dtype == torch.bfloat16

    def close(a, b, tol):
        err = (a.double() - b.double()).abs()
        return bool((err <= tol + (b.double().abs() / 64 if bf16 else 0)).all())

    res = []
    for fn in (ring.ring_flash_attn, flash_attn):
        leaves = [t.clone().requires_grad_() for t in (q, k, v)]
        o = fn(*leaves, causal=True)
        o.backward(do)
        res.append((o.detach(),) + tuple(t.grad for t in leaves))
    torch.cuda.synchronize(dev)
    assert res[0][2].shape == (B, S, hkv, D)
    assert close(res[0][0], res[1][0], 1e-2 if bf16 else TOL_O)
    for a, b in zip(res[0][1:], res[1][1:]):
        assert close(a, b, 2e-2 if bf16 else TOL_GRAD)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_merge_kernel_matches_eager_merge(dtype):
    """fa_sm100_merge (torch.ops.fav.merge_) against the plain-torch merge, three
    blocks in a row, including rows whose block LSE is +inf (no visible key)."""
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    B, C, H, D = 2, 300, 3, 64
    acc_o = acc_lse = ref_o = ref_lse = None
    for i in range(3):
        o = torch.randn((B, C, H, D), device=dev, generator=g).to(dtype)
        lse = torch.randn((B, H, C), device=dev, generator=g) * 3
        if i == 1:
            lse[:, :, :7] = float("inf")
        acc_o, acc_lse = ring._merge(acc_o, acc_lse, o, lse)
        lse_e = torch.where(torch.isposinf(lse), torch.full_like(lse, float("-inf")), lse)
        ref_o, ref_lse = ring._merge_eager(ref_o, ref_lse, o, lse_e)
    torch.cuda.synchronize(dev)
    assert torch.allclose(acc_lse, ref_lse, atol=1e-5, rtol=1e-5)
    assert torch.allclose(acc_o, ref_o, atol=1e-5, rtol=1e-4)


def test_ring_one_rank_long_sequence():
    """The long-context config exactly (B=1, S=131072, H=32, D=128, causal): the
    ring (one rank, zigzag chunks of 65536 rows) against the single-GPU kernel on
    the full tensor, and sampled query rows of O, LSE and dQ of two heads against
    the exact oracle evaluated row by row."""
    from oracle.attention_oracle import attention_rows
    dev = torch.device("cuda", 0)
    B, S, H, D = 1, 131072, 32, 128
    g = torch.Generator(device=dev).manual_seed(21)
    q, k, v, do = (torch.randn((B, S, H, D), device=dev, generator=g, dtype=torch.float16)
                   for _ in range(4))
    scale = 1.0 / math.sqrt(D)
    leaves = [t.clone().requires_grad_() for t in (q, k, v)]
    o = ring.ring_flash_attn(*leaves, causal=True)
    o.backward(do)
    with torch.no_grad():
        _, lse = ring._ring_forward(q, k, v, True, scale, None)
    full = [t.clone().requires_grad_() for t in (q, k, v)]
    of = flash_attn(*full, causal=True)
    of.backward(do)
    torch.cuda.synchronize(dev)
    assert maxdiff(o.detach(), of.detach()) <= TOL_O
    for a, b in zip(leaves, full):
        assert maxdiff(a.grad, b.grad) <= TOL_GRAD
    rows = [0, 1, 4097, 65535, 65536, 99999, S - 1]
    for h in (0, 31):
        sl = lambda t: t[:, :, h:h + 1].cpu()  # noqa: E731
        o_r, lse_r, dq_r = attention_rows(sl(q), sl(k), sl(v), 0, 0, rows, causal=True,
                                          scale=scale, do=sl(do))
        assert maxdiff(o.detach()[0, rows, h].cpu(), o_r) <= TOL_O
        assert maxdiff(lse[0, h, rows].cpu(), lse_r) <= 2e-3
        assert maxdiff(leaves[0].grad[0, rows, h].cpu(), dq_r) <= TOL_GRAD


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _two_gpu_inputs(hkv):
    q, k, v, do = make_inputs(1, 4096, 4, 128, seed=12)
    return q, k[:, :, :hkv].contiguous(), v[:, :, :hkv].contiguous(), do


def _worker(rank, world, port, hkv, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        q, k, v, do = _two_gpu_inputs(hkv)
        sh = lambda t: ring.zigzag_shard(t, rank, world).to(dev)
        qs, ks, vs = (sh(t).requires_grad_() for t in (q, k, v))
        o = ring.ring_flash_attn(qs, ks, vs, causal=True)
        o.backward(sh(do))
        torch.cuda.synchronize(dev)
        out_q.put((rank,) + tuple(t.detach().float().cpu().numpy() for t in (o, qs.grad, ks.grad, vs.grad)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("hkv", [4, 2])
def test_ring_two_gpus_matches_oracle(hkv):
    """hkv=2: grouped-query K/V blocks travel between the ranks with 2 heads."""
    world = 2
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, hkv, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([out_q.get(timeout=300) for _ in range(world)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    o, dq, dk, dv = (ring.zigzag_unshard([torch.from_numpy(r[i]) for r in res]) for i in range(1, 5))
    q, k, v, do = _two_gpu_inputs(hkv)
    rep = 4 // hkv
    ke, ve = k.repeat_interleave(rep, dim=2), v.repeat_interleave(rep, dim=2)
    heads = [(0, 1), (0, 2)]
    ref = oracle_heads(q, ke, ve, do, True, 1 / math.sqrt(128), heads)
    assert maxdiff(pick_heads(o, heads), ref["o"]) <= TOL_O
    assert maxdiff(pick_heads(dq, heads), ref["dq"]) <= TOL_GRAD
    if hkv == 4:
        for g, n in zip((dk, dv), ("dk", "dv")):
            assert maxdiff(pick_heads(g, heads), ref[n]) <= TOL_GRAD
    else:
        # K/V head j gathers the gradients of query heads rep*j .. rep*j + rep - 1
        full = oracle_heads(q, ke, ve, do, True, 1 / math.sqrt(128), [(0, 2), (0, 3)])
        for g, n in ((dk, "dk"), (dv, "dv")):
            ref_kv = full[n][0] + full[n][1]  # query heads 2 and 3 -> K/V head 1
            assert maxdiff(g[0, :, 1], ref_kv) <= TOL_GRAD
