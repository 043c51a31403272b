"""Ring context-parallel attention: host logic on CPU ranks (gloo).

The per-block kernels are replaced by the CPU oracle; zigzag sharding, block
masks, the LSE merge, the K/V rotation and the dK/dV return hop are the
product code.  Result and gradients are compared with the unsharded oracle.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flash_attn_volta_b200 import ring
from oracle.attention_oracle import attention_bwd, attention_bwd_given_lse, attention_fwd
from tests.helpers import make_inputs, maxdiff


def _expand(q, k, v):
    rep = q.shape[2] // k.shape[2]
    return rep, k.repeat_interleave(rep, dim=2), v.repeat_interleave(rep, dim=2)


def _oracle_block_fwd(q, k, v, causal, scale):
    _, k, v = _expand(q, k, v)
    o, lse = attention_fwd(q, k, v, causal, scale, dtype=torch.float64)
    return o.float(), lse.float()


def _oracle_block_bwd(do, q, k, v, o, lse, causal, scale):
    """Grouped K/V: the gradients of the expanded heads summed over each group."""
    B, C, Hkv, D = k.shape
    rep, k, v = _expand(q, k, v)
    dq, dk, dv = attention_bwd_given_lse(do, q, k, v, o, lse, causal, scale)
    dk, dv = (t.reshape(B, C, Hkv, rep, D).sum(3) for t in (dk, dv))
    return dq.float(), dk.float(), dv.float()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(hkv):
    """(B=2, S=64, H=4, D=16); K and V with `hkv` heads."""
    q, k, v, do = [t.float() for t in make_inputs(2, 64, 4, 16, seed=5)]
    return q, k[:, :, :hkv].contiguous(), v[:, :, :hkv].contiguous(), do


def _worker(rank, world, port, causal, hkv, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ring.block_fwd, ring.block_bwd = _oracle_block_fwd, _oracle_block_bwd
        q, k, v, do = _inputs(hkv)
        shard = lambda t: ring.zigzag_shard(t, rank, world).requires_grad_()
        qs, ks, vs = shard(q), shard(k), shard(v)
        o = ring.ring_flash_attn(qs, ks, vs, causal=causal)
        o.backward(ring.zigzag_shard(do, rank, world))
        out_q.put((rank,) + tuple(t.detach().cpu().numpy() for t in (o, qs.grad, ks.grad, vs.grad)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,causal,hkv", [
    (1, True, 4), (1, False, 4), (2, True, 4), (2, False, 4), (4, True, 4), (4, False, 4),
    (2, True, 2), (4, True, 1), (2, False, 1)])
def test_ring_matches_full_attention(world, causal, hkv):
    """hkv < 4: grouped-query (2) and multi-query (1) K/V."""
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, causal, hkv, out_q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([out_q.get(timeout=120) for _ in range(world)], key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    o, dq, dk, dv = (ring.zigzag_unshard([torch.from_numpy(r[i]) for r in res]) for i in range(1, 5))
    q, k, v, do = _inputs(hkv)
    rep, ke, ve = _expand(q, k, v)
    o_ref, _ = attention_fwd(q, ke, ve, causal, dtype=torch.float64)
    dq_r, dk_r, dv_r = attention_bwd(do, q, ke, ve, causal)
    B, S, _, D = k.shape
    g_ref = (dq_r, dk_r.reshape(B, S, hkv, rep, D).sum(3), dv_r.reshape(B, S, hkv, rep, D).sum(3))
    assert maxdiff(o, o_ref) < 1e-5
    for g, r in zip((dq, dk, dv), g_ref):
        assert maxdiff(g, r) < 1e-5


def test_zigzag_roundtrip_and_balance():
    x = torch.arange(2 * 48).reshape(2, 48)
    shards = [ring.zigzag_shard(x, r, 4) for r in range(4)]
    assert torch.equal(ring.zigzag_unshard(shards), x)
    # causal work per rank (number of unmasked (q, k) pairs) is equal
    S, C = 48, 6
    work = []
    for r in range(4):
        ids = ring.zigzag_chunk_ids(r, 4)
        work.append(sum(min(i * C + t + 1, S) for i in ids for t in range(C)))
    assert len(set(work)) == 1


def test_block_backward_oracle_reduces_to_plain_backward():
    q, k, v, do = make_inputs(1, 40, 2, 16, seed=6)
    o, lse = attention_fwd(q, k, v, True, dtype=torch.float64)
    a = attention_bwd_given_lse(do, q, k, v, o, lse, True)
    b = attention_bwd(do, q, k, v, True)
    for x, y in zip(a, b):
        assert maxdiff(x, y) < 1e-10


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_dkdv_contribution_sets(world):
    """Which key chunks of rank k the queries of rank q reach (the dK/dV chunks
    a backward step sends to k's owner): under the zigzag causal layout a rank
    behind the key rank reaches only its first chunk, the others both; without a
    causal mask always both.  Sender and receiver use the same function."""
    for q in range(world):
        for k in range(world):
            want = [0] if k < q else [0, 1]
            assert ring._contributions(q, k, world, True) == want, (q, k)
            assert ring._contributions(q, k, world, False) == [0, 1]
