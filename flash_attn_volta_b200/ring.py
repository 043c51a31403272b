"""Ring context-parallel attention over the sequence axis (NCCL send/recv).

For sequences too long for one GPU's time budget (the long-context training
variant: B=1, S=131072, H=32, D=128, causal over 8 GPUs).  The reference has
no multi-GPU path; this is the build's own design on top of the single-GPU
kernels:

* Zigzag sharding: the sequence is cut into 2·G chunks of C = S / (2G) rows
  and rank r holds chunks r and 2G-1-r of q, k, v (and o, dO).  Under a causal
  mask every rank then has the same amount of work.
* Forward: G steps; at step s rank r holds the K/V chunks of rank (r - s) mod G
  and computes its two query chunks against them.  A (query chunk i, key chunk
  j) block is skipped if j > i, causal if j == i and full if j < i (without a
  causal mask every block is full).  Every block is a square C x C attention —
  exactly what the single-GPU kernel computes — returning (O_ij, LSE_ij); the
  partial results are merged with lse = logaddexp(lse, lse_ij) and
  O = sum_j exp(lse_ij - lse) O_ij in fp32 (each O_ij arrives rounded to the
  element type by the kernel).  The next K and V blocks are exchanged (one
  batched isend/irecv to r+1 / from r-1) while the current one is computed.
* Backward: the same K/V ring; each block's (dq, dk, dv) come from the
  single-GPU backward fed with the *final* O and LSE (so P and delta are the
  global ones, as in the reference's Algorithm-4 backward); dq accumulates
  locally.  A step's dK/dV contributions go straight to the owner of that
  K/V block (rank - step), in the kernels' element type and only for the key
  chunks the step's queries attend to, and the owner accumulates them in fp32:
  under the zigzag causal layout about half of the steps touch one key chunk
  only, so this moves ~3x fewer bytes than an fp32 accumulator travelling
  with its block.  The transfer of step s overlaps the compute of step s + 1.

Received blocks land in local buffers before a kernel reads them: no kernel
touches another GPU's memory.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from . import ops
from .backward import flash_attn_backward
from .forward import flash_attn_forward


def _kernel_block_fwd(q, k, v, causal, scale):
    return flash_attn_forward(q, k, v, causal=causal, sm_scale=scale, return_softmax_lse=True)


def _kernel_block_bwd(do, q, k, v, o, lse, causal, scale):
    return flash_attn_backward(do, q, k, v, o, lse, causal=causal, sm_scale=scale)


# The per-block computations; the CPU tests substitute the oracle here.
block_fwd = _kernel_block_fwd
block_bwd = _kernel_block_bwd


def zigzag_chunk_ids(rank: int, world: int) -> tuple[int, int]:
    return rank, 2 * world - 1 - rank


def zigzag_shard(x: torch.Tensor, rank: int, world: int, dim: int = 1) -> torch.Tensor:
    """This rank's two chunks of x along `dim`, concatenated (length 2*S/(2*world))."""
    S = x.shape[dim]
    assert S % (2 * world) == 0, f"sequence length {S} not divisible by 2*world={2 * world}"
    chunks = x.chunk(2 * world, dim=dim)
    a, b = zigzag_chunk_ids(rank, world)
    return torch.cat([chunks[a], chunks[b]], dim=dim).contiguous()


def zigzag_unshard(shards: list, dim: int = 1) -> torch.Tensor:
    """Inverse of zigzag_shard given every rank's shard (rank order)."""
    world = len(shards)
    chunks = [None] * (2 * world)
    for r, s in enumerate(shards):
        a, b = zigzag_chunk_ids(r, world)
        chunks[a], chunks[b] = s.chunk(2, dim=dim)
    return torch.cat(chunks, dim=dim)


def _block_mode(i: int, j: int, causal: bool):
    """None = skip, True = causal (diagonal) block, False = full block."""
    if not causal:
        return False
    if j > i:
        return None
    return j == i


def _merge_eager(acc_o, acc_lse, o, lse):
    """The merge in plain torch operations, for CPU tensors (the gloo tests,
    whose blocks come from the oracle)."""
    o = o.float()
    if acc_o is None:
        return o, lse.clone()
    new = torch.logaddexp(acc_lse, lse)
    w_old = torch.exp(acc_lse - new).transpose(1, 2).unsqueeze(-1)
    w_new = torch.exp(lse - new).transpose(1, 2).unsqueeze(-1)
    return acc_o * w_old + o * w_new, new


def _merge(acc_o, acc_lse, o, lse):
    """Merge a block's (o (B,C,H,D), lse (B,H,C)) into the fp32 running result:
    one fa_sm100_merge kernel on the GPU (in place), plain torch on the CPU."""
    if o.device.type != "cuda":
        return _merge_eager(acc_o, acc_lse, o, lse)
    first = acc_o is None
    if first:
        acc_o = torch.empty(o.shape, dtype=torch.float32, device=o.device)
        acc_lse = torch.empty(lse.shape, dtype=torch.float32, device=o.device)
    ops.load()
    torch.ops.fav.merge_(acc_o, acc_lse, o, lse, first)
    return acc_o, acc_lse


def _peers(group, rank: int, world: int):
    nxt = dist.get_global_rank(group, (rank + 1) % world) if group is not None else (rank + 1) % world
    prv = dist.get_global_rank(group, (rank - 1) % world) if group is not None else (rank - 1) % world
    return nxt, prv


def _exchange(sends, group, rank: int, world: int):
    """Start sending each tensor of `sends` to rank+1 and receiving tensors of
    the same shapes from rank-1 (one batched NCCL call); returns (recvs, works)."""
    nxt, prv = _peers(group, rank, world)
    recvs = [torch.empty_like(t) for t in sends]
    p2p = [dist.P2POp(dist.isend, t, nxt, group) for t in sends]
    p2p += [dist.P2POp(dist.irecv, t, prv, group) for t in recvs]
    return recvs, dist.batch_isend_irecv(p2p)


def _finish(works):
    # NCCL works: the current stream waits on the device; the host does not block
    for w in works:
        w.wait()


def _world(group):
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def _ring_forward(q2, k2, v2, causal, scale, group):
    rank, world = _world(group)
    q = [c.contiguous() for c in q2.chunk(2, dim=1)]
    ids_q = zigzag_chunk_ids(rank, world)
    kv = (k2, v2)
    acc = [[None, None], [None, None]]  # per query chunk: [o, lse]
    for step in range(world):
        src = (rank - step) % world
        ids_k = zigzag_chunk_ids(src, world)
        # the next K/V block travels while this one is computed
        pending = _exchange(kv, group, rank, world) if step < world - 1 else None
        ks, vs = kv[0].chunk(2, dim=1), kv[1].chunk(2, dim=1)
        for a in range(2):
            for b in range(2):
                mode = _block_mode(ids_q[a], ids_k[b], causal)
                if mode is None:
                    continue
                o, lse = block_fwd(q[a], ks[b].contiguous(), vs[b].contiguous(), mode, scale)
                acc[a] = list(_merge(acc[a][0], acc[a][1], o, lse))
        if pending is not None:
            recvs, works = pending
            _finish(works)
            kv = tuple(recvs)
    o = torch.cat([acc[0][0], acc[1][0]], dim=1).to(q2.dtype)
    lse = torch.cat([acc[0][1], acc[1][1]], dim=2).contiguous()
    return o, lse


def _contributions(q_rank: int, k_rank: int, world: int, causal: bool) -> list:
    """Key chunks (0 / 1) of rank k_rank that the query chunks of rank q_rank
    attend to: the dK / dV chunks a backward step of q_rank on k_rank's block
    contributes to (the same on the sending and the receiving side)."""
    ids_q, ids_k = zigzag_chunk_ids(q_rank, world), zigzag_chunk_ids(k_rank, world)
    return [b for b in range(2)
            if any(_block_mode(ids_q[a], ids_k[b], causal) is not None for a in range(2))]


def _ring_backward(do2, q2, k2, v2, o2, lse2, causal, scale, group):
    rank, world = _world(group)
    q = [c.contiguous() for c in q2.chunk(2, dim=1)]
    do = [c.contiguous() for c in do2.chunk(2, dim=1)]
    o = [c.contiguous() for c in o2.chunk(2, dim=1)]
    lse = [c.contiguous() for c in lse2.chunk(2, dim=2)]
    ids_q = zigzag_chunk_ids(rank, world)
    dq = torch.zeros(q2.shape, dtype=torch.float32, device=q2.device)
    dqs = dq.chunk(2, dim=1)
    # dK / dV of this rank's own K/V block, accumulated here in fp32.  At step s
    # this rank computes the contributions of its queries to block src = rank - s
    # and sends them straight to that block's owner, in the kernels' element
    # type (which their outputs are rounded to already; two contributions to
    # one chunk are summed in fp32 first) and only for the key chunks its
    # queries attend to.  The owner receives from rank + s at the same step.
    dk_acc = torch.zeros(k2.shape, dtype=torch.float32, device=q2.device)
    dv_acc = torch.zeros(v2.shape, dtype=torch.float32, device=q2.device)
    dks_acc, dvs_acc = dk_acc.chunk(2, dim=1), dv_acc.chunk(2, dim=1)
    kv = (k2, v2)
    inflight = None  # (works, recv tensors, chunk ids, send tensors kept alive)
    for step in range(world):
        src = (rank - step) % world
        ids_k = zigzag_chunk_ids(src, world)
        pending = _exchange(kv, group, rank, world) if step < world - 1 else None
        ks, vs = kv[0].chunk(2, dim=1), kv[1].chunk(2, dim=1)
        part = {}  # key chunk -> [dk, dv] (fp32 once a second contribution arrives)
        for a in range(2):
            for b in range(2):
                mode = _block_mode(ids_q[a], ids_k[b], causal)
                if mode is None:
                    continue
                g = block_bwd(do[a], q[a], ks[b].contiguous(), vs[b].contiguous(), o[a], lse[a],
                              mode, scale)
                dqs[a].add_(g[0])  # fp32 += element type in one kernel
                if b in part:
                    part[b] = [part[b][0].float().add_(g[1]), part[b][1].float().add_(g[2])]
                else:
                    part[b] = [g[1], g[2]]
        if inflight is not None:
            works, recvs, chunks, _ = inflight
            _finish(works)
            for i, b in enumerate(chunks):
                dks_acc[b].add_(recvs[2 * i])
                dvs_acc[b].add_(recvs[2 * i + 1])
            inflight = None
        if step == 0:
            for b, (gk, gv) in part.items():
                dks_acc[b].add_(gk)
                dvs_acc[b].add_(gv)
        else:
            dst, peer = (rank - step) % world, (rank + step) % world
            sends = []
            for b in sorted(part):
                sends += [part[b][0].to(k2.dtype).contiguous(), part[b][1].to(v2.dtype).contiguous()]
            chunks = _contributions(peer, rank, world, causal)
            shape = ks[0].shape
            recvs = [torch.empty(shape, dtype=k2.dtype, device=q2.device)
                     for _ in range(2 * len(chunks))]
            g_dst = dist.get_global_rank(group, dst) if group is not None else dst
            g_peer = dist.get_global_rank(group, peer) if group is not None else peer
            p2p = [dist.P2POp(dist.isend, t, g_dst, group) for t in sends]
            p2p += [dist.P2POp(dist.irecv, t, g_peer, group) for t in recvs]
            works = dist.batch_isend_irecv(p2p) if p2p else []
            inflight = (works, recvs, chunks, sends)
        if pending is not None:
            recvs_kv, works_kv = pending
            _finish(works_kv)
            kv = tuple(recvs_kv)
    if inflight is not None:
        works, recvs, chunks, _ = inflight
        _finish(works)
        for i, b in enumerate(chunks):
            dks_acc[b].add_(recvs[2 * i])
            dvs_acc[b].add_(recvs[2 * i + 1])
    return dq.to(q2.dtype), dk_acc.to(k2.dtype), dv_acc.to(v2.dtype)


class _RingFlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, sm_scale, group):
        o, lse = _ring_forward(q, k, v, causal, sm_scale, group)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.sm_scale, ctx.group = causal, sm_scale, group
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        do = do.contiguous().to(q.dtype)
        dq, dk, dv = _ring_backward(do, q, k, v, o, lse, ctx.causal, ctx.sm_scale, ctx.group)
        return dq, dk, dv, None, None, None


def ring_flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = True,
                    sm_scale: Optional[float] = None, group=None) -> torch.Tensor:
    """Attention over a sequence sharded across the ranks of `group` (zigzag).

    Args:
        q: this rank's zigzag shard, (B, 2*C, H, D) — see zigzag_shard.
        k, v: the same rows of K and V, (B, 2*C, H_kv, D) with H % H_kv == 0
            (grouped-query / multi-query attention: query head h reads K/V head
            h // (H // H_kv); the K/V blocks travel with H_kv heads).
        causal: top-left causal mask over the full (unsharded) sequence.
        sm_scale: softmax scale (default 1/sqrt(D)).
        group: process group (default: the world).

    Returns the rank's shard of the output, same layout; autograd-aware.
    """
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    assert k.shape == v.shape and q.dim() == 4 and q.shape[1] % 2 == 0
    assert q.shape[:2] == k.shape[:2] and q.shape[3] == k.shape[3], \
        "q and k/v must have the same batch, sequence shard and head_dim"
    assert k.shape[2] > 0 and q.shape[2] % k.shape[2] == 0, \
        "the query heads must be a multiple of the key/value heads"
    return _RingFlashAttnFn.apply(q, k, v, causal, sm_scale, group)
