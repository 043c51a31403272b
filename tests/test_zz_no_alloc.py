"""fa_sm100_bwd_noalloc — the backward for callers that cannot allocate.

Some callers cannot call cudaMalloc (or any allocator, torch's included) when
they run the backward: runtimes that only hand out pre-planned buffers, or an
execution phase in which allocation is forbidden.  fa_sm100_bwd_noalloc serves
them from a static device array inside the library instead of a
caller-provided workspace.  This test calls it through the C ABI, twice in a
row with different inputs, and checks each result against fa_sm100_bwd (the
entry point with a workspace) and against the exact CPU oracle on sampled
heads, within the suite's gradient tolerance; it also checks that a call made
after the first one (which looks up the array's address) allocates no device
memory, neither through torch's allocator nor from the driver.  It is
collected last so that a stop-at-first-failure run has already run the rest.
"""
import ctypes
import math

import pytest
import torch

from flash_attn_volta_b200 import _lib, check_status, flash_attn_forward
from tests.helpers import TOL_GRAD, make_inputs, maxdiff, oracle_heads, pick_heads

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)


def _bwd_both(B, S, H, D, causal, seed):
    lib = _lib.load()
    q, k, v, do = make_inputs(B, S, H, D, seed=seed)
    qd, kd, vd, dod = (t.to(DEV) for t in (q, k, v, do))
    o, lse = flash_attn_forward(qd, kd, vd, causal=causal, return_softmax_lse=True)
    scale = 1.0 / math.sqrt(D)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    status = _lib.status_word(DEV)
    ptrs = [t.data_ptr() for t in (dod, qd, kd, vd, o)] + [lse.data_ptr()]

    ref = [torch.empty_like(qd) for _ in range(3)]
    nbytes = lib.fa_sm100_bwd_workspace_bytes(B, S, H, D)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    rc = lib.fa_sm100_bwd(*ptrs, *[t.data_ptr() for t in ref], ws.data_ptr(), nbytes,
                          B, S, H, D, scale, int(causal), status.data_ptr(), stream)
    assert rc == _lib.FA_OK, lib.fa_sm100_error_string(rc)

    got = [torch.full_like(qd, float("nan")) for _ in range(3)]
    torch.cuda.synchronize(DEV)
    alloc0 = torch.cuda.memory_stats(DEV).get("allocation.all.allocated", 0)
    free0, _ = torch.cuda.mem_get_info(DEV)
    rc = lib.fa_sm100_bwd_noalloc(*ptrs, *[t.data_ptr() for t in got], B, S, H, D, scale,
                                  int(causal), status.data_ptr(), stream)
    assert rc == _lib.FA_OK, lib.fa_sm100_error_string(rc)
    torch.cuda.synchronize(DEV)
    alloc1 = torch.cuda.memory_stats(DEV).get("allocation.all.allocated", 0)
    free1, _ = torch.cuda.mem_get_info(DEV)
    check_status(DEV)
    return (q, k, v, do), ref, got, (alloc1 - alloc0, free0 - free1)


def test_noalloc_matches_workspace_entry_and_oracle_twice():
    # warm-up call: the first call on a device looks up the static array's address
    _bwd_both(1, 64, 1, 64, False, 20)
    # two calls in a row: the second reuses the static scratch the first left behind
    for (B, S, H, D, causal, seed) in [(2, 1000, 4, 128, True, 21), (1, 333, 3, 64, False, 22)]:
        (q, k, v, do), ref, got, (d_alloc, d_free) = _bwd_both(B, S, H, D, causal, seed)
        assert d_alloc == 0, "torch allocations during the no-alloc call"
        assert d_free == 0, "device memory taken from the driver during the no-alloc call"
        for r, g in zip(ref, got):
            assert torch.isfinite(g).all()
            assert maxdiff(r, g) <= TOL_GRAD
        heads = [(0, 0), (B - 1, H - 1)]
        exact = oracle_heads(q, k, v, do, causal, 1.0 / math.sqrt(D), heads)
        for name, g in zip(("dq", "dk", "dv"), got):
            assert maxdiff(pick_heads(g.cpu(), heads), exact[name]) <= TOL_GRAD, name


def test_noalloc_rejects_shapes_beyond_its_scratch():
    lib = _lib.load()
    B, S, H, D = 1, 65536, 8, 128  # needs ~290 MiB of scratch
    assert lib.fa_sm100_bwd_workspace_bytes(B, S, H, D) > 32 * 1024 * 1024
    rc = lib.fa_sm100_bwd_noalloc(*([16] * 6), *([16] * 3), B, S, H, D, 0.1, 1, None, None)
    assert rc == _lib.FA_ERR_SCRATCH_LIMIT
    assert b"32 MiB" in lib.fa_sm100_error_string(rc)
