"""Failure detection on the GPU without faulting it.

Every on-device wait is bounded.  A test hook makes the forward kernel skip
one of its own TMA loads, so the MMA issuer's wait for that tile can never be
satisfied; with a 50 ms limit the kernel must give up, report status bit 1 to
the host, release its tensor memory and return — and the same context must
then compute correctly.
"""
import math

import pytest
import torch

from flash_attn_volta_b200 import _lib, check_status, flash_attn, flash_attn_forward
from tests.helpers import TOL_O, make_inputs, maxdiff, oracle_heads, pick_heads

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_context_stays_usable():
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    q, k, v = [t.to(dev) for t in make_inputs(1, 512, 2, 64, seed=21, n=3)]
    check_status(dev)
    lib.fa_sm100_set_wait_timeout_ns(50_000_000)
    lib.fa_sm100_set_debug_flags(1)
    try:
        flash_attn_forward(q, k, v, causal=True)
        torch.cuda.synchronize(dev)
        with pytest.raises(RuntimeError, match="timed out"):
            check_status(dev)
    finally:
        lib.fa_sm100_set_debug_flags(0)
        lib.fa_sm100_set_wait_timeout_ns(4_000_000_000)
    # the context is intact: a normal forward + backward is correct afterwards
    qc, kc, vc, do = make_inputs(1, 512, 2, 64, seed=22)
    leaves = [t.to(dev).requires_grad_() for t in (qc, kc, vc)]
    out = flash_attn(*leaves, causal=True)
    out.backward(do.to(dev))
    torch.cuda.synchronize(dev)
    check_status(dev)
    ref = oracle_heads(qc, kc, vc, do, True, 1 / math.sqrt(64), [(0, 0), (0, 1)], grads=False)
    assert maxdiff(pick_heads(out.detach().cpu(), [(0, 0), (0, 1)]), ref["o"]) <= TOL_O
