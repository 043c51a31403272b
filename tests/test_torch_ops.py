"""The torch.ops.fav operators (csrc/torch_ops.cpp + ops.py).

CPU: the operator library loads, registers fav::fwd / fav::bwd / fav::status,
and their shape functions work on meta tensors (what torch.compile traces
with).  GPU: torch.library.opcheck (schema, fake-tensor and autograd
registration checks) and torch.compile(fullgraph=True) of flash_attn, i.e.
the whole call traces without a graph break, with results equal to eager.
"""
import math

import pytest
import torch

from flash_attn_volta_b200 import ops


def test_ops_library_registers_operators():
    ops.load()
    for name in ("fwd", "bwd", "status"):
        assert hasattr(torch.ops.fav, name)
    schema = str(torch.ops.fav.fwd.default._schema)
    assert "bool causal" in schema and "float sm_scale" in schema


def test_ops_library_uses_shared_libstdcxx():
    """A static copy of libstdc++ inside the operator library crashed when torch
    formatted one of its error messages (two copies of the locale machinery in
    one process)."""
    from flash_attn_volta_b200 import build
    ops.load()
    assert not build._has_static_libstdcxx(build.ops_path())


@pytest.mark.parametrize("Hkv,Sk", [(8, 300), (2, 77)])
def test_fake_shapes_on_meta(Hkv, Sk):
    ops.load()
    q = torch.empty((2, 300, 8, 64), dtype=torch.float16, device="meta")
    k = torch.empty((2, Sk, Hkv, 64), dtype=torch.float16, device="meta")
    out, lse = torch.ops.fav.fwd(q, k, k, True, 0.125)
    assert out.shape == q.shape and out.dtype == q.dtype
    assert lse.shape == (2, 8, 300) and lse.dtype == torch.float32
    dq, dk, dv = torch.ops.fav.bwd(q, q, k, k, out, lse, True, 0.125)
    assert dq.shape == q.shape and dk.shape == k.shape and dv.shape == k.shape


def _bad_calls(dev):
    """Direct operator calls whose tensors disagree with q / k: each must raise
    (the C ABI takes every extent from q and k)."""
    mk = lambda *s: torch.zeros(s, dtype=torch.float16, device=dev)  # noqa: E731
    q, k, o = mk(1, 128, 4, 64), mk(1, 128, 2, 64), mk(1, 128, 4, 64)
    lse = torch.zeros((1, 4, 128), dtype=torch.float32, device=dev)
    return [
        lambda: torch.ops.fav.fwd(q, mk(1, 128, 3, 64), mk(1, 128, 3, 64), True, 0.125),
        lambda: torch.ops.fav.fwd(q, mk(1, 128, 2, 32), mk(1, 128, 2, 32), True, 0.125),
        lambda: torch.ops.fav.fwd(q, k, mk(1, 64, 2, 64), True, 0.125),
        lambda: torch.ops.fav.bwd(mk(1, 64, 4, 64), q, k, k, o, lse, True, 0.125),
        lambda: torch.ops.fav.bwd(o, q, k, k, mk(1, 128, 4, 32), lse, True, 0.125),
        lambda: torch.ops.fav.bwd(o, q, k, k, o, lse[:, :, :64], True, 0.125),
        lambda: torch.ops.fav.merge_(o.float(), lse[:, :2], o, lse, False),
    ]


def test_shape_mismatch_raises_on_meta():
    ops.load()
    for call in _bad_calls("meta"):
        with pytest.raises(RuntimeError):
            call()


@pytest.mark.gpu
def test_shape_mismatch_raises_on_cuda():
    ops.load()
    for call in _bad_calls("cuda"):
        with pytest.raises(RuntimeError):
            call()
    torch.cuda.synchronize()


@pytest.mark.gpu
def test_opcheck():
    ops.load()
    g = torch.Generator(device="cuda").manual_seed(0)
    mk = lambda *s: torch.randn(s, device="cuda", dtype=torch.float16, generator=g)  # noqa: E731
    q, k, v, do = mk(1, 256, 4, 64), mk(1, 256, 2, 64), mk(1, 256, 2, 64), mk(1, 256, 4, 64)
    out, lse = torch.ops.fav.fwd(q, k, v, True, 0.125)
    # the bwd operator has no autograd formula of its own (it is not differentiable)
    torch.library.opcheck(torch.ops.fav.bwd, (do, q, k, v, out, lse, True, 0.125),
                          test_utils=("test_schema", "test_faketensor"))
    for t in (q, k, v):
        t.requires_grad_()
    torch.library.opcheck(torch.ops.fav.fwd, (q, k, v, True, 0.125),
                          test_utils=("test_schema", "test_autograd_registration",
                                      "test_faketensor"))


@pytest.mark.gpu
def test_compile_fullgraph_matches_eager():
    from flash_attn_volta_b200 import flash_attn
    torch._dynamo.reset()
    g = torch.Generator(device="cuda").manual_seed(1)
    mk = lambda: torch.randn((2, 384, 4, 128), device="cuda", dtype=torch.float16,  # noqa: E731
                             generator=g)
    q, k, v, do = mk(), mk(), mk(), mk()

    def f(q, k, v):
        return flash_attn(q, k, v, causal=True) * 2.0

    cf = torch.compile(f, fullgraph=True, backend="aot_eager")
    res = []
    for fn in (f, cf):
        qq, kk, vv = (t.clone().requires_grad_() for t in (q, k, v))
        o = fn(qq, kk, vv)
        o.backward(do)
        res.append((o.detach(), qq.grad, kk.grad, vv.grad))
    for a, b in zip(*res):
        assert torch.equal(a, b) or float((a.float() - b.float()).abs().max()) <= 1e-3
    assert math.isfinite(float(res[1][0].float().abs().max()))
