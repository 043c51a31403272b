"""CPU tests of the C ABI library: it loads, exports what include/fa_sm100.h
declares, and rejects bad arguments before touching a GPU."""
import os
import re

import pytest
import torch

from flash_attn_volta_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = []
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            txt = open(os.path.join(ROOT, "include", fn)).read()
            names += re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(fa_\w+)\s*\(", txt, re.M)
    return sorted(set(names))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = _declared_functions()
    assert "fa_sm100_fwd" in names and "fa_sm100_bwd" in names
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"
    assert lib.fa_sm100_abi_version() == 3


def test_error_strings():
    lib = _lib.load()
    for code in range(7):
        assert lib.fa_sm100_error_string(code)


@pytest.mark.parametrize("shape", [(0, 16, 1, 64), (1, 0, 1, 64), (1, 16, 0, 64),
                                   (1, 16, 1, 48), (1, 16, 1, 256)])
def test_fwd_rejects_bad_shapes(shape):
    lib = _lib.load()
    B, S, H, D = shape
    rc = lib.fa_sm100_fwd(16, 16, 16, 16, None, B, S, H, D, 1.0, 0, None, None)
    assert rc == _lib.FA_ERR_ARG


def test_fwd_rejects_null_and_misaligned():
    lib = _lib.load()
    assert lib.fa_sm100_fwd(None, 16, 16, 16, None, 1, 16, 1, 64, 1.0, 0, None, None) == 1
    assert lib.fa_sm100_fwd(16, 18, 16, 16, None, 1, 16, 1, 64, 1.0, 0, None, None) == 1


def test_bwd_workspace_contract():
    lib = _lib.load()
    n = lib.fa_sm100_bwd_workspace_bytes(2, 100, 3, 64)
    rows = 2 * 3 * 128  # rows padded to 128
    assert n >= rows * 64 * 4 + 2 * rows * 4
    assert lib.fa_sm100_bwd_workspace_bytes(1, 1, 1, 48) == 0
    # too-small workspace is reported before any device work
    rc = lib.fa_sm100_bwd(16, 16, 16, 16, 16, 16, 16, 16, 16, 256, n - 1, 2, 100, 3, 64, 1.0, 0,
                          None, None)
    assert rc == _lib.FA_ERR_WORKSPACE


def test_python_api_asserts_like_reference():
    from flash_attn_volta_b200 import flash_attn_backward, flash_attn_forward
    q = torch.zeros(1, 8, 1, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):
        flash_attn_forward(q, q, q)
    with pytest.raises(AssertionError):
        flash_attn_backward(q, q, q, q, q, torch.zeros(1, 1, 8))


def test_public_api_surface():
    import flash_attn_volta_b200 as m
    assert m.__version__ == "0.2.0"
    assert set(m.__all__) == {"flash_attn_forward", "flash_attn_volta", "flash_attn_backward",
                              "flash_attn"}
    assert m.flash_attn_volta is m.flash_attn_forward


def test_ex_head_count_and_dtype_checks():
    """fa_sm100_*_ex reject a K/V head count that does not divide the query heads
    and an unknown element type before touching the device."""
    lib = _lib.load()
    f16, bf16 = _lib.DTYPE_F16, _lib.DTYPE_BF16
    args_f = (16, 16, 16, 16, None, 1, 64, 64, 8, 3, 64, f16, 0.125, 1, None, None)
    assert lib.fa_sm100_fwd_ex(*args_f) == _lib.FA_ERR_ARG
    args_f0 = (16, 16, 16, 16, None, 1, 64, 64, 8, 0, 64, bf16, 0.125, 1, None, None)
    assert lib.fa_sm100_fwd_ex(*args_f0) == _lib.FA_ERR_ARG
    args_dt = (16, 16, 16, 16, None, 1, 64, 64, 8, 2, 64, 7, 0.125, 1, None, None)
    assert lib.fa_sm100_fwd_ex(*args_dt) == _lib.FA_ERR_ARG
    args_sk = (16, 16, 16, 16, None, 1, 64, 0, 8, 2, 64, f16, 0.125, 1, None, None)
    assert lib.fa_sm100_fwd_ex(*args_sk) == _lib.FA_ERR_ARG  # no keys
    n = lib.fa_sm100_bwd_workspace_bytes(1, 64, 8, 64)
    rc = lib.fa_sm100_bwd_ex(*([256] * 9), 256, n, 1, 64, 64, 8, 3, 64, f16, 0.125, 1, None, None)
    assert rc == _lib.FA_ERR_ARG
    rc = lib.fa_sm100_bwd_ex(*([256] * 9), 256, n, 1, 64, 64, 8, 2, 64, 9, 0.125, 1, None, None)
    assert rc == _lib.FA_ERR_ARG


def test_deterministic_flag_workspace_and_checks():
    """FA_BWD_DETERMINISTIC needs no fp32 dQ accumulator; unknown flag bits are
    refused before touching the device."""
    lib = _lib.load()
    B, S, H, D = 2, 1000, 4, 128
    fused = lib.fa_sm100_bwd_workspace_bytes_flags(B, S, H, D, 0)
    det = lib.fa_sm100_bwd_workspace_bytes_flags(B, S, H, D, _lib.BWD_DETERMINISTIC)
    assert fused == lib.fa_sm100_bwd_workspace_bytes(B, S, H, D)
    rows = B * H * 1024  # rows padded to 128
    assert fused - det >= rows * D * 4 - rows * 4  # the accumulator is gone, delta is added
    assert lib.fa_sm100_bwd_workspace_bytes_flags(B, S, H, D, 2) == 0
    rc = lib.fa_sm100_bwd_flags(*([256] * 9), 256, fused, B, S, S, H, H, D, _lib.DTYPE_F16,
                                0.1, 1, 2, None, None)
    assert rc == _lib.FA_ERR_ARG


def test_merge_argument_checks():
    lib = _lib.load()
    f16 = _lib.DTYPE_F16
    assert lib.fa_sm100_merge(256, 256, 256, 256, 1, 8, 2, 48, f16, 1, None) == _lib.FA_ERR_ARG
    assert lib.fa_sm100_merge(None, 256, 256, 256, 1, 8, 2, 64, f16, 1, None) == _lib.FA_ERR_ARG
    assert lib.fa_sm100_merge(264, 256, 256, 256, 1, 8, 2, 64, f16, 1, None) == _lib.FA_ERR_ARG
    assert lib.fa_sm100_merge(256, 256, 256, 256, 1, 8, 2, 64, 5, 1, None) == _lib.FA_ERR_ARG
