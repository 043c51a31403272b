"""Compile the package's native libraries in-tree.

    python -m flash_attn_volta_b200.build [-v] [-f]

libfa_sm100.so (nvcc, sm_100a) holds every CUDA kernel of the package plus the
C ABI declared in include/fa_sm100.h.  libfa_torch_ops.so (g++ against
PyTorch's headers) registers the torch.ops.fav operators on top of that C ABI
and links libfa_sm100.so from its own directory.  Both are built next to this
file so that they travel with the source tree; nothing is installed into
site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libfa_sm100.so"
SOURCES = ["fa_api.cu", "fa_fwd.cu", "fa_bwd.cu", "fa_bwd_dq.cu", "fa_merge.cu", "fa_bwd_noalloc.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


OPS_NAME = "libfa_torch_ops.so"
OPS_SOURCES = ["torch_ops.cpp"]


def lib_path() -> str:
    return os.path.join(HERE, LIB_NAME)


def ops_path() -> str:
    return os.path.join(HERE, OPS_NAME)


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _stale(out: str, deps: list[str] | None = None) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    if deps is None:
        deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f not in OPS_SOURCES]
    deps = deps + [os.path.join(HERE, "..", "include", "fa_sm100.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build_torch_ops(force: bool = False, verbose: bool = False) -> str:
    """Compile libfa_torch_ops.so (needs libfa_sm100.so built first)."""
    import torch
    from torch.utils import cpp_extension as ce

    out = ops_path()
    deps = [os.path.join(CSRC, s) for s in OPS_SOURCES] + [lib_path()]
    if not force and not _stale(out, deps):
        return out
    cxx = os.environ.get("CXX") or shutil.which("g++") or "g++"
    inc = ce.include_paths(device_type="cuda")
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = out + ".tmp"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=fa_torch_ops"]
    cmd += [f"-I{d}" for d in inc]
    cmd += [os.path.join(CSRC, s) for s in OPS_SOURCES]
    cmd += ["-o", tmp, f"-L{HERE}", "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN"]
    cmd += [f"-L{d}" for d in libdirs]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
    # The shared libstdc++ that torch itself uses, named explicitly: a toolchain
    # whose libstdc++.so link is missing would otherwise fall back to
    # libstdc++.a and put a second, uninitialised copy of the iostream / locale
    # code into this library (torch's error messages then crash in it).
    cmd += ["-l:libstdc++.so.6"]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed with exit code {res.returncode}")
    if _has_static_libstdcxx(tmp):
        os.remove(tmp)
        raise RuntimeError(f"{cxx} linked libstdc++ statically into {out}; "
                           "use a g++ whose libstdc++.so is installed (CXX=...)")
    os.replace(tmp, out)
    return out


def _has_static_libstdcxx(path: str) -> bool:
    """True if `path` carries libstdc++'s own locale instantiations, i.e. a
    static copy of libstdc++ rather than a reference to libstdc++.so.6."""
    with open(path, "rb") as f:
        return b"locale_inst.cc" in f.read()


def build(force: bool = False, verbose: bool = False) -> str:
    """Build libfa_sm100.so, then libfa_torch_ops.so; returns the former's path."""
    out = _build_kernels(force, verbose)
    build_torch_ops(force, verbose)
    return out


def _build_kernels(force: bool = False, verbose: bool = False) -> str:
    out = lib_path()
    if not force and not _stale(out):
        return out
    tmp = out + ".tmp"
    extra = os.environ.get("FA_SM100_NVCC_EXTRA", "").split()
    cmd = [_nvcc(), *NVCC_FLAGS, *extra, "-o", tmp] + [os.path.join(CSRC, s) for s in SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed with exit code {res.returncode}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(force="-f" in sys.argv, verbose="-v" in sys.argv))
