"""Build libpad_b200.so (the C-ABI decode library) in-tree with nvcc for sm_100a,
and _pad_torch_ops.so, the thin torch operator library over it
(torch.ops.pad_b200.*, csrc/pad_torch_op.cpp, host C++ only).

    python paged-attention-decode_b200/pad_b200/build.py   # (runs without importing pad_b200)

Both libraries are written next to this file so that they travel with the
source tree; nothing is installed into site-packages.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(HERE)
REPO = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_NAME = "libpad_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
OPS_PATH = os.path.join(HERE, "_pad_torch_ops.so")
SOURCES = ["pad_decode.cu", "pad_kv_append.cu"]
OPS_SOURCE = "pad_torch_op.cpp"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libpad_b200.so")
    return cand


def _inputs():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
    files.append(os.path.join(INCLUDE, "pad_b200.h"))
    return files


def _stale(target: str, inputs) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(f) > t for f in inputs)


def needs_build() -> bool:
    return _stale(LIB_PATH, _inputs()) or _stale(OPS_PATH, [os.path.join(CSRC, OPS_SOURCE), LIB_PATH])


def _build_ops() -> None:
    """g++ the torch operator library against this interpreter's torch."""
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths(device_type="cuda")
    libdirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-fPIC", "-shared", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", INCLUDE, *[f"-I{p}" for p in inc], os.path.join(CSRC, OPS_SOURCE), "-o", OPS_PATH + ".tmp",
           *[f"-L{p}" for p in libdirs], f"-L{HERE}", "-lpad_b200", "-lc10", "-lc10_cuda", "-ltorch_cpu",
           "-ltorch_cuda", "-ltorch", "-lcudart", "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{p}" for p in libdirs]]
    subprocess.run(cmd, check=True, cwd=CSRC)
    os.replace(OPS_PATH + ".tmp", OPS_PATH)


def build(force: bool = False, verbose: bool = False) -> str:
    if force or _stale(LIB_PATH, _inputs()):
        cmd = [_nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
               "-shared", "-I", INCLUDE, "-o", LIB_PATH + ".tmp"]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        cmd += [os.path.join(CSRC, s) for s in SOURCES]
        subprocess.run(cmd, check=True, cwd=CSRC)
        os.replace(LIB_PATH + ".tmp", LIB_PATH)
    if force or _stale(OPS_PATH, [os.path.join(CSRC, OPS_SOURCE), LIB_PATH]):
        _build_ops()
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
