"""Build the sm_100a C-ABI library ``_lib/libfrsa.so`` and the PyTorch C++
extension over it (``_lib/torch_ext/frsa_torch_ext*.so``), both in-tree.

    python -m triton_fused_rope_flash_attn_b200.build [--force]

The library is one translation unit (``csrc/frsa_api.cu`` includes the kernel
files). It links only the CUDA runtime; the TMA tensor-map encoder is fetched
from the driver at run time. The extension (``csrc/frsa_torch.cpp``) is the
host side of the product path; it binds the C-ABI entry points of the loaded
library at run time, so it does not link against it.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG_DIR, "csrc")
REPO = os.path.dirname(PKG_DIR)
INCLUDE = os.path.join(REPO, "include")
LIB_DIR = os.path.join(PKG_DIR, "_lib")
LIB_PATH = os.path.join(LIB_DIR, "libfrsa.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-shared", "-Xcompiler", "-fPIC",
    "-cudart", "shared",
]


def _sources():
    out = [os.path.join(INCLUDE, "frsa.h")]
    for name in sorted(os.listdir(CSRC)):
        if name.endswith((".cu", ".cuh", ".h")):
            out.append(os.path.join(CSRC, name))
    return out


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libfrsa.so")


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(s) <= t for s in _sources())


def build_library(force: bool = False, verbose: bool = False) -> str:
    """Compile ``libfrsa.so`` unless it is newer than every source. Returns its path."""
    if not force and up_to_date():
        return LIB_PATH
    os.makedirs(LIB_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [_nvcc(), *NVCC_FLAGS, "-I", INCLUDE, "-o", tmp, os.path.join(CSRC, "frsa_api.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stdout, res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH





TORCH_EXT_NAME = "frsa_torch_ext"
TORCH_EXT_DIR = os.path.join(LIB_DIR, "torch_ext")
TORCH_EXT_SRC = os.path.join(CSRC, "frsa_torch.cpp")


def build_torch_ext(verbose: bool = False):
    """Compile (or load the up-to-date build of) the PyTorch extension; returns the module."""
    import torch.utils.cpp_extension as ce
    os.makedirs(TORCH_EXT_DIR, exist_ok=True)
    return ce.load(name=TORCH_EXT_NAME, sources=[TORCH_EXT_SRC], extra_include_paths=[INCLUDE],
                   extra_cflags=["-O3", "-std=c++17"], build_directory=TORCH_EXT_DIR,
                   with_cuda=True, verbose=verbose)


if __name__ == "__main__":
    print(build_library(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_torch_ext(verbose="-v" in sys.argv).__file__)
