"""Build the W4A16 B200 extension in-tree.

    python w4a16-gemm_b200/build.py [--force]

Produces, next to the Python package ``w4a16_opt``:

* ``w4a16_opt/libw4a16.so``  -- the C-ABI library (include/w4a16.h): all
  kernels, compiled by nvcc for sm_100a only;
* ``w4a16_opt/_C<ext>.so``   -- the thin PyTorch binding over that library.

nvcc cross-compiles without a GPU, so this runs on a CPU-only machine too.
Outputs are rebuilt only when a source is newer (or with --force).
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys
import sysconfig

PKG_ROOT = os.path.dirname(os.path.abspath(__file__))
REPO_ROOT = os.path.dirname(PKG_ROOT)
CSRC = os.path.join(PKG_ROOT, "csrc")
OUT_DIR = os.path.join(PKG_ROOT, "w4a16_opt")
INCLUDE = os.path.join(REPO_ROOT, "include")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3"]

LIB_PATH = os.path.join(OUT_DIR, "libw4a16.so")
EXT_PATH = os.path.join(OUT_DIR, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def _sources(patterns):
    out = []
    for p in patterns:
        out += glob.glob(os.path.join(CSRC, p))
    out += glob.glob(os.path.join(INCLUDE, "*.h"))
    return out


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    print("+ " + " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build_library(force=False):
    deps = _sources(["*.cu", "*.cuh", "*.h", "capi.cpp"]) + [__file__]
    if not force and not _stale(LIB_PATH, deps):
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    _run([NVCC, *ARCH_FLAGS, *NVCC_FLAGS, "-shared", "-I", INCLUDE,
          os.path.join(CSRC, "kernels.cu"), os.path.join(CSRC, "capi.cpp"), "-o", tmp])
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def build_torch_binding(force=False):
    import torch
    from torch.utils import cpp_extension as ce

    deps = [os.path.join(CSRC, "torch_ext.cpp"), LIB_PATH, __file__] + glob.glob(os.path.join(INCLUDE, "*.h"))
    if not force and not _stale(EXT_PATH, deps):
        return EXT_PATH
    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], INCLUDE]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared",
           "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in incs], os.path.join(CSRC, "torch_ext.cpp"), "-o", EXT_PATH + ".tmp",
           *[f"-L{p}" for p in libdirs], "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda",
           "-ltorch_cuda", f"-L{OUT_DIR}", "-lw4a16", "-Wl,-rpath,$ORIGIN"]
    _run(cmd)
    os.replace(EXT_PATH + ".tmp", EXT_PATH)
    return EXT_PATH


def build(force=False):
    build_library(force)
    build_torch_binding(force)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    build(args.force)
    sys.exit(0)
