"""TEST INFRASTRUCTURE ONLY -- builds the reference's own CUDA extension as a checker.

    python oracle/build_ref.py [--force]

Compiles akshay919191/W4A16-GEMM's extension (src/vectorized/kernel.cu and
src/vectorized/extension.cpp, with the headers beside them) for sm_100a, reading
the sources where they lie, into ``oracle/_ref/w4a16_ref<ext>.so``: a torch
extension module named ``w4a16_ref`` whose ``w4a16_gemm(Wp, x, scales, variant)``
is the reference implementation.  GPU parity tests compare the product against
it on the same inputs.  Nothing here is imported by the product, and no
reference source is copied into this repository.

The reference directory comes from the ``reference_dir`` argument or
$W4A16_REFERENCE_DIR; there is no default.  Without either, or where the directory
is absent (as on a GPU box, which only receives the prebuilt module), this is a
no-op.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
MODULE = "w4a16_ref"
OUT_PATH = os.path.join(OUT_DIR, MODULE + sysconfig.get_config_var("EXT_SUFFIX"))
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def reference_dir(explicit=None):
    """The reference checkout: the argument, else $W4A16_REFERENCE_DIR, else None."""
    return explicit or os.environ.get("W4A16_REFERENCE_DIR") or None


def _run(cmd):
    print("+ " + " ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def build(force=False, ref_dir=None):
    src = os.path.join(reference_dir(ref_dir), "src", "vectorized")
    kernel, ext = os.path.join(src, "kernel.cu"), os.path.join(src, "extension.cpp")
    deps = [kernel, ext] + [os.path.join(src, h) for h in ("common.cuh", "decode.cuh", "prefill.cuh")]
    if not force and os.path.exists(OUT_PATH) and all(os.path.getmtime(d) <= os.path.getmtime(OUT_PATH) for d in deps):
        return OUT_PATH
    import torch
    from torch.utils import cpp_extension as ce

    os.makedirs(OUT_DIR, exist_ok=True)
    incs = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    k_obj, e_obj = os.path.join(OUT_DIR, "kernel.o"), os.path.join(OUT_DIR, "extension.o")
    # the reference's own flags (setup.py: -O3 -std=c++17 -lineinfo, plus the flags torch's
    # CUDAExtension adds to every nvcc command), arch sm_100a
    _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo",
          *ce.COMMON_NVCC_FLAGS, "-Xcompiler", "-fPIC", *defs, *[f"-I{p}" for p in incs], "-c", kernel, "-o", k_obj])
    _run(["g++", "-O3", "-std=c++17", "-fPIC", *defs, *[f"-I{p}" for p in incs], "-c", ext, "-o", e_obj])
    _run(["g++", "-shared", k_obj, e_obj, "-o", OUT_PATH + ".tmp", *[f"-L{p}" for p in libdirs],
          "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
          "-L/usr/local/cuda/lib64", "-lcudart"])
    os.replace(OUT_PATH + ".tmp", OUT_PATH)
    for f in (k_obj, e_obj):
        os.remove(f)
    return OUT_PATH


def build_if_available(force=False, ref_dir=None):
    """Build when the reference sources are present; report and skip otherwise."""
    root = reference_dir(ref_dir)
    if not root or not os.path.isdir(os.path.join(root, "src", "vectorized")):
        print("oracle/build_ref.py: reference sources not present; skipping (prebuilt module used if any)")
        return None
    try:
        return build(force, root)
    except (subprocess.CalledProcessError, OSError) as exc:   # checker only: never blocks the product build
        print(f"oracle/build_ref.py: reference extension did not build: {exc}")
        return None


def load():
    """The reference module if it was built, else None (tests skip on None)."""
    if not os.path.exists(OUT_PATH):
        return None
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (libtorch before the extension)
    loader = importlib.machinery.ExtensionFileLoader(MODULE, OUT_PATH)
    spec = importlib.util.spec_from_file_location(MODULE, OUT_PATH, loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--reference", default=None, help="reference checkout (else $W4A16_REFERENCE_DIR)")
    a = ap.parse_args()
    print(build_if_available(a.force, a.reference))
