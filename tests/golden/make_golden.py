"""Generate the golden vectors that pin the CPU oracle to the reference itself.

Run (needs the reference checkout, only on the build machine):
    python tests/golden/make_golden.py [--ref /path/to/W4A16-GEMM]

It imports the reference's own ``tests/quant.py`` (akshay919191/W4A16-GEMM)
and records its outputs for seeded inputs:

* ``pack_*``      -- q codes and ``pack_int4(q)`` (tests/quant.py:34-48)
* ``quant_*``     -- ``quantize_w4(W, G)`` and ``dequantize_w4`` (tests/quant.py:62-80)
* ``gemm_*``      -- ``ref_gemm(x, q, scales, G)`` (tests/quant.py:83-85)
* ``cfg0_*``      -- the BASELINE configs[0] workload (M=1, N=K=4096, G=128, seed 0):
                    SHA-256 of the packed weights / scales / activations and the
                    full fp32 reference output.

The fixture ``golden.npz`` is committed; nothing at test time reads the
reference checkout.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference_quant(ref_root: str):
    path = os.path.join(ref_root, "tests", "quant.py")
    spec = importlib.util.spec_from_file_location("ref_quant", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def workload(M, N, K, G, seed):
    """Seeded inputs in the BASELINE draw order: x ~ N(0,1) fp16, q ~ U{0..15},
    scales ~ U[0.002, 0.02] fp16 [K/G, N]."""
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=gen).half()
    q = torch.randint(0, 16, (N, K), generator=gen, dtype=torch.uint8)
    scales = (torch.rand(K // G, N, generator=gen) * 0.018 + 0.002).half()
    return x, q, scales


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().numpy().tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("W4A16_REF"),
                    help="reference checkout to import tests/quant.py from (or $W4A16_REF)")
    ap.add_argument("--out", default=os.path.join(HERE, "golden.npz"))
    args = ap.parse_args()
    if not args.ref:
        ap.error("pass --ref <reference checkout> or set W4A16_REF")
    rq = load_reference_quant(args.ref)
    out = {}

    # 1. packing, several shapes incl. ones that are not multiples of 64 / 512
    for i, (N, K) in enumerate([(16, 64), (32, 128), (48, 192), (64, 512), (80, 640), (208, 384)]):
        gen = torch.Generator().manual_seed(100 + i)
        q = torch.randint(0, 16, (N, K), generator=gen, dtype=torch.uint8)
        out[f"pack_{N}x{K}_q"] = q.numpy()
        out[f"pack_{N}x{K}_wp"] = rq.pack_int4(q).numpy()

    # 2. quantizer + dequant for both group sizes
    for G in (64, 128):
        gen = torch.Generator().manual_seed(200 + G)
        W = torch.randn(64, 512, generator=gen) * 0.02
        q, s = rq.quantize_w4(W, G)
        out[f"quant_G{G}_W"] = W.numpy()
        out[f"quant_G{G}_q"] = q.numpy()
        out[f"quant_G{G}_scales"] = s.numpy()
        out[f"quant_G{G}_deq"] = rq.dequantize_w4(q, s, G).numpy()

    # 3. reference GEMM on small seeded problems (ragged M, both G)
    for (M, N, K, G) in [(1, 64, 512, 64), (3, 128, 1024, 128), (17, 80, 640, 64), (16, 208, 384, 128)]:
        x, q, s = workload(M, N, K, G, seed=7)
        key = f"gemm_{M}x{N}x{K}_G{G}"
        out[key + "_x"] = x.numpy()
        out[key + "_wp"] = rq.pack_int4(q).numpy()
        out[key + "_scales"] = s.numpy()
        out[key + "_y"] = rq.ref_gemm(x, q, s, G).numpy()

    # 4. checksums of the full-size inputs and the full output
    x, q, s = workload(1, 4096, 4096, 128, seed=0)
    wp = rq.pack_int4(q)
    out["cfg0_sha_wp"] = np.array(sha(wp))
    out["cfg0_sha_scales"] = np.array(sha(s))
    out["cfg0_sha_x"] = np.array(sha(x))
    out["cfg0_y"] = rq.ref_gemm(x, q, s, 128).numpy()

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays, {os.path.getsize(args.out)} bytes")


if __name__ == "__main__":
    sys.exit(main())
