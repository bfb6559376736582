"""The decode kernel's stream-K partition, checked on the host.

``partition_check.cpp`` includes the partition header the kernels are built from
(csrc/decode_partition.h) and walks every CTA's range the way decode_kernel does, for
some 5800 (N, K, #SMs) cases: unit coverage, the first/last-CTA closed forms, direct
writes versus partial slots, and the slots decode_combine_kernel reads.  It plays the
role the reference's numpy emulation of its kernel's data flow plays
(akshay919191/W4A16-GEMM tests/layout.py) for this kernel's work split.
"""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "w4a16-gemm_b200", "csrc")


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_decode_partition(tmp_path):
    exe = tmp_path / "partition_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-Wall", "-Werror", "-I", CSRC,
                    os.path.join(HERE, "partition_check.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok ")
