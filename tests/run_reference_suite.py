"""Run the reference project's own, unmodified test suite against this package.

The reference's tests (tests/test_w4a16.py with its conftest.py and quant.py) import the
operator module as ``w4a16_opt``.  This script copies that test directory from a reference
checkout into a scratch directory, puts this repository's package directory first on
``PYTHONPATH`` (so ``import w4a16_opt`` is this build's module) and runs pytest there on the
current GPU.  Nothing is edited: a pass shows that the drop-in boundary needs no change to
the reference's callers or tests.

    python tests/run_reference_suite.py --reference <reference checkout> [-- extra pytest args]

The checkout comes from ``--reference`` or the W4A16_REFERENCE_DIR environment variable; there
is no default.  It is not part of ``pytest -m gpu``, since the reference's sources do not
travel with this repository.
"""
import argparse
import os
import shutil
import subprocess
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "w4a16-gemm_b200")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("W4A16_REFERENCE_DIR"),
                    help="reference checkout (holds tests/test_w4a16.py)")
    ap.add_argument("pytest_args", nargs="*", help="passed to pytest after the test file")
    args = ap.parse_args(argv)
    if not args.reference:
        ap.error("give --reference or set W4A16_REFERENCE_DIR")
    src = os.path.join(args.reference, "tests")
    if not os.path.isfile(os.path.join(src, "test_w4a16.py")):
        ap.error(f"{src}/test_w4a16.py not found")
    with tempfile.TemporaryDirectory(prefix="w4a16_refsuite_") as tmp:
        dst = os.path.join(tmp, "tests")
        shutil.copytree(src, dst, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
        env = dict(os.environ)
        env["PYTHONPATH"] = os.pathsep.join([PKG] + [p for p in env.get("PYTHONPATH", "").split(os.pathsep) if p])
        cmd = [sys.executable, "-m", "pytest", "tests/test_w4a16.py", "-q", "-rs", "-p", "no:cacheprovider",
               *args.pytest_args]
        return subprocess.call(cmd, cwd=tmp, env=env)


if __name__ == "__main__":
    sys.exit(main())
