"""Install the reference's Python package (cst_ssm) into baseline/_ref/.

Test/benchmark infrastructure only: the unmodified reference package, so that
the GPU tests can run the reference's own layers on CUDA beside this
project's kernels and bench.py can time the reference's own CPU path.  The
checkout is copied to a temporary directory first (its setup.py writes build
files next to itself and the checkout may be read-only) and installed with
pip --target, offline, without its dependencies (torch and numpy are already
present).  Without a GPU visible its setup.py builds no CUDA extension; the
reference's kernels are built by build_ref.py instead.

    python oracle/install_ref.py [--reference <checkout>] [--target baseline/_ref]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get(
        "CST_SSM_REFERENCE", os.path.join(os.path.dirname(REPO), "reference")))
    ap.add_argument("--target", default=os.path.join(REPO, "baseline", "_ref"))
    args = ap.parse_args()
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "reference")
        shutil.copytree(args.reference, src, ignore=shutil.ignore_patterns(".git", "*.pyc", "__pycache__"))
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", args.target, src]
        env = dict(os.environ, FORCE_CUDA="0", CUDA_VISIBLE_DEVICES="")
        subprocess.run(cmd, check=True, env=env)
    print("installed", os.path.join(args.target, "cst_ssm"))


if __name__ == "__main__":
    main()
