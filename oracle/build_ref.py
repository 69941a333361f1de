"""Compile the reference's own CUDA extensions for sm_100a into oracle/_ref/.

Test/benchmark infrastructure only: the two pybind CUDA files of the reference
(cst_ssm/ops/csrc/eacs_scan_cuda.cu, eacs_cell_cuda.cu) are compiled where
they lie in the reference checkout, with torch.utils.cpp_extension (the same
toolchain the reference's JIT loader uses) and an explicit sm_100a target.
Outputs go to oracle/_ref/ only (git-ignored; they travel to the GPU machine
with the working tree).  bench.py times them beside this project's kernels.

    python oracle/build_ref.py [--reference <checkout>]

The checkout defaults to CST_SSM_REFERENCE, else `reference` beside the repository.
"""
from __future__ import annotations

import argparse
import os

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get(
        "CST_SSM_REFERENCE", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")))
    args = ap.parse_args()
    from torch.utils.cpp_extension import load
    csrc = os.path.join(args.reference, "cst_ssm", "ops", "csrc")
    os.makedirs(OUT, exist_ok=True)
    flags = ["-O3", "-gencode", "arch=compute_100a,code=sm_100a"]
    for name, src in (("ref_eacs_scan_cuda", "eacs_scan_cuda.cu"),
                      ("ref_eacs_cell_cuda", "eacs_cell_cuda.cu")):
        bdir = os.path.join(OUT, name)
        os.makedirs(bdir, exist_ok=True)
        load(name=name, sources=[os.path.join(csrc, src)], extra_cuda_cflags=flags,
             build_directory=bdir, verbose=False)
        print("built", os.path.join(bdir, name + ".so"))


if __name__ == "__main__":
    main()
