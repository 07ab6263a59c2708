"""ORACLE — test infrastructure only.

Compile the reference's own CUDA kernels (csrc/sparse_attention.cu from the
mounted reference) plus oracle/ref_shim.cu into oracle/_ref/libref_sma.so
for use as a GPU-side checker in the GPU tests.  The reference sources are
compiled where they lie (nothing is copied into this repository), with the
flags of the reference's JIT build (run.py:129-147: -O3 --use_fast_math)
retargeted to sm_100a.  Outputs go to oracle/_ref/ only (git-ignored; the
built .so travels with the working tree to GPU machines).

    python oracle/build_ref.py --reference <reference root>
    (or SMA_REFERENCE_ROOT=<reference root> python oracle/build_ref.py)

The root the library was built from is recorded in oracle/_ref/reference_root.txt
(tests that import the reference's Python module on the CPU machine read it
there; GPU machines have no copy of the reference and do not need it).
"""

import argparse
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libref_sma.so")
ROOT_RECORD = os.path.join(OUT_DIR, "reference_root.txt")


def recorded_reference_root():
    """The reference root of the last build, if it is still present here."""
    if not os.path.exists(ROOT_RECORD):
        return None
    with open(ROOT_RECORD) as f:
        root = f.read().strip()
    return root if os.path.isdir(os.path.join(root, "python")) else None


def build(reference, force=False):
    csrc = os.path.join(reference, "csrc")
    ref_cu = os.path.join(csrc, "sparse_attention.cu")
    shim = os.path.join(HERE, "ref_shim.cu")
    inputs = [ref_cu, os.path.join(csrc, "sparse_attention.h"), os.path.join(csrc, "utils.cuh"), shim]
    os.makedirs(OUT_DIR, exist_ok=True)
    with open(ROOT_RECORD, "w") as f:
        f.write(os.path.abspath(reference) + "\n")
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(p) for p in inputs):
        return LIB
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [
        nvcc, "-O3", "--use_fast_math", "-std=c++17",
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
        "-I", csrc, shim, ref_cu, "-o", LIB,
    ]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference kernel build failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def build_if_available(reference):
    """Build when the reference sources are present; otherwise keep whatever
    prebuilt library is already in oracle/_ref/ (GPU machines have no mount)."""
    if reference and os.path.isdir(os.path.join(reference, "csrc")):
        return build(reference)
    return LIB if os.path.exists(LIB) else None


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SMA_REFERENCE_ROOT"),
                    help="root of the reference checkout (default: $SMA_REFERENCE_ROOT)")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    if not a.reference:
        ap.error("name the reference root with --reference or SMA_REFERENCE_ROOT")
    print(build(a.reference, a.force))
