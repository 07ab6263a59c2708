"""Build libsma.so (the C-ABI library with the sm_100a kernels) in-tree.

Usage:  python build.py [--verbose] [--ptxas-info]

Each csrc/*.cu is compiled with nvcc for sm_100a only into _build/, then
linked into libsma.so next to this file.  The CUDA runtime is linked
statically and the driver API (cuTensorMapEncodeTiled) is reached through
cudaGetDriverEntryPoint, so the library loads without a GPU or libcuda and
depends on nothing but the C/C++ runtime.
"""

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD_DIR = os.path.join(HERE, "_build")
LIB_PATH = os.path.join(HERE, "libsma.so")

SOURCES = ["sma_capi.cu", "pack_mask.cu", "attn_fwd.cu", "attn_fwd_chain.cu", "tma_map.cu", "attn_bwd.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I",
    INCLUDE,
    "-I",
    CSRC,
]


def _nvcc():
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libsma.so")
    return nvcc


def _newest_input_mtime():
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    paths.append(os.path.abspath(__file__))
    return max(os.path.getmtime(p) for p in paths)


def up_to_date():
    return os.path.exists(LIB_PATH) and os.path.getmtime(LIB_PATH) >= _newest_input_mtime()


def build(verbose=False, ptxas_info=False, force=False):
    """Compile libsma.so if any source is newer than it; return its path."""
    if not force and not ptxas_info and up_to_date():
        return LIB_PATH
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)

    def compile_one(src):
        obj = os.path.join(BUILD_DIR, os.path.splitext(src)[0] + ".o")
        cmd = [nvcc, "-c", os.path.join(CSRC, src), "-o", obj] + ARCH_FLAGS + COMMON_FLAGS
        if ptxas_info:
            cmd += ["-Xptxas", "-v"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
        return obj, res.stdout + res.stderr

    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(compile_one, SOURCES))
    if verbose or ptxas_info:
        for _, log in results:
            if log.strip():
                print(log)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, "-shared", "-o", tmp] + [o for o, _ in results] + ARCH_FLAGS + ["-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, ptxas_info=a.ptxas_info, force=a.force or a.ptxas_info))
    sys.exit(0)
