import glob
import json
import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "sparse-mask-attention-auto-research_b200")
GOLDEN_DIR = os.path.join(REPO, "tests", "golden")
for p in (REPO, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)

# Tolerances on |out - fp32 reference| (the stated bar): fp16 a flat 2e-3;
# bf16 1e-2 plus half a bf16 ulp of the reference value, because a correctly
# rounded bf16 output of a value in [4, 8) may already sit 2^-6 = 0.0156 from
# the FP32 value, above a flat 1e-2 (out_bound below).
OUT_TOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2}
_MANT_BITS = {torch.float16: 10, torch.bfloat16: 7}
_HALF_ULP_ALLOWANCE = {torch.float16: False, torch.bfloat16: True}


def ulp(x, dtype):
    """Spacing of `dtype` values at |x| (normal range)."""
    e = torch.floor(torch.log2(x.abs().clamp_min(2.0 ** -14)))
    return torch.pow(2.0, e - _MANT_BITS[dtype])


def out_bound(ref, dtype):
    """Elementwise bound on |out - ref| for an output rounded to `dtype`."""
    if not _HALF_ULP_ALLOWANCE[dtype]:
        return torch.full_like(ref, OUT_TOL[dtype])
    return OUT_TOL[dtype] + 0.5 * ulp(ref, dtype)


def record_parity(name, **values):
    """Print a per-case parity figure and, when SMA_PARITY_REPORT names a
    file, append it there as one JSON line."""
    line = {"case": name, **values}
    print("PARITY " + json.dumps(line))
    path = os.environ.get("SMA_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(line) + "\n")
# LSE is written in FP32 from FP32 accumulators: absolute tolerance.
LSE_TOL = 2e-3
FLT_MAX = float(np.finfo(np.float32).max)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libsma.so")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def _from_bits(u16, dtype):
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).view(dtype)


def load_golden(path):
    """A golden case as a dict of torch tensors (CPU) + meta."""
    z = np.load(path)
    meta = json.loads(str(z["meta"]))
    n = int(z["n"])
    mask = np.unpackbits(z["mask"], axis=-1, bitorder="little")[..., :n].astype(bool)
    case = dict(meta=meta, mask=torch.from_numpy(mask))
    if "packed" in z:
        case["packed"] = torch.from_numpy(z["packed"])
    if meta["kind"] == "attention":
        dtype = getattr(torch, meta["dtype"])
        case.update(
            q=_from_bits(z["q"], dtype),
            k=_from_bits(z["k"], dtype),
            v=_from_bits(z["v"], dtype),
            out=torch.from_numpy(z["out"]),
            lse=torch.from_numpy(z["lse"]),
            dtype=dtype,
        )
    elif meta["kind"] == "backward":
        dtype = getattr(torch, meta["dtype"])
        case.update(
            q=_from_bits(z["q"], dtype),
            k=_from_bits(z["k"], dtype),
            v=_from_bits(z["v"], dtype),
            dout=_from_bits(z["dout"], dtype),
            lse=torch.from_numpy(z["lse"]),
            dq=torch.from_numpy(z["dq"]),
            dk=torch.from_numpy(z["dk"]),
            dv=torch.from_numpy(z["dv"]),
            dtype=dtype,
        )
    return case


def golden_paths(kind):
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, f"{kind}_*.npz")))


def golden_path(name):
    return os.path.join(GOLDEN_DIR, name + ".npz")


def golden_ids(kind):
    return [os.path.basename(p)[:-4] for p in golden_paths(kind)]
