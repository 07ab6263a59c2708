"""Cross-check against the reference's own CUDA kernels, built from the
reference sources into oracle/_ref/libref_sma.so (oracle/build_ref.py), on
identical inputs at every workload's full size: pack_mask bit for bit,
attention output within the stated tolerance plus one output ulp (both
outputs are rounded to the input dtype), LSE within 2e-3."""

import ctypes
import math
import os

import pytest
import torch

from conftest import FLT_MAX, LSE_TOL, OUT_TOL, REPO, record_parity, ulp
from python import pack_mask, sparse_attn_cuda, workloads

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
REF_LIB = os.path.join(REPO, "oracle", "_ref", "libref_sma.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF_LIB):
        pytest.skip("reference kernel library not built (oracle/build_ref.py)")
    lib = ctypes.CDLL(REF_LIB)
    vp = ctypes.c_void_p
    lib.ref_pack_mask.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp]
    lib.ref_attn_fwd.argtypes = [ctypes.c_int, vp, vp, vp, vp, vp, vp] + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_int, vp]
    return lib


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("name", ["c1", "c2", "c3", "c4", "c5"])
def test_matches_reference_kernel(ref, name):
    q, k, v, m = workloads.make_inputs(name, seed=9, device=DEV)
    B, H, N, D = q.shape
    packed_ref = torch.zeros(B, H, N, (N + 31) // 32, dtype=torch.int32, device=DEV)
    assert ref.ref_pack_mask(m.data_ptr(), packed_ref.data_ptr(), B, H, N, _stream()) == 0
    packed = pack_mask(m)
    assert torch.equal(packed, packed_ref)

    scale = 1.0 / math.sqrt(D)
    out_ref = torch.empty_like(q)
    lse_ref = torch.empty(B, H, N, dtype=torch.float32, device=DEV)
    bf = 1 if q.dtype == torch.bfloat16 else 0
    assert ref.ref_attn_fwd(bf, q.data_ptr(), k.data_ptr(), v.data_ptr(), packed_ref.data_ptr(), out_ref.data_ptr(),
                            lse_ref.data_ptr(), B, H, N, D, scale, 1, _stream()) == 0
    out = torch.empty_like(q)
    lse = torch.empty(B, H, N, dtype=torch.float32, device=DEV)
    sparse_attn_cuda.forward(q, k, v, packed, out, lse, scale, True)
    sparse_attn_cuda.device_status()
    diff = (out.float() - out_ref.float()).abs()
    bound = OUT_TOL[q.dtype] + ulp(out_ref.float(), q.dtype)
    err = diff.max().item()
    record_parity(f"{name} vs reference CUDA kernel", max_abs_out=err)
    assert (diff <= bound).all(), f"{name}: max |ours - reference kernel| = {err}"
    empty = lse_ref == -FLT_MAX
    assert torch.equal(empty, lse == -FLT_MAX)
    assert (lse[~empty] - lse_ref[~empty]).abs().max().item() <= LSE_TOL
