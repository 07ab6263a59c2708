"""sma_attn_bwd_noalloc: the backward with the library's fixed device
scratch instead of caller-provided buffers.  Two calls in a row must give
the results of sma_attn_bwd (sparse_attn_cuda.backward, caller scratch):
dk and dv bit for bit, dq up to the order of the FP32 partial-sum atomics."""

import math

import pytest
import torch

from python import _lib, pack_mask, sparse_attn_cuda, workloads

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _inputs(seed, name="c1", B=2, H=3):
    q, k, v, m = workloads.make_inputs(name, seed=seed, device=DEV, B=B, H=H)
    g = torch.Generator(device=DEV).manual_seed(seed + 100)
    dout = torch.randn(q.shape, generator=g, device=DEV).to(q.dtype)
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D)
    packed = pack_mask(m)
    out = torch.empty_like(q)
    lse = torch.empty(B, H, N, device=DEV, dtype=torch.float32)
    sparse_attn_cuda.forward(q, k, v, packed, out, lse, scale, True)
    return q, k, v, out, dout, lse, packed, scale


def _noalloc(q, k, v, out, dout, lse, packed, scale, dq, dk, dv):
    lib = _lib.load()
    B, H, N, D = q.shape
    dtype = _lib.SMA_DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.SMA_DTYPE_FP16
    return lib.sma_attn_bwd_noalloc(
        dtype, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(),
        lse.data_ptr(), packed.data_ptr(), dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), B, H, N, D, scale,
        torch.cuda.current_stream().cuda_stream,
    )


def _check_case(seed, name="c1", B=2, H=3):
    q, k, v, out, dout, lse, packed, scale = _inputs(seed, name, B, H)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    assert _noalloc(q, k, v, out, dout, lse, packed, scale, dq, dk, dv) == _lib.SMA_OK
    sparse_attn_cuda.device_status()
    dq_r, dk_r, dv_r = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    sparse_attn_cuda.backward(dout, q, k, v, out, lse, packed, dq_r, dk_r, dv_r, scale)
    sparse_attn_cuda.device_status()
    assert torch.equal(dk, dk_r) and torch.equal(dv, dv_r)
    big = float(dq_r.float().abs().max())
    assert float((dq.float() - dq_r.float()).abs().max()) <= 2e-3 * big


def test_two_calls_in_a_row_match_the_allocating_entry():
    for seed in (1, 2):
        _check_case(seed)


def test_bf16_head_dim_128():
    """The block-sparse bf16 recipe at head dim 128, two calls in a row."""
    for seed in (3, 4):
        _check_case(seed, "c3", B=1, H=2)


def test_largest_accepted_problem():
    """252 heads of N = 512, D = 64: B*H*N*(D+1) is just under the 8 Mi floats
    of the scratch, so Delta ends at its last 129 KiB."""
    heads = (8 << 20) // (512 * 65)
    assert heads * 512 * 65 <= 8 << 20 < (heads + 1) * 512 * 65
    for seed in (5, 6):
        _check_case(seed, "c1", B=1, H=heads)


def test_oversize_input_is_rejected():
    lib = _lib.load()
    t = torch.zeros(16, device=DEV, dtype=torch.float16)
    p = t.data_ptr()
    # 64 * 64 heads * 1024 rows * 65 floats is far above the 32 MiB scratch.
    rc = lib.sma_attn_bwd_noalloc(_lib.SMA_DTYPE_FP16, p, p, p, p, p, p, p, p, p, p, 64, 64, 1024, 64, 0.125, None)
    assert rc == _lib.SMA_ERR_ARG
    assert b"scratch" in lib.sma_last_error()
