"""Host-side checks of sparse_attention_from_host (no GPU needed): device
tensors, dtypes and shapes are refused before any copy, and the slice count
rule."""

import pytest
import torch

from python.streaming import default_slices, slice_bounds, sparse_attention_from_host


def _host(N=64, D=64, dtype=torch.float16):
    q = torch.randn(1, 2, N, D).to(dtype)
    return q, q.clone(), q.clone(), torch.rand(1, 2, N, N) < 0.5


def test_rejects_bad_arguments():
    q, k, v, m = _host()
    with pytest.raises(RuntimeError, match="Unsupported dtype"):
        sparse_attention_from_host(q.float(), k.float(), v.float(), m)
    with pytest.raises(RuntimeError, match="same shape"):
        sparse_attention_from_host(q, k[:, :1], v, m)
    with pytest.raises(RuntimeError, match="mask must be a bool"):
        sparse_attention_from_host(q, k, v, m.int())
    with pytest.raises(RuntimeError, match="mask must be a bool"):
        sparse_attention_from_host(q, k, v, m[..., :32])
    with pytest.raises(RuntimeError, match="4D"):
        sparse_attention_from_host(q[0], k[0], v[0], m[0])
    with pytest.raises(RuntimeError, match="out must be"):
        sparse_attention_from_host(q, k, v, m, out=torch.empty(1, 2, 64, 32, dtype=q.dtype))


def test_default_slices():
    # About 20 MB of inputs per slice, at most 8, at most one per head.
    mb = 1 << 20
    assert default_slices(192, 88 * mb) == 4    # B16 H12 N512 D64 fp16
    assert default_slices(768, 50 * mb) == 2    # B64 H12 N128 D64
    assert default_slices(256, 469 * mb) == 8   # B8 H32 N1024 D128 bf16
    assert default_slices(1, 469 * mb) == 1     # one head
    assert default_slices(16, 1 * mb) == 1      # small inputs


def test_slice_bounds_decrease_and_cover():
    assert slice_bounds(192, 4) == [0, 76, 134, 172, 192]   # 76, 58, 38, 20 heads
    assert slice_bounds(14, 4) == [0, 5, 9, 12, 14]
    assert slice_bounds(3, 1) == [0, 3]
    for bh in (1, 2, 7, 192, 4096):
        for n in range(1, 9):
            b = slice_bounds(bh, n)
            assert b[0] == 0 and b[-1] == bh and all(x <= y for x, y in zip(b, b[1:]))
