"""The oracle pinned against the reference's own outputs (tests/golden/, made
by running the reference's CPU code).  CPU only."""

import numpy as np
import pytest
import torch

from conftest import FLT_MAX, golden_ids, golden_path, golden_paths, load_golden
from oracle import oracle


@pytest.mark.parametrize("path", golden_paths("pack") + golden_paths("attn"), ids=golden_ids("pack") + golden_ids("attn"))
def test_pack_bit_exact_vs_reference(path):
    case = load_golden(path)
    got = oracle.pack_mask(case["mask"].numpy())
    want = case["packed"].numpy()
    assert got.dtype == np.int32
    assert got.shape == want.shape
    assert np.array_equal(got, want)


@pytest.mark.parametrize("path", golden_paths("pack"), ids=golden_ids("pack"))
def test_unpack_roundtrip(path):
    case = load_golden(path)
    n = case["mask"].shape[-1]
    assert np.array_equal(oracle.unpack_mask(case["packed"].numpy(), n), case["mask"].numpy())


def test_bit31_is_sign_bit():
    case = load_golden(golden_path("pack_bit31"))
    p = oracle.pack_mask(case["mask"].numpy())
    assert (p == np.int32(-2147483648)).all()


@pytest.mark.parametrize("path", golden_paths("attn"), ids=golden_ids("attn"))
def test_attention_vs_reference(path):
    case = load_golden(path)
    scale = case["meta"]["scale"]
    q, k, v, m = (case[x].float().numpy() for x in ("q", "k", "v", "mask"))
    out = oracle.attention(q, k, v, m, scale)
    np.testing.assert_allclose(out, case["out"].numpy(), atol=2e-5, rtol=1e-4)
    lse = oracle.lse(q, k, m, scale)
    want = case["lse"].numpy().copy()
    want[np.isneginf(want)] = -FLT_MAX  # reference CUDA convention for empty rows
    np.testing.assert_allclose(lse, want, atol=2e-5, rtol=1e-5)


def test_parallel_matches_serial():
    case = load_golden(golden_path("attn_c2_mini"))
    scale = case["meta"]["scale"]
    q, k, v, m = (case[x].float().numpy() for x in ("q", "k", "v", "mask"))
    out, lse = oracle.attention_parallel(q, k, v, m, scale, threads=3, with_lse=True, chunk=1)
    assert np.array_equal(out, oracle.attention(q, k, v, m, scale))
    assert np.array_equal(lse, oracle.lse(q, k, m, scale))
    assert np.array_equal(oracle.pack_mask_parallel(m.astype(bool), threads=3, chunk=1), oracle.pack_mask(m))


def test_empty_rows_are_zero():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 1, 16, 64)).astype(np.float32) for _ in range(3))
    m = rng.random((1, 1, 16, 16)) < 0.5
    m[0, 0, 3] = False
    out = oracle.attention(q, k, v, m, 0.125)
    assert np.all(out[0, 0, 3] == 0)
    assert oracle.lse(q, k, m, 0.125)[0, 0, 3] == -FLT_MAX


def test_planted_error_is_caught():
    """A mistake planted in the oracle's inputs must break agreement with the
    reference fixture (guards against a vacuous comparison)."""
    case = load_golden(golden_path("attn_c1_mini"))
    m = case["mask"].numpy().copy()
    m[0, 0, 10, np.argmax(m[0, 0, 10])] = False  # drop one kept key
    out = oracle.attention(*(case[x].float().numpy() for x in ("q", "k", "v")), m, case["meta"]["scale"])
    assert np.abs(out - case["out"].numpy()).max() > 1e-3
    packed = oracle.pack_mask(m)
    assert not np.array_equal(packed, case["packed"].numpy())


@pytest.mark.parametrize("path", golden_paths("pack") + golden_paths("attn"), ids=golden_ids("pack") + golden_ids("attn"))
def test_occupancy_matches_reference_packed_bits(path):
    """The occupancy restatement agrees with the reference's packed words:
    a (query tile, key tile) block is live iff one of its packed words is
    non-zero."""
    case = load_golden(path)
    mask = case["mask"].numpy()
    n = mask.shape[-1]
    words = case["packed"].numpy().view(np.uint32)  # reference bits [B, H, N, W]
    occ = oracle.occupancy(mask).view(np.uint32)
    qt = (n + 127) // 128
    for t in range(min(qt, 64)):
        cols = words[..., 4 * t:4 * t + 4]
        for r in range(qt):
            live = (cols[:, :, 128 * r:128 * (r + 1)] != 0).any(axis=(2, 3))
            assert np.array_equal((occ[:, :, r, t // 32] >> (t % 32)) & 1, live.astype(np.uint32))


@pytest.mark.parametrize("path", golden_paths("bwd"), ids=golden_ids("bwd"))
def test_backward_vs_reference(path):
    """The oracle's backward against the reference's own CPU backward
    (python/sparse_attention.py:97-111) on the same inputs."""
    case = load_golden(path)
    scale = case["meta"]["scale"]
    q, k, v, dout, m = (case[x].float().numpy() for x in ("q", "k", "v", "dout", "mask"))
    dq, dk, dv = oracle.attention_backward(q, k, v, m, scale, dout)
    for got, name in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        want = case[name].numpy()
        np.testing.assert_allclose(got, want, atol=1e-4 * max(1.0, np.abs(want).max()), rtol=1e-4, err_msg=name)
    empty = ~case["mask"].numpy().any(axis=-1)
    assert np.all(dq[empty] == 0), "rows with no kept key get no gradient"


def test_backward_planted_error_is_caught():
    case = load_golden(golden_path("bwd_c1_mini"))
    m = case["mask"].numpy().copy()
    m[0, 1, 20, np.argmax(m[0, 1, 20])] = False  # drop one kept key
    q, k, v, dout = (case[x].float().numpy() for x in ("q", "k", "v", "dout"))
    dq, dk, dv = oracle.attention_backward(q, k, v, m, case["meta"]["scale"], dout)
    assert np.abs(dq - case["dq"].numpy()).max() > 1e-3
