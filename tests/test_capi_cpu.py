"""The C-ABI library loads without a GPU, exports every symbol its header
declares, and rejects bad arguments before touching the device.  CPU only:
no call here launches work."""

import ctypes
import os
import re

import pytest

from conftest import REPO

import python._lib as L  # noqa: E402

HEADER = os.path.join(REPO, "include", "sma_capi.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sma_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(L.LIB_PATH):
        pytest.fail("libsma.so is not built (run __graft_entry__.build())")
    return L.load()


def test_header_declares_the_boundary():
    fns = header_functions()
    for name in ("sma_pack_mask", "sma_attn_fwd", "sma_last_error", "sma_device_status"):
        assert name in fns


def test_every_declared_symbol_is_exported(lib):
    for name in header_functions():
        assert hasattr(lib, name), name
    assert set(header_functions()) == set(L.SIGNATURES), "ctypes signature table out of sync with the header"


def test_abi_version(lib):
    assert lib.sma_abi_version() == 1


def _attn(lib, dtype=0, q=16, k=16, v=16, m=16, o=16, lse=None, B=1, H=1, N=64, D=64, scale=0.125):
    return lib.sma_attn_fwd(dtype, q, k, v, m, o, lse, B, H, N, D, scale, None)


def test_attn_rejects_bad_dtype(lib):
    assert _attn(lib, dtype=7) == L.SMA_ERR_DTYPE
    assert b"dtype" in lib.sma_last_error()


def test_attn_rejects_head_dim(lib):
    for d in (32, 96, 256):
        assert _attn(lib, D=d) == L.SMA_ERR_UNSUPPORTED_D


def test_attn_rejects_long_sequence(lib):
    assert _attn(lib, N=L.SMA_MAX_SEQ_LEN + 1) == L.SMA_ERR_UNSUPPORTED_N
    assert _attn(lib, N=L.SMA_MAX_SEQ_LEN + 1, D=128) == L.SMA_ERR_UNSUPPORTED_N
    assert b"65536" in lib.sma_last_error()
    # The map holds 64 key tiles per query tile: longer sequences are refused with it.
    args = (0, 16, 16, 16, 16, 16, 16, None, 1, 1, L.SMA_MAX_SEQ_LEN_OCCUPANCY + 1, 64, 0.125, None)
    assert lib.sma_attn_fwd_occupancy(*args) == L.SMA_ERR_UNSUPPORTED_N


def test_attn_rejects_bad_args(lib):
    assert _attn(lib, B=-1) == L.SMA_ERR_ARG
    assert _attn(lib, q=None) == L.SMA_ERR_ARG
    assert _attn(lib, q=8) == L.SMA_ERR_ARG  # not 16-byte aligned
    assert b"aligned" in lib.sma_last_error()


def test_attn_rejects_bad_scale(lib):
    for bad in (0.0, -0.125, float("inf"), float("nan")):
        assert _attn(lib, scale=bad) == L.SMA_ERR_ARG
        assert b"scale" in lib.sma_last_error()


def test_fused_pack_rejects_unsupported(lib):
    assert lib.sma_pack_mask_occupancy(16, 16, 16, 1, 1, 100, None) == L.SMA_ERR_ARG  # N % 32 != 0
    assert lib.sma_pack_mask_occupancy(16, 16, 16, 1, 1, L.SMA_MAX_SEQ_LEN_OCCUPANCY + 32, None) == L.SMA_ERR_UNSUPPORTED_N
    assert lib.sma_pack_mask_occupancy(None, 16, 16, 1, 1, 64, None) == L.SMA_ERR_ARG
    assert lib.sma_pack_mask_occupancy(8, 16, 16, 1, 1, 64, None) == L.SMA_ERR_ARG  # mask not 16-byte aligned
    assert lib.sma_pack_mask_occupancy(None, None, None, 0, 4, 64, None) == L.SMA_OK


def test_attn_with_map_rejects_bad_map(lib):
    args = (0, 16, 16, 16, 16)
    assert lib.sma_attn_fwd_occupancy(*args, None, 16, None, 1, 1, 64, 64, 0.125, None) == L.SMA_ERR_ARG
    assert lib.sma_attn_fwd_occupancy(*args, 18, 16, None, 1, 1, 64, 64, 0.125, None) == L.SMA_ERR_ARG


def test_empty_problems_are_noops(lib):
    assert _attn(lib, B=0) == L.SMA_OK
    assert lib.sma_pack_mask(None, None, 0, 4, 64, None) == L.SMA_OK


def test_pack_rejects_bad_args(lib):
    assert lib.sma_pack_mask(None, None, 1, 1, 64, None) == L.SMA_ERR_ARG
    assert lib.sma_pack_mask(16, 16, -1, 1, 64, None) == L.SMA_ERR_ARG


def test_timeout_setter(lib):
    assert lib.sma_set_wait_timeout_ns(0) == L.SMA_ERR_ARG
    assert lib.sma_set_wait_timeout_ns(2_000_000_000) == L.SMA_OK


def test_check_raises_with_message(lib):
    _attn(lib, dtype=9)
    with pytest.raises(L.SmaError, match="dtype"):
        L.check(L.SMA_ERR_DTYPE)


def _bwd(lib, dtype=0, ptr=16, lse=16, mask=16, acc=16, delta=16, B=1, H=1, N=64, D=64, scale=0.125):
    p = ptr
    return lib.sma_attn_bwd(dtype, p, p, p, p, p, lse, mask, p, p, p, acc, delta, B, H, N, D, scale, None)


def test_bwd_rejects_bad_arguments(lib):
    """The backward's argument checks run before any CUDA call."""
    assert _bwd(lib, dtype=7) == L.SMA_ERR_DTYPE
    for d in (32, 96, 256):
        assert _bwd(lib, D=d) == L.SMA_ERR_UNSUPPORTED_D
    assert _bwd(lib, N=L.SMA_MAX_SEQ_LEN + 1) == L.SMA_ERR_UNSUPPORTED_N
    assert b"65536" in lib.sma_last_error()
    for bad in (0.0, -1.0, float("inf"), float("nan")):
        assert _bwd(lib, scale=bad) == L.SMA_ERR_ARG
    assert _bwd(lib, B=-1) == L.SMA_ERR_ARG
    assert _bwd(lib, ptr=None) == L.SMA_ERR_ARG
    assert b"null" in lib.sma_last_error()
    assert _bwd(lib, ptr=8) == L.SMA_ERR_ARG  # q/k/v/out/dout/dq/dk/dv must be 16-byte aligned
    assert _bwd(lib, acc=8) == L.SMA_ERR_ARG  # so must the FP32 dQ accumulator
    assert b"16-byte" in lib.sma_last_error()
    assert _bwd(lib, lse=2) == L.SMA_ERR_ARG  # lse / delta / mask words: 4-byte aligned
    assert _bwd(lib, delta=6) == L.SMA_ERR_ARG
    assert b"4-byte" in lib.sma_last_error()


def test_bwd_empty_problem_is_a_noop(lib):
    for dims in (dict(B=0), dict(H=0), dict(N=0)):
        assert _bwd(lib, ptr=None, lse=None, mask=None, acc=None, delta=None, **dims) == L.SMA_OK


def test_bwd_noalloc_rejects_problems_beyond_its_scratch(lib):
    """B*H*N*(D+1) FP32 values must fit the fixed 32 MiB scratch; the check
    comes before any CUDA call, and an empty problem is a no-op."""
    def call(B, H, N, D):
        return lib.sma_attn_bwd_noalloc(0, 16, 16, 16, 16, 16, 16, 16, 16, 16, 16, B, H, N, D, 0.125, None)

    assert call(1, 256, 512, 64) == L.SMA_ERR_ARG  # 256*512*65 floats > 8 Mi
    assert b"scratch" in lib.sma_last_error()
    # The argument checks of sma_attn_bwd come first, with its codes.
    assert call(1, 1, L.SMA_MAX_SEQ_LEN + 1, 64) == L.SMA_ERR_UNSUPPORTED_N
    assert call(1, 1, 64, 96) == L.SMA_ERR_UNSUPPORTED_D
    assert lib.sma_attn_bwd_noalloc(7, 16, 16, 16, 16, 16, 16, 16, 16, 16, 16, 64, 64, 1024, 64, 0.125,
                                    None) == L.SMA_ERR_DTYPE
    assert call(-1, 1, 64, 64) == L.SMA_ERR_ARG
    assert call(0, 1, 64, 64) == L.SMA_OK
    # Largest accepted size: B*H*N*(D+1) just under 8 Mi floats; one more head is rejected.
    heads = (8 << 20) // (512 * 65)
    assert call(1, heads + 1, 512, 64) == L.SMA_ERR_ARG
