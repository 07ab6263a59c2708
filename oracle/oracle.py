"""ORACLE — test infrastructure, not part of the product.

CPU restatement, in numpy, of the reference's algorithm for the hot path of
yulangz/sparse-mask-attention-auto-research.  Only tests/, the smoke check
in __graft_entry__.py and bench.py's CPU-baseline leg may import this module,
and only as the checker / the timed CPU baseline; the library never calls it.

Pinned against the reference: tests/golden/*.npz were produced by running the
reference's own Python code (python/sparse_attention.py, CPU path) with
tests/golden/make_golden.py, and tests/test_oracle.py checks every function
here against them (pack_mask bit-exact, attention and LSE to FP32 rounding).

Functions
  pack_mask(mask)                 python/sparse_attention.py:189-206
  occupancy(mask)                 live (query tile, key tile) blocks of the mask,
                                  the map the fused packer writes
                                  (same bits as csrc/sparse_attention.cu:20-42)
  attention(q, k, v, mask, scale) python/sparse_attention.py:26-44
  lse(q, k, mask, scale)          python/sparse_attention.py:74-76, with the
                                  CUDA path's -FLT_MAX for rows with no set bit
                                  (csrc/sparse_attention.cu:139-142)
  attention_parallel(...)         the same, split over heads on a thread pool
  attention_backward(q, k, v, mask, scale, dout)
                                  python/sparse_attention.py:97-111 (the
                                  reference's CPU backward formulas)
"""

import concurrent.futures
import os

import numpy as np

FLT_MAX = np.float32(3.4028234663852886e38)


def pack_mask(mask):
    """bool [..., N, N] -> int32 [..., N, ceil(N/32)].

    Bit b of word w of a row is mask[..., 32*w + b] (python/sparse_attention.py:199-205:
    ``packed[..., w] |= mask[..., col].int() << bit``); columns past N give 0
    bits; bit 31 lands in the sign bit of the int32, as in the reference.
    """
    mask = np.asarray(mask).astype(bool)
    n = mask.shape[-1]
    n_words = (n + 31) // 32
    pad = n_words * 32 - n
    if pad:
        mask = np.concatenate([mask, np.zeros(mask.shape[:-1] + (pad,), dtype=bool)], axis=-1)
    lead = mask.shape[:-1]
    by = np.packbits(mask.reshape(lead + (n_words, 32)), axis=-1, bitorder="little")  # [..., W, 4] uint8
    words = by.astype(np.uint32)
    packed = words[..., 0] | (words[..., 1] << 8) | (words[..., 2] << 16) | (words[..., 3] << 24)
    return packed.astype(np.uint32).view(np.int32)


def occupancy(mask, tile=128):
    """bool [B, H, N, N] -> int32 [B, H, ceil(N/tile), 2]: bit t of the pair
    for query tile qt is set iff mask[..., tile*qt : tile*(qt+1), tile*t :
    tile*(t+1)] has a True (t < 64).  The reference has no such map; this
    restates what the fused packer must produce from the same mask, i.e.
    which (query tile, key tile) blocks the reference's kernel would find
    any kept key in (csrc/sparse_attention.cu:110-111 tests every bit)."""
    mask = np.asarray(mask).astype(bool)
    B, H, n, _ = mask.shape
    qt = (n + tile - 1) // tile
    pad = qt * tile - n
    if pad:
        mask = np.pad(mask, ((0, 0), (0, 0), (0, pad), (0, pad)))
    blocks = mask.reshape(B, H, qt, tile, qt, tile).any(axis=(3, 5))  # [B, H, qt, kt]
    out = np.zeros((B, H, qt, 2), dtype=np.uint32)
    for t in range(min(qt, 64)):
        out[..., t // 32] |= blocks[..., t].astype(np.uint32) << np.uint32(t % 32)
    return out.view(np.int32)


def unpack_mask(packed, n):
    """Inverse of pack_mask: int32 [..., N, W] -> bool [..., N, n]."""
    p = np.ascontiguousarray(np.asarray(packed).view(np.uint32))
    by = p.view(np.uint8).reshape(p.shape + (4,))  # little-endian bytes of each word
    bits = np.unpackbits(by, axis=-1, bitorder="little").reshape(p.shape[:-1] + (p.shape[-1] * 32,))
    return bits[..., :n].astype(bool)


def _scores(q, k, scale):
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    return np.matmul(q, np.swapaxes(k, -1, -2)) * np.float32(scale)


def attention(q, k, v, mask, scale):
    """FP32 masked-softmax attention (python/sparse_attention.py:26-44):
    scores = q k^T * scale; masked entries -> -inf; softmax over keys;
    rows with no kept key -> 0 (the reference's nan_to_num); out = P v."""
    s = _scores(q, k, scale)
    mask = np.asarray(mask).astype(bool)
    s = np.where(mask, s, np.float32(-np.inf))
    m = s.max(axis=-1, keepdims=True)
    empty = ~np.isfinite(m)
    m = np.where(empty, np.float32(0), m)
    e = np.exp(s - m)
    denom = e.sum(axis=-1, keepdims=True)
    p = np.where(empty, np.float32(0), e / np.where(empty, np.float32(1), denom))
    return np.matmul(p.astype(np.float32), np.asarray(v, dtype=np.float32))


def lse(q, k, mask, scale):
    """Natural log-sum-exp of the scaled, masked scores per row
    (python/sparse_attention.py:74-76); rows with no kept key get -FLT_MAX,
    the value the reference CUDA kernel writes (csrc/sparse_attention.cu:141)."""
    s = _scores(q, k, scale)
    mask = np.asarray(mask).astype(bool)
    s = np.where(mask, s, np.float32(-np.inf))
    m = s.max(axis=-1)
    empty = ~np.isfinite(m)
    m0 = np.where(empty, np.float32(0), m)
    out = m0 + np.log(np.exp(s - m0[..., None]).sum(axis=-1))
    return np.where(empty, -FLT_MAX, out).astype(np.float32)


def attention_backward(q, k, v, mask, scale, dout):
    """FP32 gradients (dq, dk, dv) of attention() for the upstream gradient
    `dout`, with the reference's CPU backward formulas
    (python/sparse_attention.py:97-111): P = softmax of the masked scaled
    scores (0 on rows with no kept key); dv = P^T dout; dP = dout v^T, 0 where
    masked; dS = P * (dP - rowsum(dP * P)) * scale; dq = dS k; dk = dS^T q."""
    q = np.asarray(q, dtype=np.float32)
    k = np.asarray(k, dtype=np.float32)
    v = np.asarray(v, dtype=np.float32)
    dout = np.asarray(dout, dtype=np.float32)
    mask = np.asarray(mask).astype(bool)
    s = np.where(mask, _scores(q, k, scale), np.float32(-np.inf))
    m = s.max(axis=-1, keepdims=True)
    empty = ~np.isfinite(m)
    m = np.where(empty, np.float32(0), m)
    e = np.exp(s - m)
    denom = e.sum(axis=-1, keepdims=True)
    p = np.where(empty, np.float32(0), e / np.where(empty, np.float32(1), denom)).astype(np.float32)
    dv = np.matmul(np.swapaxes(p, -1, -2), dout)
    dp = np.where(mask, np.matmul(dout, np.swapaxes(v, -1, -2)), np.float32(0))
    ds = p * (dp - (dp * p).sum(axis=-1, keepdims=True)) * np.float32(scale)
    dq = np.matmul(ds, k)
    dk = np.matmul(np.swapaxes(ds, -1, -2), q)
    return dq.astype(np.float32), dk.astype(np.float32), dv.astype(np.float32)


def _flat(x):
    x = np.asarray(x)
    return x.reshape((-1,) + x.shape[-2:])


def attention_parallel(q, k, v, mask, scale, threads=None, with_lse=False, chunk=4):
    """attention() (and lse()) over heads on a thread pool; numpy releases
    the GIL in matmul and the element-wise kernels, so this uses all cores.
    BLAS itself is kept single-threaded by the caller when timing."""
    shape = np.asarray(q).shape
    qf, kf, vf, mf = _flat(q), _flat(k), _flat(v), _flat(mask)
    nh = qf.shape[0]
    out = np.empty(qf.shape, dtype=np.float32)
    lse_out = np.empty(qf.shape[:2], dtype=np.float32) if with_lse else None
    threads = threads or os.cpu_count() or 1

    def work(i0):
        i1 = min(nh, i0 + chunk)
        out[i0:i1] = attention(qf[i0:i1], kf[i0:i1], vf[i0:i1], mf[i0:i1], scale)
        if with_lse:
            lse_out[i0:i1] = lse(qf[i0:i1], kf[i0:i1], mf[i0:i1], scale)

    with concurrent.futures.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(work, range(0, nh, chunk)))
    out = out.reshape(shape)
    if with_lse:
        return out, lse_out.reshape(shape[:-1])
    return out


def pack_mask_parallel(mask, threads=None, chunk=4):
    """pack_mask() over heads on a thread pool."""
    shape = np.asarray(mask).shape
    mf = _flat(mask)
    nh = mf.shape[0]
    n = shape[-1]
    out = np.empty((nh, n, (n + 31) // 32), dtype=np.int32)
    threads = threads or os.cpu_count() or 1

    def work(i0):
        i1 = min(nh, i0 + chunk)
        out[i0:i1] = pack_mask(mf[i0:i1])

    with concurrent.futures.ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(work, range(0, nh, chunk)))
    return out.reshape(shape[:-1] + ((n + 31) // 32,))
