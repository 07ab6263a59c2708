// bool [rows, N] -> uint32 [rows, ceil(N/32)] bit packing.
//
// Semantics follow the reference packer (python/sparse_attention.py:189-206,
// csrc/sparse_attention.cu:20-42): bit b of word w of a row is set iff the
// mask byte at column 32*w + b is true (non-zero); bits at columns >= N are 0.
//
// Layout in HBM: the input is B*H*N rows of N bytes, the output B*H*N rows of
// ceil(N/32) words, both row-major and contiguous.  The kernel is purely
// HBM-bound (N^2 bytes read and N^2/8 written per head), so the design goal
// is fully coalesced 16-byte loads and 4-byte stores with enough bytes in
// flight per SM, not arithmetic.
//
// Fast path (N % 32 == 0 and 16-byte aligned input): every output word is one
// aligned 32-byte chunk of the flat input, independent of row boundaries.  A
// warp packs 32 consecutive words per round (1 KiB of input), four rounds per
// thread with all eight 16-byte loads issued before any use.
// General path: one thread per output word with byte loads (any N, any
// alignment).
#include "mask_bits.cuh"
#include "sma_internal.h"
#include "sma_ptx.cuh"

namespace sma {
namespace {

constexpr int kPackThreads = 256;
constexpr int kPackRounds = 4;
constexpr int kOccTileRows = 128;  // query rows per occupancy item (the attention tile)

__global__ void __launch_bounds__(kPackThreads) pack_mask_aligned_kernel(
    const uint4* __restrict__ in, uint32_t* __restrict__ out, int64_t total_words) {
  pdl_launch_dependents();  // the attention kernel after this one may start its set-up
  const int lane = threadIdx.x & 31;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * kPackThreads + threadIdx.x) >> 5;
  const int64_t base = warp_global * (32 * kPackRounds);
  uint4 lo[kPackRounds], hi[kPackRounds];
#pragma unroll
  for (int r = 0; r < kPackRounds; ++r) {
    const int64_t w = base + r * 32 + lane;
    if (w < total_words) {
      lo[r] = __ldcs(in + 2 * w);
      hi[r] = __ldcs(in + 2 * w + 1);
    } else {
      lo[r] = make_uint4(0, 0, 0, 0);
      hi[r] = lo[r];
    }
  }
#pragma unroll
  for (int r = 0; r < kPackRounds; ++r) {
    const int64_t w = base + r * 32 + lane;
    if (w < total_words) out[w] = pack32_any(lo[r], hi[r]);
  }
}

__global__ void __launch_bounds__(kPackThreads) pack_mask_generic_kernel(
    const uint8_t* __restrict__ in, uint32_t* __restrict__ out, int64_t rows, int64_t n,
    int64_t n_words) {
  pdl_launch_dependents();  // the attention kernel after this one may start its set-up
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * kPackThreads + threadIdx.x;
  if (idx >= rows * n_words) return;
  const int64_t row = idx / n_words;
  const int64_t w = idx - row * n_words;
  const uint8_t* src = in + row * n + w * 32;
  const int64_t cols = (n - w * 32) < 32 ? (n - w * 32) : 32;
  uint32_t bits = 0;
  for (int b = 0; b < cols; ++b) bits |= static_cast<uint32_t>(src[b] != 0) << b;
  out[idx] = bits;
}

// Fused pack + occupancy map (aligned input only).  One CTA per (batch*head,
// 128-row query tile): it packs the tile's rows like the aligned kernel and
// ORs the packed words per 128-key tile, so that occ[item][0..1] bit t says
// whether key tile t (keys 128t .. 128t+127) has any set bit in the item's
// rows (t < 64, i.e. N <= 8192).  The attention kernel skips dead key tiles
// with this map instead of re-reading the packed rows.
constexpr int kOccRounds = 4;
constexpr int kOccThreads = 256;  // one item (128 rows x N/32 words) per CTA

__global__ void __launch_bounds__(kOccThreads) pack_mask_occ_kernel(
    const uint4* __restrict__ in, uint32_t* __restrict__ out, uint32_t* __restrict__ occ, int n, int n_words,
    int q_tiles) {
  pdl_launch_dependents();  // the attention kernel after this one may start its set-up
  __shared__ uint32_t s_bits[2];
  const int item = blockIdx.x;  // batch*head * q_tiles + query tile
  const int bh = item / q_tiles;
  const int qt = item - bh * q_tiles;
  const int rows = min(kOccTileRows, n - qt * kOccTileRows);
  const int64_t base = (static_cast<int64_t>(bh) * n + static_cast<int64_t>(qt) * kOccTileRows) * n_words;
  const int words = rows * n_words;
  if (threadIdx.x < 2) s_bits[threadIdx.x] = 0u;
  uint32_t lo = 0u, hi = 0u;
  for (int w0 = threadIdx.x; w0 < words; w0 += kOccThreads * kOccRounds) {
    uint4 a[kOccRounds], b[kOccRounds];
#pragma unroll
    for (int r = 0; r < kOccRounds; ++r) {
      const int w = w0 + r * kOccThreads;
      if (w < words) {
        a[r] = __ldcs(in + 2 * (base + w));
        b[r] = __ldcs(in + 2 * (base + w) + 1);
      } else {
        a[r] = make_uint4(0, 0, 0, 0);
        b[r] = a[r];
      }
    }
#pragma unroll
    for (int r = 0; r < kOccRounds; ++r) {
      const int w = w0 + r * kOccThreads;
      if (w < words) {
        const uint32_t word = pack32_any(a[r], b[r]);
        out[base + w] = word;
        if (word != 0u) {
          const int tile = (w % n_words) >> 2;  // four 32-column words per key tile
          if (tile < 32) lo |= 1u << tile;
          else hi |= 1u << (tile - 32);
        }
      }
    }
  }
  lo = __reduce_or_sync(0xffffffffu, lo);
  hi = __reduce_or_sync(0xffffffffu, hi);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    if (lo) atomicOr(&s_bits[0], lo);
    if (hi) atomicOr(&s_bits[1], hi);
  }
  __syncthreads();
  if (threadIdx.x < 2) occ[2 * static_cast<int64_t>(item) + threadIdx.x] = s_bits[threadIdx.x];
}

}  // namespace

int launch_pack_mask(const uint8_t* mask, uint32_t* packed, int64_t rows, int64_t n,
                     cudaStream_t stream, const char** msg) {
  if (rows < 0 || n < 0) {
    *msg = "pack_mask: negative size";
    return kErrArg;
  }
  if (rows == 0 || n == 0) return kOk;
  if (mask == nullptr || packed == nullptr) {
    *msg = "pack_mask: null pointer";
    return kErrArg;
  }
  const int64_t n_words = (n + 31) / 32;
  const bool aligned = (n % 32 == 0) && (reinterpret_cast<uintptr_t>(mask) % 16 == 0) &&
                       (reinterpret_cast<uintptr_t>(packed) % 4 == 0);
  if (aligned) {
    const int64_t total_words = rows * n_words;
    const int64_t words_per_block = (kPackThreads / 32) * 32 * kPackRounds;
    const int64_t blocks = (total_words + words_per_block - 1) / words_per_block;
    if (blocks > 0x7FFFFFFFll) {
      *msg = "pack_mask: input too large";
      return kErrArg;
    }
    pack_mask_aligned_kernel<<<static_cast<unsigned>(blocks), kPackThreads, 0, stream>>>(
        reinterpret_cast<const uint4*>(mask), packed, total_words);
  } else {
    const int64_t total = rows * n_words;
    const int64_t blocks = (total + kPackThreads - 1) / kPackThreads;
    if (blocks > 0x7FFFFFFFll) {
      *msg = "pack_mask: input too large";
      return kErrArg;
    }
    pack_mask_generic_kernel<<<static_cast<unsigned>(blocks), kPackThreads, 0, stream>>>(
        mask, packed, rows, n, n_words);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *msg = cudaGetErrorString(e);
    return kErrLaunch;
  }
  return kOk;
}

int launch_pack_mask_occ(const uint8_t* mask, uint32_t* packed, uint32_t* occ, int64_t bh, int64_t n,
                         cudaStream_t stream, const char** msg) {
  if (bh < 0 || n < 0) {
    *msg = "pack_mask_occupancy: negative size";
    return kErrArg;
  }
  if (bh == 0 || n == 0) return kOk;
  if (mask == nullptr || packed == nullptr || occ == nullptr) {
    *msg = "pack_mask_occupancy: null pointer";
    return kErrArg;
  }
  if (n % 32 != 0 || (reinterpret_cast<uintptr_t>(mask) % 16) != 0 || (reinterpret_cast<uintptr_t>(packed) % 4) != 0 ||
      (reinterpret_cast<uintptr_t>(occ) % 4) != 0) {
    *msg = "pack_mask_occupancy: needs N % 32 == 0, a 16-byte aligned mask and 4-byte aligned outputs";
    return kErrArg;
  }
  if (n > kMaxSeqLenOcc) {
    *msg = "pack_mask_occupancy: sequence length above the occupancy map's maximum (8192)";
    return kErrUnsupportedN;
  }
  const int64_t q_tiles = (n + kOccTileRows - 1) / kOccTileRows;
  const int64_t items = bh * q_tiles;
  if (items > 0x7FFFFFFFll) {
    *msg = "pack_mask_occupancy: input too large";
    return kErrArg;
  }
  pack_mask_occ_kernel<<<static_cast<unsigned>(items), kOccThreads, 0, stream>>>(
      reinterpret_cast<const uint4*>(mask), packed, occ, static_cast<int>(n), static_cast<int>(n / 32),
      static_cast<int>(q_tiles));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    *msg = cudaGetErrorString(e);
    return kErrLaunch;
  }
  return kOk;
}

}  // namespace sma
