// Fused masked-softmax attention backward, head dims 64 and 128 (sm_100a).
//
// The reference binds no CUDA backward (python/sparse_attention.py:93-96 calls
// sparse_attn_cuda.backward, which csrc/binding.cpp never defines); its CPU
// formulas (python/sparse_attention.py:97-111) define the result:
//   P   = softmax of the masked scaled scores, rebuilt here from the forward's
//         LSE: P_ij = bit(i,j) ? exp(scale * q_i.k_j - lse_i) : 0
//   dV  = P^T dO
//   dP  = dO V^T (0 where masked; P is 0 there, so dS is too)
//   dS  = P * (dP - Delta),  Delta_i = sum_d dO_id O_id  (= rowsum(P * dP))
//   dQ  = scale * dS K,   dK = scale * dS^T Q
//
// Kernels (one stream, in order):
//   bwd_delta_kernel   Delta from dO and O (FP32), D/8 threads per row; also
//                      zeroes the FP32 dQ accumulator
//   attn_bwd_kernel    persistent, one CTA per SM looping over the items
//                      (batch*head, 128-key tile).  Per item K and V stay in
//                      shared memory, dK and dV accumulate in TMEM, and the
//                      CTA walks only the 128-row query tiles whose mask block
//                      with its key tile has a set bit (listed ahead by a
//                      scanner warp).  Per live query tile:
//                        MMA  S^T = K Q^T, dP^T = V dO^T   (M = keys)
//                        P^T, dS^T in registers (thread t = key t), written
//                        back to TMEM (fp16/bf16) and dS to shared memory
//                        MMA  dV += P^T dO, dK += dS^T Q  (A from TMEM)
//                             dQ_part = dS K              (A from shared memory, M-major)
//                        dQ_part * scale is added into an FP32 accumulator in
//                        global memory (staged in shared memory, TMA bulk
//                        reduce-add)
//   bwd_dq_convert_kernel  FP32 accumulator -> dq in the input dtype
//
// Warps (E = 8 element-wise warps for D = 64, 4 for D = 128): 0..E-1 compute
// (P^T and dS^T; thread <-> TMEM lane 32(w%4) + lane, warp w takes 32-query
// chunks of the tile by w/4), E loader (TMA of K, V, Q, dO; mask words, LSE and
// Delta of the query tile staged in shared memory), E+1 MMA issuer and TMEM
// owner, E+2..E+5 epilogue (dQ_part of each live tile into the FP32
// accumulator, dK and dV of each item; warp w reads TMEM lanes 32(w%4)..+31),
// so the epilogues of one tile overlap the element-wise work of the next, E+6
// scanner (each item's live query tiles, kSlots items ahead).
// TMEM layout per head dim: see BwdCfg.
// Every wait is bounded and reports through the device error word.
#include <cfloat>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "sma_internal.h"
#include "sma_ptx.cuh"

namespace sma {
namespace {

constexpr int kT = 128;  // query rows and keys per tile
constexpr int kTmemCols = 512;
constexpr uint32_t kColS = 0, kColDP = 128, kColDV = 256;
constexpr float kLog2e = 1.44269504088896340736f;

// Per head dim.  Tiles of K, V, Q, dO are kT rows of D/64 128-byte swizzle
// chunks.  D = 64 double-buffers K/V (the next item's keys load while the
// current item computes) and the query tiles (the loader fills tile i+1 while
// tile i is computed); D = 128 has shared memory for one of each.
// TMEM: S^T [0,128) and dP^T [128,256) (P^T / dS^T packed over their first
// 64 columns; for D = 64 the packed P^T / dS^T of query columns 64-127 at
// [448,480) / [480,512) instead), dV [256, 256+D), dK [256+D, 256+2D);
// dQ_part in 64-column halves: D = 64 at [384,448), D = 128 over the S^T /
// dP^T columns that P^T / dS^T leave free, [64,128) and [192,256).
template <int D>
struct BwdCfg {
  static_assert(D == 64 || D == 128, "head dim");
  // Element-wise warps.  D = 64 runs two per TMEM lane quadrant, each taking
  // half of a tile's 128 query columns; the second half's packed P^T / dS^T
  // go to the free columns [448, 512), so neither warp writes columns the
  // other still reads.  D = 128 has no free columns and runs one per quadrant
  // (packing in place, chunk by chunk).
  static constexpr int kEwWarps = D == 64 ? 8 : 4;
  static constexpr int kChunksPerWarp = 16 / kEwWarps;  // 32-query chunks of a tile per element-wise warp
  static constexpr int kLoaderWarp = kEwWarps;
  static constexpr int kMmaWarp = kEwWarps + 1;
  static constexpr int kScanWarp = kEwWarps + 6;  // after the 4 epilogue warps
  static constexpr int kThreads = (kEwWarps + 7) * 32;
  // Packed P^T / dS^T of 32-query chunk c (16 columns each).
  __host__ __device__ static constexpr uint32_t col_p(int c) {
    return (D == 64 && c >= 2) ? 448u + (c - 2) * 16u : kColS + c * 16u;
  }
  __host__ __device__ static constexpr uint32_t col_ds(int c) {
    return (D == 64 && c >= 2) ? 480u + (c - 2) * 16u : kColDP + c * 16u;
  }
  static constexpr int kDChunks = D / 64;
  static constexpr int kTileBytes = kT * D * 2;  // 16 / 32 KiB
  static constexpr int kKVBufs = D == 64 ? 2 : 1;
  static constexpr int kQBufs = D == 64 ? 2 : 1;
  static constexpr uint32_t kColDK = kColDV + D;
  __host__ __device__ static constexpr uint32_t col_dq(int h) { return D == 64 ? 384u : (h == 0 ? 64u : 192u); }
  // With dQ_part in its own TMEM columns (D = 64), the next tile's S^T / dP^T
  // may be issued while the epilogue warps still read this tile's dQ_part, and
  // a tile's dQ_part product is issued after the next tile's S^T / dP^T, so
  // the element-wise warps do not wait behind it in the tensor pipe; dS is
  // then double-buffered in shared memory.
  static constexpr bool kDQApart = D == 64;
  static constexpr int kDSBufs = kDQApart ? 2 : 1;
  // dQ_part staging boxes (4 KiB: 32 rows of 32 FP32 columns) per epilogue warp.
  static constexpr int kStageBoxes = D == 64 ? 1 : 2;
  static constexpr int kOffK = 0;
  static constexpr int kOffV = kKVBufs * kTileBytes;
  static constexpr int kOffQ = 2 * kKVBufs * kTileBytes;
  static constexpr int kOffDO = kOffQ + kQBufs * kTileBytes;
  // dS buffers: two 16 KiB M-major chunks of 64 queries each.
  static constexpr int kOffDS = kOffDO + kQBufs * kTileBytes;
  static constexpr int kOffMask = kOffDS + kDSBufs * 2 * kT * 128;
  static constexpr int kOffLse = kOffMask + kQBufs * 4 * kT * 4;
  static constexpr int kOffDelta = kOffLse + kQBufs * kT * 4;
  // dQ_part staging for the bulk reduce: kStageBoxes 4 KiB boxes per epilogue
  // warp (its 32 rows by 32 FP32 columns, 128-byte swizzle), reused for the
  // D/32 column boxes of a tile in turn.
  static constexpr int kOffDQ = (kOffDelta + kQBufs * kT * 4 + 1023) / 1024 * 1024;
  static constexpr int kOffCtl = kOffDQ + 4 * kStageBoxes * 4096;
  // Above half of the SM's shared memory, so one CTA holds an SM (its TMEM
  // allocation takes all 512 columns).
  static constexpr size_t kSmemBytes = D == 64 ? 216 * 1024 : 200 * 1024;
};

// Items whose live query-tile lists the scanner warp publishes ahead, and
// words of a list (one bit per 128-row query tile; 16 words cover N <= 65536).
constexpr int kSlots = 4;
constexpr int kLiveWords = 16;

struct BwdCtl {
  uint64_t kv_full[2];    // K and V of a live item landed in buffer b
  uint64_t kv_free[2];    // products of the live item in K/V buffer b complete (committed by the MMA issuer)
  uint64_t acc_free;      // dV and dK of a live item read out of TMEM (4 epilogue warps)
  uint64_t ld_full[2];    // live query tile staged in buffer b (Q, dO by TMA; mask, LSE, Delta by the loader)
  uint64_t st_full;       // S^T and dP^T complete
  uint64_t p_full;        // P^T, dS^T in TMEM and dS in shared memory (compute warps)
  uint64_t pt_free;       // dV, dK products of a tile complete (they read P^T / dS^T in TMEM)
  uint64_t dq_full;       // all products of a tile complete (dQ_part in TMEM)
  uint64_t dq_free;       // dQ_part of a tile read out of TMEM (4 epilogue warps)
  uint64_t tile_free[2];  // compute warps and the MMA issuer done with buffer b
  uint64_t item_full[kSlots];  // live list of an item published (scanner warp)
  uint64_t item_free[kSlots];  // every other warp done with that list
  uint64_t drain;
  uint32_t live_bits[kSlots][kLiveWords];
  uint32_t n_live[kSlots];
  uint32_t tmem_base;
  uint32_t abort_flag;
};

// Shared memory: K[kKVBufs] | V[kKVBufs] | Q[kQBufs] | dO[kQBufs] | dS[kDSBufs]
// | mask words [kQBufs][4][128] | -lse2 [kQBufs][128] | -Delta [kQBufs][128] |
// dQ staging [4 warps][kStageBoxes][32][32] FP32 | control (with the live lists).
static_assert(BwdCfg<64>::kOffCtl + sizeof(BwdCtl) <= BwdCfg<64>::kSmemBytes, "shared memory layout");
static_assert(BwdCfg<128>::kOffCtl + sizeof(BwdCtl) <= BwdCfg<128>::kSmemBytes, "shared memory layout");

// Packed FP32 pairs (sm_100a f32x2 instructions): one issue slot for two lanes' worth of FMA / add / multiply.
__device__ __forceinline__ uint64_t f2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t x) {
  if constexpr (BF16) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&x));
  } else {
    return __half22float2(*reinterpret_cast<__half2*>(&x));
  }
}

// Bits of packed-mask word cw of a row that address columns < N.
__device__ __forceinline__ uint32_t valid_bits(int cw, int N) {
  const int valid = N - cw * 32;
  return valid >= 32 ? 0xFFFFFFFFu : (valid <= 0 ? 0u : ((1u << valid) - 1u));
}

// Next set bit of a live list from cursor (w, x): the query tile index, or -1.
__device__ __forceinline__ int next_live_tile(const uint32_t* bits, int& w, uint32_t& x) {
  while (x == 0u) {
    if (++w >= kLiveWords) return -1;
    x = bits[w];
  }
  const int b = __ffs(x) - 1;
  x &= x - 1u;
  return w * 32 + b;
}

// Delta[row] = sum_d dO[row, d] * O[row, d] in FP32; D/8 threads per row, one
// 16-byte load of each operand per thread.  Each thread also zeroes the 8 FP32
// dQ accumulator elements of its 8 (row, d), which the backward kernel then
// reduce-adds into (one pass instead of a separate memset).
template <int D, bool BF16>
__global__ void __launch_bounds__(256) bwd_delta_kernel(const uint4* __restrict__ dout, const uint4* __restrict__ out,
                                                         float* __restrict__ delta, float4* __restrict__ dq_acc,
                                                         int64_t rows) {
  constexpr int kPerRow = D / 8;
  const int64_t gid = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  const int64_t row = gid / kPerRow;
  float acc = 0.f;
  if (row < rows) {
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    dq_acc[2 * gid] = zero;
    dq_acc[2 * gid + 1] = zero;
    const uint4 a = __ldg(dout + gid), b = __ldg(out + gid);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 x = unpack2<BF16>(aw[e]), y = unpack2<BF16>(bw[e]);
      acc = fmaf(x.x, y.x, acc);
      acc = fmaf(x.y, y.y, acc);
    }
  }
#pragma unroll
  for (int o = 1; o < kPerRow; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (row < rows && (threadIdx.x % kPerRow) == 0) delta[row] = acc;
}

// dq[i] = acc[i] in the input dtype, 8 elements per thread.
template <bool BF16>
__global__ void __launch_bounds__(256) bwd_dq_convert_kernel(const float4* __restrict__ acc, uint4* __restrict__ dq,
                                                              int64_t n8) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= n8) return;
  const float4 a = acc[2 * i], b = acc[2 * i + 1];
  dq[i] = make_uint4(pack2<BF16>(a.x, a.y), pack2<BF16>(a.z, a.w), pack2<BF16>(b.x, b.y), pack2<BF16>(b.z, b.w));
}

template <int D, bool BF16>
__global__ void __launch_bounds__(BwdCfg<D>::kThreads, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq, const uint32_t* __restrict__ mask,
                    const float* __restrict__ lse, const float* __restrict__ delta, uint16_t* __restrict__ dk,
                    uint16_t* __restrict__ dv, int N, int W, int KT, int QT, int total_items, int vec, float scale,
                    uint32_t* err_word, uint64_t timeout_ns) {
  using C = BwdCfg<D>;
  constexpr int kQBufs = C::kQBufs;
  constexpr int kKVBufs = C::kKVBufs;
  constexpr int kTileBytes = C::kTileBytes;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t base = smem_u32(smem);
  if ((base & 1023u) != 0u) {
    if (threadIdx.x == 0) atomicOr(err_word, kDevErrLayout);
    return;
  }
  BwdCtl& ctl = *reinterpret_cast<BwdCtl*>(smem + C::kOffCtl);
  // Per buffer b: word w of query row i at s_mask[b * 4 * kT + w * kT + i];
  // -LSE * log2(e) and -Delta per query row at s_lse / s_delta [b * kT + i]
  // (negated, so that the element-wise pass adds them in packed pairs).
  uint32_t* s_mask = reinterpret_cast<uint32_t*>(smem + C::kOffMask);
  float* s_lse = reinterpret_cast<float*>(smem + C::kOffLse);
  float* s_delta = reinterpret_cast<float*>(smem + C::kOffDelta);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Persistent: CTA c takes items c, c + G, c + 2G, ... of item = batch*head *
  // KT + key tile, so the CTAs running at one time cover the key tiles of a
  // few heads side by side and share those heads' Q and dO in L2.  The scanner
  // warp publishes each item's live query tiles (a bit per 128-row tile whose
  // mask block with the key tile has a set bit) kSlots items ahead; the other
  // warps walk only those.  Counters over all items of the CTA: j (items; list
  // slot j % kSlots), li (items with a live tile; K/V buffer li % kKVBufs), lt
  // (live query tiles; staging buffer lt % kQBufs).
  const int G = static_cast<int>(gridDim.x);
  const int n_items = (total_items - static_cast<int>(blockIdx.x) + G - 1) / G;
  volatile uint32_t* abort_flag = &ctl.abort_flag;

  if (threadIdx.x == 128) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&ctl.kv_full[b]), 1);
      mbar_init(smem_u32(&ctl.kv_free[b]), 1);
      mbar_init(smem_u32(&ctl.ld_full[b]), 1);
      mbar_init(smem_u32(&ctl.tile_free[b]), C::kEwWarps + 1);  // compute warps + the MMA issuer
    }
    for (int sl = 0; sl < kSlots; ++sl) {
      mbar_init(smem_u32(&ctl.item_full[sl]), 1);
      mbar_init(smem_u32(&ctl.item_free[sl]), C::kEwWarps + 6);  // compute, loader, MMA, 4 epilogue warps
    }
    mbar_init(smem_u32(&ctl.acc_free), 4);
    mbar_init(smem_u32(&ctl.st_full), 1);
    mbar_init(smem_u32(&ctl.p_full), C::kEwWarps);
    mbar_init(smem_u32(&ctl.pt_free), 1);
    mbar_init(smem_u32(&ctl.dq_full), 1);
    mbar_init(smem_u32(&ctl.dq_free), 4);
    mbar_init(smem_u32(&ctl.drain), 1);
    ctl.abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == C::kMmaWarp) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;
  pdl_wait_prior_grid();

  auto fail = [&]() {
    ctl.abort_flag = 1;
    atomicOr(err_word, kDevErrTimeout);
  };
  // Whole-warp wait on the live list of item j.
  auto wait_item = [&](int j) -> bool {
    return __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.item_full[j % kSlots]), (j / kSlots) & 1,
                                                      abort_flag, timeout_ns));
  };

  if (warp == C::kLoaderWarp) {
    // ================================================================ loader
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      tma_prefetch_desc(&tm_dq);
    }
    bool ok = true;
    int lt = 0, li = 0;  // li: live items, whose K/V copies were started
    int last_copy = -1;  // last live tile (in lt) whose Q/dO copies were started
    // Mask words, LSE and Delta of query tile qt of (bh, kt), 4 rows per lane:
    // all loads issued at once, into registers.
    auto fetch = [&](int fbh, int fkt, int qt, uint32_t (&w4)[4][4], float (&l2)[4], float (&de)[4]) {
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
        const int row = qt * kT + lane + 32 * rr;
        const bool in = qt >= 0 && row < N;
        const int64_t r64 = static_cast<int64_t>(fbh) * N + (in ? row : 0);
        const uint32_t* mrow = mask + r64 * W + fkt * 4;
        if (vec) {
          uint4 x = make_uint4(0u, 0u, 0u, 0u);
          if (in) x = __ldg(reinterpret_cast<const uint4*>(mrow));
          w4[rr][0] = x.x;
          w4[rr][1] = x.y;
          w4[rr][2] = x.z;
          w4[rr][3] = x.w;
        } else {
#pragma unroll
          for (int w = 0; w < 4; ++w) w4[rr][w] = (in && fkt * 4 + w < W) ? __ldg(mrow + w) : 0u;
        }
        l2[rr] = in ? __ldg(lse + r64) : 0.f;
        de[rr] = in ? __ldg(delta + r64) : 0.f;
      }
    };
    // K and V of the next live item into buffer li % kKVBufs, once the
    // products of live item li - kKVBufs are complete.
    auto issue_kv = [&](int bh, int kt) -> bool {
      const int bkv = li % kKVBufs;
      if (li >= kKVBufs &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.kv_free[bkv]), ((li - kKVBufs) / kKVBufs) & 1,
                                                     abort_flag, timeout_ns)))
        return false;
      if (lane == 0) {
        mbar_arrive_expect_tx(smem_u32(&ctl.kv_full[bkv]), 2 * kTileBytes);
#pragma unroll
        for (int dc = 0; dc < C::kDChunks; ++dc) {
          tma_load_3d(base + C::kOffK + bkv * kTileBytes + dc * kT * 128, &tm_k, smem_u32(&ctl.kv_full[bkv]),
                      dc * 64, kt * kT, bh);
          tma_load_3d(base + C::kOffV + bkv * kTileBytes + dc * kT * 128, &tm_v, smem_u32(&ctl.kv_full[bkv]),
                      dc * 64, kt * kT, bh);
        }
      }
      ++li;
      return true;
    };
    // Live tile lt (query tile qt of (bh, kt)) into staging buffer lt % kQBufs,
    // once the compute warps are done with live tile lt - kQBufs and the
    // products reading its Q / dO are complete (the MMA issuer's arrival is a
    // tcgen05.commit).
    auto stage = [&](int bh, int kt, int qt, const uint32_t (&w4)[4][4], const float (&l2)[4],
                     const float (&de)[4]) -> bool {
      const int b = lt % kQBufs;
      if (lt >= kQBufs &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.tile_free[b]), ((lt - kQBufs) / kQBufs) & 1,
                                                     abort_flag, timeout_ns)))
        return false;
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
        const int i = lane + 32 * rr;
#pragma unroll
        for (int w = 0; w < 4; ++w) s_mask[b * 4 * kT + w * kT + i] = w4[rr][w] & valid_bits(kt * 4 + w, N);
        // -FLT_MAX (a row with no kept key) becomes +inf here; such a row has
        // no mask bit, so its P is 0 by the select and never uses this value.
        s_lse[b * kT + i] = -(l2[rr] * kLog2e);
        s_delta[b * kT + i] = -de[rr];
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(smem_u32(&ctl.ld_full[b]), 2 * kTileBytes);
#pragma unroll
        for (int dc = 0; dc < C::kDChunks; ++dc) {
          tma_load_3d(base + C::kOffQ + b * kTileBytes + dc * kT * 128, &tm_q, smem_u32(&ctl.ld_full[b]), dc * 64,
                      qt * kT, bh);
          tma_load_3d(base + C::kOffDO + b * kTileBytes + dc * kT * 128, &tm_do, smem_u32(&ctl.ld_full[b]),
                      dc * 64, qt * kT, bh);
        }
        last_copy = lt;
      }
      ++lt;
      return true;
    };
    // The loads of the next live tile are issued before this one waits for
    // its buffer, so their latency overlaps a tile; at an item's last live
    // tile that is the first live tile of the next item, when it has one.
    uint32_t nw[4][4];
    float nl[4], nd[4];
    bool have_next = false;  // nw / nl / nd hold the first live tile of item j
    for (int j = 0; ok && j < n_items; ++j) {
      if (!wait_item(j)) {
        ok = false;
        break;
      }
      const int sl = j % kSlots;
      const int n = static_cast<int>(ctl.n_live[sl]);
      if (n > 0) {
        const int item = static_cast<int>(blockIdx.x) + j * G;
        const int bh = item / KT;
        const int kt = item - bh * KT;
        if (!issue_kv(bh, kt)) {
          ok = false;
          break;
        }
        const uint32_t* bits = ctl.live_bits[sl];
        int cw = 0;
        uint32_t cx = bits[0];
        int qt_next = next_live_tile(bits, cw, cx);
        if (!have_next) fetch(bh, kt, qt_next, nw, nl, nd);
        have_next = false;
        for (int t = 0; t < n; ++t) {
          const int qt = qt_next;
          uint32_t w4[4][4];
          float l2[4], de[4];
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
            l2[rr] = nl[rr];
            de[rr] = nd[rr];
#pragma unroll
            for (int w = 0; w < 4; ++w) w4[rr][w] = nw[rr][w];
          }
          if (t + 1 < n) {
            qt_next = next_live_tile(bits, cw, cx);
            fetch(bh, kt, qt_next, nw, nl, nd);
          } else if (j + 1 < n_items) {
            // The next item's list (published kSlots items ahead of the
            // slowest reader, so never behind this warp's own release).
            if (!wait_item(j + 1)) {
              ok = false;
              break;
            }
            const int sl1 = (j + 1) % kSlots;
            if (ctl.n_live[sl1] > 0u) {
              int w1 = 0;
              uint32_t x1 = ctl.live_bits[sl1][0];
              const int item1 = item + G;
              fetch(item1 / KT, item1 - (item1 / KT) * KT, next_live_tile(ctl.live_bits[sl1], w1, x1), nw, nl, nd);
              have_next = true;
            }
          }
          if (!stage(bh, kt, qt, w4, l2, de)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.item_free[sl]));
    }
    if (!ok && lane == 0) {
      fail();
      // Let the copies this warp started land before the CTA exits.
      uint32_t zero = 0;
      for (int jj = li - kKVBufs; jj < li; ++jj)
        if (jj >= 0) mbar_wait_bounded(smem_u32(&ctl.kv_full[jj % kKVBufs]), (jj / kKVBufs) & 1, &zero, timeout_ns);
      for (int g = last_copy - kQBufs + 1; g <= last_copy; ++g)
        if (g >= 0) mbar_wait_bounded(smem_u32(&ctl.ld_full[g % kQBufs]), (g / kQBufs) & 1, &zero, timeout_ns);
    }
  } else if (warp == C::kMmaWarp) {
    // ================================================================ MMA issuer
    bool ok = true;
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_f16(kT, kT, BF16 ? 1 : 0, 0);       // S^T, dP^T (M = keys)
      constexpr uint32_t idesc_kv = make_idesc_f16(kT, D, BF16 ? 1 : 0, 1);       // dV, dK (B M/N-major)
      constexpr uint32_t idesc_q = make_idesc_f16(kT, 64, BF16 ? 1 : 0, 1, 1);    // dQ half (A and B M/N-major)
      uint32_t lt = 0;
      int li = 0;
      // dQ_part = dS K of live tile L (K of its item at sKL) in 64-dim halves:
      // 16 keys per step; dS's two 64-query chunks are kT * 128 bytes apart,
      // as are K's 64-dim chunks.  With dQ_part in its own columns, the
      // epilogue warps must have read tile L-1's first.
      auto issue_dq = [&](uint32_t L, uint32_t sKL) -> bool {
        if constexpr (C::kDQApart) {
          if (L > 0 && !mbar_wait_bounded(smem_u32(&ctl.dq_free), (L - 1) & 1, abort_flag, timeout_ns)) return false;
          tc_fence_after();
        }
        const uint32_t sDS = base + C::kOffDS + (L % C::kDSBufs) * (2 * kT * 128);
#pragma unroll
        for (int h = 0; h < C::kDChunks; ++h)
#pragma unroll
          for (int kk = 0; kk < kT / 16; ++kk)
            mma_ss(tmem + C::col_dq(h), smem_desc_sw128(sDS + kk * 2048, kT * 128, 1024),
                   smem_desc_sw128(sKL + h * (kT * 128) + kk * 2048, kT * 128, 1024), idesc_q, kk > 0 ? 1u : 0u);
        mma_commit(smem_u32(&ctl.dq_full));
        return true;
      };
      // D = 64: the live tile whose dQ_part is still to be issued, the K it
      // reads, and (once its item has ended) the K/V buffer to release after it.
      int pend = -1, pend_kv = -1;
      uint32_t pend_sk = 0;
      auto flush = [&]() -> bool {
        if (pend < 0) return true;
        if (!issue_dq(static_cast<uint32_t>(pend), pend_sk)) return false;
        if (pend_kv >= 0) mma_commit(smem_u32(&ctl.kv_free[pend_kv]));
        pend = -1;
        pend_kv = -1;
        return true;
      };
      for (int j = 0; ok && j < n_items; ++j) {
        const int sl = j % kSlots;
        if (!mbar_wait_bounded(smem_u32(&ctl.item_full[sl]), (j / kSlots) & 1, abort_flag, timeout_ns)) {
          ok = false;
          break;
        }
        const int n = static_cast<int>(ctl.n_live[sl]);
        if (n > 0) {
          const int bkv = li % kKVBufs;
          const uint32_t sK = base + C::kOffK + bkv * kTileBytes, sV = base + C::kOffV + bkv * kTileBytes;
          if (!mbar_wait_bounded(smem_u32(&ctl.kv_full[bkv]), (li / kKVBufs) & 1, abort_flag, timeout_ns)) {
            ok = false;
            break;
          }
          for (int t = 0; t < n; ++t, ++lt) {
            const int b = lt % kQBufs;
            const uint32_t sQ = base + C::kOffQ + b * kTileBytes, sDO = base + C::kOffDO + b * kTileBytes;
            // Tile lt staged.  The S^T / dP^T columns are free once the
            // previous live tile's dV / dK products (which read P^T / dS^T
            // there) are complete and, where dQ_part shares those columns
            // (D = 128), its dQ_part has been read.  MMAs into different
            // accumulators are not ordered by issue.
            if (!mbar_wait_bounded(smem_u32(&ctl.ld_full[b]), (lt / kQBufs) & 1, abort_flag, timeout_ns) ||
                (lt > 0 && !mbar_wait_bounded(smem_u32(C::kDQApart ? &ctl.pt_free : &ctl.dq_free), (lt - 1) & 1,
                                              abort_flag, timeout_ns))) {
              ok = false;
              break;
            }
            tc_fence_after();
            // 16 head dims per step: swizzle chunk kk/4 of the rows, 32 bytes into it.
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * (kT * 128) + (kk & 3) * 32;
              mma_ss(tmem + kColS, smem_desc_sw128(sK + off, 16, 1024), smem_desc_sw128(sQ + off, 16, 1024), idesc_s,
                     kk > 0 ? 1u : 0u);
            }
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * (kT * 128) + (kk & 3) * 32;
              mma_ss(tmem + kColDP, smem_desc_sw128(sV + off, 16, 1024), smem_desc_sw128(sDO + off, 16, 1024),
                     idesc_s, kk > 0 ? 1u : 0u);
            }
            // st_full also covers every earlier product, so the dQ_part that
            // last read this tile's dS buffer has done so before it is rewritten.
            mma_commit(smem_u32(&ctl.st_full));
            // D = 64: the previous live tile's dQ_part, behind this tile's S^T / dP^T.
            if (C::kDQApart && !flush()) {
              ok = false;
              break;
            }
            // P^T / dS^T of this tile; before the first dV / dK product of a
            // live item, the epilogue warps must have read the previous live
            // item's dV / dK.
            if (!mbar_wait_bounded(smem_u32(&ctl.p_full), lt & 1, abort_flag, timeout_ns) ||
                (t == 0 && li > 0 && !mbar_wait_bounded(smem_u32(&ctl.acc_free), (li - 1) & 1, abort_flag, timeout_ns))) {
              ok = false;
              break;
            }
            tc_fence_after();
            // 16 query rows per step: 8 packed TMEM columns of P^T / dS^T, 2048
            // bytes (16 rows of 128) into the M/N-major shared-memory operands,
            // whose 64-dim chunks (D = 128) are kT * 128 bytes apart.
#pragma unroll
            for (int kk = 0; kk < kT / 16; ++kk)
              mma_ts(tmem + kColDV, tmem + C::col_p(kk >> 1) + (kk & 1) * 8,
                     smem_desc_sw128(sDO + kk * 2048, kT * 128, 1024), idesc_kv, (t > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
            for (int kk = 0; kk < kT / 16; ++kk)
              mma_ts(tmem + C::kColDK, tmem + C::col_ds(kk >> 1) + (kk & 1) * 8,
                     smem_desc_sw128(sQ + kk * 2048, kT * 128, 1024), idesc_kv, (t > 0 || kk > 0) ? 1u : 0u);
            // Q / dO of the staging buffer are released when dV / dK complete
            // (the dQ product reads neither).
            if constexpr (C::kDQApart) {
              mma_commit(smem_u32(&ctl.pt_free));
              mma_commit(smem_u32(&ctl.tile_free[b]));
              pend = static_cast<int>(lt);
              pend_sk = sK;
            } else {
              mma_commit(smem_u32(&ctl.tile_free[b]));
              if (!issue_dq(lt, sK)) {
                ok = false;
                break;
              }
            }
          }
          if (!ok) break;
          ++li;
          // K/V buffer bkv may be refilled once this item's products are
          // complete.  D = 64: the last tile's dQ_part stays pending (issued
          // behind the next tile's S^T / dP^T, and bkv released after it) only
          // when the next item has a live tile; otherwise it is issued now, so
          // no warp waits on it across items the scanner has yet to publish.
          if constexpr (C::kDQApart) {
            bool keep = false;
            if (j + 1 < n_items) {
              if (!mbar_wait_bounded(smem_u32(&ctl.item_full[(j + 1) % kSlots]), ((j + 1) / kSlots) & 1, abort_flag,
                                     timeout_ns)) {
                ok = false;
                break;
              }
              keep = ctl.n_live[(j + 1) % kSlots] > 0u;
            }
            pend_kv = bkv;
            if (!keep && !flush()) {
              ok = false;
              break;
            }
          } else {
            mma_commit(smem_u32(&ctl.kv_free[bkv]));
          }
        }
        mbar_arrive(smem_u32(&ctl.item_free[sl]));
      }
      if (ok && !flush()) ok = false;
      if (!ok) fail();
      // Every MMA this thread issued must complete before TMEM is released.
      mma_commit(smem_u32(&ctl.drain));
      uint32_t zero = 0;
      mbar_wait_bounded(smem_u32(&ctl.drain), 0, &zero, timeout_ns);
    }
  } else if (warp == C::kScanWarp) {
    // ================================================================ scanner
    // Item j's live list: bit qt set when some query row of tile qt keeps a
    // key of the item's key tile.  4 query tiles per batch, 4 rows per lane.
    bool ok = true;
    for (int j = 0; j < n_items; ++j) {
      const int sl = j % kSlots;
      if (j >= kSlots &&
          !__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.item_free[sl]), ((j / kSlots) - 1) & 1,
                                                     abort_flag, timeout_ns))) {
        ok = false;
        break;
      }
      const int item = static_cast<int>(blockIdx.x) + j * G;
      const int bh = item / KT;
      const int kt = item - bh * KT;
      uint32_t vmask[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) vmask[w] = valid_bits(kt * 4 + w, N);
      uint32_t my_word = 0u;  // lane w: word w of the list
      for (int q0 = 0; q0 < QT; q0 += 4) {
        uint4 v[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int rr = 0; rr < 4; ++rr) {
            const int row = (q0 + u) * kT + lane + 32 * rr;
            uint4 x = make_uint4(0u, 0u, 0u, 0u);
            if (q0 + u < QT && row < N) {
              const uint32_t* mrow = mask + (static_cast<int64_t>(bh) * N + row) * W + kt * 4;
              if (vec) {
                x = __ldg(reinterpret_cast<const uint4*>(mrow));
              } else {
                x.x = __ldg(mrow);
                x.y = kt * 4 + 1 < W ? __ldg(mrow + 1) : 0u;
                x.z = kt * 4 + 2 < W ? __ldg(mrow + 2) : 0u;
                x.w = kt * 4 + 3 < W ? __ldg(mrow + 3) : 0u;
              }
            }
            v[u][rr] = x;
          }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t any = 0u;
#pragma unroll
          for (int rr = 0; rr < 4; ++rr)
            any |= (v[u][rr].x & vmask[0]) | (v[u][rr].y & vmask[1]) | (v[u][rr].z & vmask[2]) |
                   (v[u][rr].w & vmask[3]);
          const int qt = q0 + u;
          if (__any_sync(0xffffffffu, any != 0u) && lane == (qt >> 5)) my_word |= 1u << (qt & 31);
        }
      }
      if (lane < kLiveWords) ctl.live_bits[sl][lane] = my_word;
      const int n = __reduce_add_sync(0xffffffffu, __popc(my_word));
      if (lane == 0) ctl.n_live[sl] = static_cast<uint32_t>(n);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.item_full[sl]));
    }
    if (!ok && lane == 0) fail();
  } else {
    auto wait_all = [&](uint64_t& bar, uint32_t parity) -> bool {
      const bool all =
          __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&bar), parity, abort_flag, timeout_ns));
      tc_fence_after();
      return all;
    };
    auto arrive_warp = [&](uint64_t& bar) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar));
    };
    // Warp w reads TMEM lanes 32(w%4)..+31: thread t is key t of the tile
    // (P^T, dS^T, dK, dV) and query row t (dQ_part).
    const int t = (warp & 3) * 32 + lane;
    const uint32_t t_lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    bool ok = true;
    uint32_t lt = 0;
    if (warp < C::kEwWarps) {
      // ============================================================== compute
      const float c2 = scale * kLog2e;
      const int my_word = (t >> 5) * kT;  // the word holding this key, for each query row
      const uint32_t kbit = 1u << (t & 31);  // this key's bit in a query row's mask word
      const uint64_t c2x2 = f2(c2, c2);
      for (int j = 0; ok && j < n_items; ++j) {
        ok = wait_all(ctl.item_full[j % kSlots], (j / kSlots) & 1);
        if (!ok) break;
        const int n = static_cast<int>(ctl.n_live[j % kSlots]);
        arrive_warp(ctl.item_free[j % kSlots]);  // only the count is needed
        for (int tt = 0; tt < n; ++tt, ++lt) {
          const int b = lt % kQBufs;
          const uint32_t* my_words = s_mask + b * 4 * kT + my_word;
          const float* t_lse = s_lse + b * kT;
          const float* t_delta = s_delta + b * kT;
          ok = wait_all(ctl.ld_full[b], (lt / kQBufs) & 1) && wait_all(ctl.st_full, lt & 1);
          if (!ok) break;
#pragma unroll 1
          for (int c = (warp >> 2) * C::kChunksPerWarp; c < ((warp >> 2) + 1) * C::kChunksPerWarp; ++c) {
            float s[32], dp[32];
            tmem_ld32f(t_lane + kColS + c * 32, s);
            tmem_ld32f(t_lane + kColDP + c * 32, dp);
            tmem_wait_ld();
            uint32_t pw[16], dw[16];
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
              const uint4 m4 = *reinterpret_cast<const uint4*>(my_words + c * 32 + e);
              const float4 l4 = *reinterpret_cast<const float4*>(t_lse + c * 32 + e);
              const float4 d4 = *reinterpret_cast<const float4*>(t_delta + c * 32 + e);
              const uint32_t mm[4] = {m4.x, m4.y, m4.z, m4.w};
              // x = s * scale * log2(e) - lse2 and ds = p * (dp - Delta), two queries per instruction.
              float x[4], p[4], ds[4];
              f2_split(fma2(f2(s[e], s[e + 1]), c2x2, f2(l4.x, l4.y)), x[0], x[1]);
              f2_split(fma2(f2(s[e + 2], s[e + 3]), c2x2, f2(l4.z, l4.w)), x[2], x[3]);
#pragma unroll
              for (int u = 0; u < 4; ++u) p[u] = (mm[u] & kbit) ? ex2f(x[u]) : 0.f;
              f2_split(mul2(f2(p[0], p[1]), add2(f2(dp[e], dp[e + 1]), f2(d4.x, d4.y))), ds[0], ds[1]);
              f2_split(mul2(f2(p[2], p[3]), add2(f2(dp[e + 2], dp[e + 3]), f2(d4.z, d4.w))), ds[2], ds[3]);
              pw[e / 2] = pack2<BF16>(p[0], p[1]);
              pw[e / 2 + 1] = pack2<BF16>(p[2], p[3]);
              dw[e / 2] = pack2<BF16>(ds[0], ds[1]);
              dw[e / 2 + 1] = pack2<BF16>(ds[2], ds[3]);
            }
            // P^T and dS^T packed: in place over S^T / dP^T columns this warp
            // has already read (chunk c writes columns 16c.., whose values
            // belong to chunks <= c), or into the free columns (see col_p).
            tmem_st16(t_lane + C::col_p(c), pw);
            tmem_st16(t_lane + C::col_ds(c), dw);
            // dS for the dQ MMA: row t of the M-major operand, queries
            // 32c .. 32c+31 = 16-byte chunks 4(c&1) .. +3 of 64-query chunk c/2,
            // 128-byte swizzle (chunk index XOR row % 8).
            uint8_t* drow = smem + C::kOffDS + (lt % C::kDSBufs) * (2 * kT * 128) + (c >> 1) * (kT * 128) + t * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(drow + ((((c & 1) * 4 + q) ^ (t & 7)) * 16)) =
                  make_uint4(dw[4 * q], dw[4 * q + 1], dw[4 * q + 2], dw[4 * q + 3]);
          }
          tmem_wait_st();
          fence_proxy_async_smem();  // dS written by this thread, read by the tensor core
          arrive_warp(ctl.p_full);
          arrive_warp(ctl.tile_free[b]);
        }
      }
    } else {
      // ============================================================== epilogue
      uint8_t* s_dq = smem + C::kOffDQ + (warp & 3) * (C::kStageBoxes * 4096);
      uint32_t li = 0;
      for (int j = 0; ok && j < n_items; ++j) {
        const int sl = j % kSlots;
        ok = wait_all(ctl.item_full[sl], (j / kSlots) & 1);
        if (!ok) break;
        const int item = static_cast<int>(blockIdx.x) + j * G;
        const int bh = item / KT;
        const int key = (item - bh * KT) * kT + t;
        const int n = static_cast<int>(ctl.n_live[sl]);
        const uint32_t* bits = ctl.live_bits[sl];
        int cw = 0;
        uint32_t cx = bits[0];
        for (int tt = 0; tt < n; ++tt, ++lt) {
          const int qt = next_live_tile(bits, cw, cx);
          ok = wait_all(ctl.dq_full, lt & 1);
          if (!ok) break;
          // dQ_part row t = query row qt*128 + t: all of it into registers,
          // TMEM released, then scaled, staged (this warp's 32 rows) and added
          // into the FP32 accumulator by TMA bulk reduce-adds, kStageBoxes
          // boxes of 32 columns per pass.  A box starting at or past row N has
          // nothing to add; the rows of a box past N are clipped by the TMA unit.
          float u[D];
#pragma unroll
          for (int h = 0; h < D / 32; ++h) tmem_ld32f(t_lane + C::col_dq(h >> 1) + (h & 1) * 32, u + 32 * h);
          tmem_wait_ld();
          arrive_warp(ctl.dq_free);
          const int row0 = qt * kT + (warp & 3) * 32;
#pragma unroll
          for (int pass = 0; pass < D / (32 * C::kStageBoxes); ++pass) {
            // This warp's staging area is free once its previous reduce-adds have read it.
            if (lane == 0) bulk_wait_group_read0();
            __syncwarp();
#pragma unroll
            for (int h = 0; h < C::kStageBoxes; ++h) {
              uint8_t* srow = s_dq + h * 4096 + lane * 128;
#pragma unroll
              for (int c = 0; c < 8; ++c) {
                const float* x = u + 32 * (C::kStageBoxes * pass + h) + 4 * c;
                *reinterpret_cast<float4*>(srow + ((c ^ (lane & 7)) * 16)) =
                    make_float4(x[0] * scale, x[1] * scale, x[2] * scale, x[3] * scale);
              }
            }
            fence_proxy_async_smem();  // staged by every lane, read by the TMA unit
            __syncwarp();
            if (lane == 0 && qt >= 0 && row0 < N) {
#pragma unroll
              for (int h = 0; h < C::kStageBoxes; ++h)
                tma_reduce_add_3d(&tm_dq, smem_u32(s_dq + h * 4096), (C::kStageBoxes * pass + h) * 32, row0, bh);
              bulk_commit_group();
            }
          }
        }
        if (!ok) break;
        // dV and dK of this key tile (lane t = key); zero when no query tile
        // was live.  The dq_full wait of the item's last live tile covered all
        // of its products.
#pragma unroll 1
        for (int h = 0; h < D / 32; ++h) {
          uint32_t vw[16], kw[16];
          if (n > 0) {
            float u[32];
            tmem_ld32f(t_lane + kColDV + h * 32, u);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) vw[e] = pack2<BF16>(u[2 * e], u[2 * e + 1]);
            tmem_ld32f(t_lane + C::kColDK + h * 32, u);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) kw[e] = pack2<BF16>(u[2 * e] * scale, u[2 * e + 1] * scale);
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) vw[e] = kw[e] = 0u;
          }
          if (key < N) {
            uint4* dvr = reinterpret_cast<uint4*>(dv + (static_cast<int64_t>(bh) * N + key) * D + h * 32);
            uint4* dkr = reinterpret_cast<uint4*>(dk + (static_cast<int64_t>(bh) * N + key) * D + h * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              dvr[q] = make_uint4(vw[4 * q], vw[4 * q + 1], vw[4 * q + 2], vw[4 * q + 3]);
              dkr[q] = make_uint4(kw[4 * q], kw[4 * q + 1], kw[4 * q + 2], kw[4 * q + 3]);
            }
          }
        }
        if (n > 0) {
          arrive_warp(ctl.acc_free);  // live item li's dV / dK read out of TMEM
          ++li;
        }
        arrive_warp(ctl.item_free[sl]);
      }
      // The reduce-adds must finish (and stop reading shared memory) before the CTA exits.
      if (lane == 0) bulk_wait_group0();
    }
    if (!ok && lane == 0) fail();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, bool BF16>
int launch(const BwdParams& p, const char** msg) {
  using C = BwdCfg<D>;
  const int64_t BH = p.B * p.H;
  const int64_t N = p.N;
  const int64_t W = (N + 31) / 32;
  const int64_t KT = (N + kT - 1) / kT;
  const int64_t QT = (N + kT - 1) / kT;
  if (BH * KT > 0x7FFFFFFFll) {
    *msg = "backward: batch*heads too large";
    return kErrArg;
  }
  CUtensorMap mq, mk, mv, mdo, mdq;
  CUresult rc = make_tensor_map_3d(&mq, p.q, p.dtype, D, BH, N, kT);
  if (rc == CUDA_SUCCESS) rc = make_tensor_map_3d(&mk, p.k, p.dtype, D, BH, N, kT);
  if (rc == CUDA_SUCCESS) rc = make_tensor_map_3d(&mv, p.v, p.dtype, D, BH, N, kT);
  if (rc == CUDA_SUCCESS) rc = make_tensor_map_3d(&mdo, p.dout, p.dtype, D, BH, N, kT);
  if (rc == CUDA_SUCCESS) rc = make_tensor_map_3d_f32(&mdq, p.dq_accum, D, BH, N, 32);
  if (rc != CUDA_SUCCESS) {
    *msg = tensor_map_error("backward", rc);
    return kErrCuda;
  }
  DeviceProps dp;
  if (!device_props(&dp, msg)) return kErrCuda;
  static std::atomic<bool> smem_set[kMaxDevices] = {};
  auto kern = attn_bwd_kernel<D, BF16>;
  {
    cudaError_t e = ensure_smem_limit(kern, C::kSmemBytes, dp.device, smem_set);
    if (e != cudaSuccess) {
      *msg = cudaGetErrorString(e);
      return kErrLaunch;
    }
  }
  const int64_t rows = BH * N;
  bwd_delta_kernel<D, BF16><<<static_cast<unsigned>((rows * (D / 8) + 255) / 256), 256, 0, p.stream>>>(
      static_cast<const uint4*>(p.dout), static_cast<const uint4*>(p.out), p.delta,
      reinterpret_cast<float4*>(p.dq_accum), rows);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    const int vec = (W % 4 == 0 && (reinterpret_cast<uintptr_t>(p.mask) & 15u) == 0) ? 1 : 0;
    // One CTA per SM (over half of its shared memory and all 512 TMEM columns each).
    const int64_t items = BH * KT;
    const int64_t grid = items < dp.sms ? items : dp.sms;
    kern<<<static_cast<unsigned>(grid), C::kThreads, C::kSmemBytes, p.stream>>>(
        mq, mk, mv, mdo, mdq, p.mask, p.lse, p.delta, static_cast<uint16_t*>(p.dk),
        static_cast<uint16_t*>(p.dv), static_cast<int>(N), static_cast<int>(W), static_cast<int>(KT),
        static_cast<int>(QT), static_cast<int>(items), vec, p.scale, p.err_word, p.timeout_ns);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) {
    const int64_t n8 = rows * D / 8;
    bwd_dq_convert_kernel<BF16><<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, p.stream>>>(
        reinterpret_cast<const float4*>(p.dq_accum), static_cast<uint4*>(p.dq), n8);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    *msg = cudaGetErrorString(e);
    return kErrLaunch;
  }
  return kOk;
}

}  // namespace

int launch_attn_bwd(const BwdParams& p, const char** msg) {
  if (p.D != 64 && p.D != 128) {
    *msg = "backward: head dim must be 64 or 128";
    return kErrUnsupportedD;
  }
  if (p.N > kMaxSeqLen) {
    *msg = "backward: sequence length above the supported maximum (65536)";
    return kErrUnsupportedN;
  }
  if (p.D == 128) return p.dtype == 1 ? launch<128, true>(p, msg) : launch<128, false>(p, msg);
  return p.dtype == 1 ? launch<64, true>(p, msg) : launch<64, false>(p, msg);
}

}  // namespace sma
