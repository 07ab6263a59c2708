// Persistent fused masked-softmax attention forward, head dim 64 (sm_100a).
//
// Same computation as attn_fwd.cu (reference csrc/sparse_attention.cu:64-143):
// O = softmax_masked(scale * Q K^T) V per (batch*head, query row), O = 0 and
// lse = -FLT_MAX for rows with no set mask bit.
//
// One CTA per SM loops over work items (batch*head, 128-row query tile),
// heaviest query tiles first.  Keys are processed in 128-wide tiles so that
// QK^T issues N=128 MMAs (an M=128,K=16 tcgen05.mma costs the same ~64
// cycles for N=64 as for N=128); tiles with no set mask bit in the item's
// rows are skipped before their K/V are loaded.
//
// The 128 keys of a tile are split between two softmax warpgroups: WG0 owns
// keys 0-63, WG1 keys 64-127.  Each keeps its own running max / sum and its
// own O accumulator in TMEM (O0, O1), so the two never synchronise inside
// the key loop; the epilogue merges the halves:
//   O = (O0 2^(m0-m) + O1 2^(m1-m)) / (l0 2^(m0-m) + l1 2^(m1-m)),  m = max(m0, m1).
//
// Warps (384 threads, one CTA per SM):
//   0-3  softmax WG0    4-7 softmax WG1   (thread t of a WG owns query row t)
//   8    loader: TMA-loads Q (two buffers) and the K and V of every live tile
//        through two stage rings shared by all items
//   9    TMEM allocator + QK^T issuer (one thread)
//   10   PV issuer (one thread): two issuing threads keep the tensor pipe
//        fed (a tcgen05.mma occupies its issuing thread ~60-100 cycles)
//   11   scheduler: per item, bulk-copies the packed-mask row block (two
//        slots), scans it for live key tiles and publishes the list; it runs
//        up to two items ahead so item start-up latency is hidden
//
// TMEM (512 columns): S buffers 2 x 128 | P buffers 2 x (32 + 32) | O0 64 | O1 64
//
// Pipelining: S and P are double-buffered, so QK^T of tile g+2 and PV of
// tile g overlap the softmax of tile g+1; inside a softmax warp the
// exponentials of tile g are interleaved with the masked max of tile g+1.
// Every wait is bounded (mbar_wait_bounded) and reports through err_word.
#include <cfloat>
#include <cstdio>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "sma_internal.h"
#include "sma_ptx.cuh"

namespace sma {
namespace {

constexpr int kD = 64;
constexpr int kBM = 128;
constexpr int kBN = 128;
constexpr int kHalf = kBN / 2;  // keys per softmax warpgroup
constexpr int kThreads = 384;  // 3 warpgroups: 2 softmax + {producer, MMA, 2 idle}
// Register split (setmaxnreg): the CTA launches at 168 registers per thread
// (384 x 168 = 64512); the softmax warpgroups then take 224 each and the
// producer/MMA warpgroup keeps 56: 2 x 128 x 224 + 128 x 56 = 64512.
constexpr int kRegsLaunch = 168;
constexpr int kRegsSoftmax = 192;
constexpr int kRegsControl = 120;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsControl == kThreads * kRegsLaunch, "register split");
constexpr int kMaxStages = 4;
constexpr int kMaxTiles = 16;  // N <= 2048
constexpr int kTmemCols = 512;
constexpr int kSCol = 0;        // 2 x 128
constexpr int kPCol = 256;      // 2 x 64 (WG0 half, WG1 half)
constexpr int kOCol = 384;      // O0 [384,448), O1 [448,512)
constexpr int kQBytes = kBM * kD * 2;      // 16 KiB
constexpr int kKBytes = kBN * kD * 2;      // 16 KiB
constexpr int kStageBytes = 2 * kKBytes;   // K + V
constexpr int kStagingBytes = kBM * kD * 2;
constexpr float kRescaleThreshold = 8.0f;
constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kLog2e = 1.44269504088896340736f;
constexpr int kMaxDevices = 64;
constexpr size_t kMinSmem = 120 * 1024;

struct Ctl {
  uint64_t sched_full[2];
  uint64_t mask_empty[2];
  uint64_t mask_full[2];
  uint64_t q_full[2];
  uint64_t q_empty[2];
  uint64_t k_full[kMaxStages];
  uint64_t k_empty[kMaxStages];
  uint64_t v_full[kMaxStages];
  uint64_t v_empty[kMaxStages];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t o_free;
  uint64_t drain[2];
  uint32_t tmem_base;
  uint32_t abort_flag;
  uint32_t n_live[2];
  uint16_t live[2][kMaxTiles];
  float xm[2][kBM];   // per-row running max of each half (epilogue exchange)
  float xl[2][kBM];   // per-row FP32 sum of each half
  float xo[2][kBM];   // per-row sum of the weights as rounded for the MMA
};

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
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

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

struct Item {
  int qt, bh, q0, rows_valid;
};

__device__ __forceinline__ Item item_of(int w, int BH, int QT, int N) {
  Item it;
  it.qt = QT - 1 - w / BH;  // heaviest (largest) query tiles first
  it.bh = w % BH;
  it.q0 = it.qt * kBM;
  it.rows_valid = min(kBM, N - it.q0);
  return it;
}

template <bool BF16, int NS>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_persist_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                            const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                            const uint32_t* __restrict__ mask, float* __restrict__ lse, int N, int BH, int W,
                            int KT, int total_items, float scale_log2, uint32_t* err_word, uint64_t timeout_ns) {
  extern __shared__ __align__(1024) uint8_t smem[];
  // Q[2] | stages | O staging | mask[2] | control
  const uint32_t base = smem_u32(smem);
  if ((base & 1023u) != 0u) {
    if (threadIdx.x == 0) atomicOr(err_word, kDevErrLayout);
    return;
  }
  const uint32_t sQ0 = base;
  const uint32_t sStage = sQ0 + 2 * kQBytes;
  const uint32_t sOut = sStage + NS * kStageBytes;
  uint8_t* out_ptr = smem + (sOut - base);
  const uint32_t mask_words = static_cast<uint32_t>(kBM) * W;
  const uint32_t mask_buf_bytes = (mask_words * 4u + 15u) & ~15u;
  uint32_t* smask0 = reinterpret_cast<uint32_t*>(out_ptr + kStagingBytes);
  Ctl& ctl = *reinterpret_cast<Ctl*>(reinterpret_cast<uint8_t*>(smask0) + 2 * mask_buf_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int QT = (N + kBM - 1) / kBM;
  const int G = gridDim.x;
  const int n_items = total_items > static_cast<int>(blockIdx.x)
                          ? (total_items - static_cast<int>(blockIdx.x) + G - 1) / G
                          : 0;
  volatile uint32_t* abort_flag = &ctl.abort_flag;

  if (threadIdx.x == 256) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&ctl.sched_full[b]), 1);
      mbar_init(smem_u32(&ctl.mask_empty[b]), 8);
      mbar_init(smem_u32(&ctl.mask_full[b]), 1);
      mbar_init(smem_u32(&ctl.q_full[b]), 1);
      mbar_init(smem_u32(&ctl.q_empty[b]), 1);
      mbar_init(smem_u32(&ctl.s_full[b]), 1);
      mbar_init(smem_u32(&ctl.s_free[b]), 8);
      mbar_init(smem_u32(&ctl.p_full[b]), 8);
      mbar_init(smem_u32(&ctl.pv_done[b]), 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_u32(&ctl.k_full[s]), 1);
      mbar_init(smem_u32(&ctl.k_empty[s]), 1);
      mbar_init(smem_u32(&ctl.v_full[s]), 1);
      mbar_init(smem_u32(&ctl.v_empty[s]), 1);
    }
    mbar_init(smem_u32(&ctl.o_free), 8);
    mbar_init(smem_u32(&ctl.drain[0]), 1);
    mbar_init(smem_u32(&ctl.drain[1]), 1);
    ctl.abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;
#ifdef SMA_REG_SPLIT
  if (warp >= 8)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
  else
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
#endif

  auto fail = [&]() {
    ctl.abort_flag = 1;
    atomicOr(err_word, kDevErrTimeout);
  };

  if (warp == 11) {
    // ================================================================ scheduler
    // Runs up to two items ahead of the softmax: bulk-copies each item's
    // packed-mask row block into its slot, scans it for live key tiles and
    // publishes the list (sched_full).
    uint32_t bulk_count[2] = {0u, 0u};  // bulk copies issued into each slot
    bool mask_pending = false;          // abort path: a copy is in flight
    int pending_slot = 0;
    bool ok = true;
    for (int j = 0; ok && j < n_items; ++j) {
      const int slot = j & 1;
      const Item it = item_of(static_cast<int>(blockIdx.x) + j * G, BH, QT, N);
      uint32_t* smask = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(smask0) + slot * mask_buf_bytes);
      // The softmax warps read this slot's mask words until they finish item j-2.
      if (j >= 2) {
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.mask_empty[slot]), ((j - 2) >> 1) & 1,
                                                       abort_flag, timeout_ns));
        if (!ok) break;
      }
      const uint32_t* gmask = mask + (static_cast<int64_t>(it.bh) * N + it.q0) * W;
      const uint32_t nbytes = static_cast<uint32_t>(it.rows_valid) * W * 4u;
      const bool bulk_ok = ((reinterpret_cast<uintptr_t>(gmask) & 15u) == 0) && ((nbytes & 15u) == 0);
      if (bulk_ok) {
        if (lane == 0) {
          mbar_arrive_expect_tx(smem_u32(&ctl.mask_full[slot]), nbytes);
          bulk_load(smem_u32(smask), gmask, nbytes, smem_u32(&ctl.mask_full[slot]));
        }
        mask_pending = true;
        pending_slot = slot;
      } else {
        for (uint32_t i = lane; i < static_cast<uint32_t>(it.rows_valid) * W; i += 32) smask[i] = gmask[i];
      }
      for (uint32_t i = it.rows_valid * W + lane; i < mask_words; i += 32) smask[i] = 0u;
      if (bulk_ok) {
        // mask_full[slot] completes once per bulk copy into the slot.
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.mask_full[slot]), bulk_count[slot] & 1,
                                                       abort_flag, timeout_ns));
        if (!ok) break;
        ++bulk_count[slot];
        mask_pending = false;
      }
      __syncwarp();
      // Column-word liveness over the 128 rows (lanes read consecutive words).
      uint32_t colbits[2] = {0u, 0u};  // W <= 64
      if (W <= 32 && (32 % W) == 0) {
        const int c = lane % W, g = lane / W, GG = 32 / W;
        uint32_t acc = 0;
#pragma unroll 8
        for (int r = g; r < kBM; r += GG) acc |= smask[r * W + c];
        uint32_t nz = __ballot_sync(0xffffffffu, acc != 0u);
        for (int sh = W; sh < 32; sh <<= 1) nz |= nz >> sh;
        colbits[0] = (W == 32) ? nz : (nz & ((1u << W) - 1u));
      } else {
        for (int c0 = 0; c0 < W; c0 += 32) {
          const int c = c0 + lane;
          uint32_t acc = 0;
          if (c < W) {
#pragma unroll 8
            for (int r = 0; r < kBM; ++r) acc |= smask[r * W + c];
          }
          colbits[c0 >> 5] = __ballot_sync(0xffffffffu, acc != 0u);
        }
      }
      if (lane == 0) {
        uint32_t n = 0;
        for (int t = 0; t < KT; ++t) {
          const int w0 = t * 4;  // four 32-bit words per 128-key tile
          if ((colbits[w0 >> 5] >> (w0 & 31)) & 0xFu) ctl.live[slot][n++] = static_cast<uint16_t>(t);
        }
        ctl.n_live[slot] = n;
        mbar_arrive(smem_u32(&ctl.sched_full[slot]));
      }
      __syncwarp();
    }
    if (!ok && lane == 0) {
      fail();
      uint32_t zero = 0;
      if (mask_pending)
        mbar_wait_bounded(smem_u32(&ctl.mask_full[pending_slot]), bulk_count[pending_slot] & 1, &zero, timeout_ns);
    }
  } else if (warp == 8) {
    // ================================================================ loader
    // Streams Q (two buffers) and K / V of every live tile of every item
    // through the stage rings, as far ahead as the rings allow.
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_o);
      uint32_t kv_count = 0;   // K/V tiles issued over all items
      uint32_t q_count = 0;    // Q tiles issued (items with at least one live tile)
      bool k_only = false;     // abort path: K of tile kv_count issued, V not
      bool ok = true;
      for (int j = 0; ok && j < n_items; ++j) {
        const int slot = j & 1;
        if (!mbar_wait_bounded(smem_u32(&ctl.sched_full[slot]), (j >> 1) & 1, abort_flag, timeout_ns)) {
          ok = false;
          break;
        }
        const uint32_t n = ctl.n_live[slot];
        if (n == 0) continue;
        const Item it = item_of(static_cast<int>(blockIdx.x) + j * G, BH, QT, N);
        // Q of this item into Q buffer q_count % 2, once the last QK^T of the
        // item that used it has completed.
        const int qb = q_count & 1;
        if (q_count >= 2 &&
            !mbar_wait_bounded(smem_u32(&ctl.q_empty[qb]), ((q_count - 2) >> 1) & 1, abort_flag, timeout_ns)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(smem_u32(&ctl.q_full[qb]), kQBytes);
        tma_load_3d(sQ0 + qb * kQBytes, &tm_q, smem_u32(&ctl.q_full[qb]), 0, it.q0, it.bh);
        ++q_count;
        // K and V of a tile go to separate rings: K is released as soon as
        // its QK^T completes, V only after the PV.
        for (uint32_t t = 0; ok && t < n; ++t, ++kv_count) {
          const int stage = kv_count % NS;
          const uint32_t reuse_parity = ((kv_count / NS) - 1) & 1;
          const int kt = ctl.live[slot][t];
          const uint32_t sK = sStage + stage * kStageBytes;
          if (kv_count >= static_cast<uint32_t>(NS) &&
              !mbar_wait_bounded(smem_u32(&ctl.k_empty[stage]), reuse_parity, abort_flag, timeout_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(smem_u32(&ctl.k_full[stage]), kKBytes);
          tma_load_3d(sK, &tm_k, smem_u32(&ctl.k_full[stage]), 0, kt * kBN, it.bh);
          if (kv_count >= static_cast<uint32_t>(NS) &&
              !mbar_wait_bounded(smem_u32(&ctl.v_empty[stage]), reuse_parity, abort_flag, timeout_ns)) {
            ok = false;
            k_only = true;  // this tile's K copy is in flight, its V copy is not
            break;
          }
          mbar_arrive_expect_tx(smem_u32(&ctl.v_full[stage]), kKBytes);
          tma_load_3d(sK + kKBytes, &tm_v, smem_u32(&ctl.v_full[stage]), 0, kt * kBN, it.bh);
        }
      }
      if (!ok) {
        fail();
        // Let the copies this thread started land before the CTA exits.
        uint32_t zero = 0;
        const uint32_t first = kv_count > static_cast<uint32_t>(NS) ? kv_count - NS : 0u;
        for (uint32_t c = first; c < kv_count; ++c) {
          mbar_wait_bounded(smem_u32(&ctl.k_full[c % NS]), (c / NS) & 1, &zero, timeout_ns);
          mbar_wait_bounded(smem_u32(&ctl.v_full[c % NS]), (c / NS) & 1, &zero, timeout_ns);
        }
        if (k_only) mbar_wait_bounded(smem_u32(&ctl.k_full[kv_count % NS]), (kv_count / NS) & 1, &zero, timeout_ns);
        for (uint32_t q = (q_count > 2 ? q_count - 2 : 0); q < q_count; ++q)
          mbar_wait_bounded(smem_u32(&ctl.q_full[q & 1]), (q >> 1) & 1, &zero, timeout_ns);
      }
    }
  } else if (warp == 9) {
    // ================================================================ QK^T issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kBM, kBN, BF16 ? 1 : 0, 0);
      bool ok = true;
      uint32_t g = 0;        // global tile index (all items of this CTA)
      uint32_t q_count = 0;  // items with at least one live tile
      for (int j = 0; ok && j < n_items; ++j) {
        const int slot = j & 1;
        if (!mbar_wait_bounded(smem_u32(&ctl.sched_full[slot]), (j >> 1) & 1, abort_flag, timeout_ns)) {
          ok = false;
          break;
        }
        const uint32_t n = ctl.n_live[slot];
        if (n == 0) continue;
        const int qb = q_count & 1;
        if (!mbar_wait_bounded(smem_u32(&ctl.q_full[qb]), (q_count >> 1) & 1, abort_flag, timeout_ns)) {
          ok = false;
          break;
        }
        const uint32_t sQ = sQ0 + qb * kQBytes;
        for (uint32_t t = 0; t < n; ++t, ++g) {
          const int stage = g % NS;
          const int sb = g & 1;
          if (!mbar_wait_bounded(smem_u32(&ctl.k_full[stage]), (g / NS) & 1, abort_flag, timeout_ns) ||
              (g >= 2 && !mbar_wait_bounded(smem_u32(&ctl.s_free[sb]), ((g - 2) >> 1) & 1, abort_flag, timeout_ns))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sK = sStage + stage * kStageBytes;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk)
            mma_ss(tmem + kSCol + sb * kBN, smem_desc_sw128(sQ + kk * 32, 16, 1024),
                   smem_desc_sw128(sK + kk * 32, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
          mma_commit(smem_u32(&ctl.s_full[sb]));
          mma_commit(smem_u32(&ctl.k_empty[stage]));
          if (t + 1 == n) mma_commit(smem_u32(&ctl.q_empty[qb]));  // Q buffer free after the last QK^T
        }
        ++q_count;
      }
      if (!ok) fail();
      // Every MMA this thread issued must complete (and every commit arrive)
      // before the CTA releases TMEM and exits.
      mma_commit(smem_u32(&ctl.drain[0]));
      uint32_t zero = 0;
      mbar_wait_bounded(smem_u32(&ctl.drain[0]), 0, &zero, timeout_ns);
    }
  } else if (warp == 10) {
    // ================================================================ PV issuer
    if (lane == 0) {
      constexpr uint32_t idesc_pv = make_idesc_f16(kBM, kD, BF16 ? 1 : 0, 1);
      bool ok = true;
      uint32_t g = 0;
      for (int j = 0; ok && j < n_items; ++j) {
        const int slot = j & 1;
        if (!mbar_wait_bounded(smem_u32(&ctl.sched_full[slot]), (j >> 1) & 1, abort_flag, timeout_ns)) {
          ok = false;
          break;
        }
        const uint32_t n = ctl.n_live[slot];
        if (n == 0) continue;
        for (uint32_t t = 0; t < n; ++t, ++g) {
          const int stage = g % NS;
          const int pb = g & 1;
          // O0/O1 are overwritten by an item's first PV: the epilogue of the
          // previous item must have read them.
          if ((t == 0 && j > 0 && !mbar_wait_bounded(smem_u32(&ctl.o_free), (j - 1) & 1, abort_flag, timeout_ns)) ||
              !mbar_wait_bounded(smem_u32(&ctl.p_full[pb]), (g >> 1) & 1, abort_flag, timeout_ns) ||
              !mbar_wait_bounded(smem_u32(&ctl.v_full[stage]), (g / NS) & 1, abort_flag, timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sV = sStage + stage * kStageBytes + kKBytes;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int kk = 0; kk < kHalf / 16; ++kk) {
              const uint64_t bdesc = smem_desc_sw128(sV + h * (kHalf * 128) + kk * 2048, kBN * 128, 1024);
              mma_ts(tmem + kOCol + h * kD, tmem + kPCol + pb * kHalf + h * (kHalf / 2) + kk * 8, bdesc, idesc_pv,
                     (t > 0 || kk > 0) ? 1u : 0u);
            }
          }
          mma_commit(smem_u32(&ctl.v_empty[stage]));
          mma_commit(smem_u32(&ctl.pv_done[pb]));
        }
      }
      if (!ok) fail();
      mma_commit(smem_u32(&ctl.drain[1]));
      uint32_t zero = 0;
      mbar_wait_bounded(smem_u32(&ctl.drain[1]), 0, &zero, timeout_ns);
    }
  } else if (warp < 8) {
    // ================================================================ softmax WGs
    const int wg = warp >> 2;           // key half: 0 -> keys 0-63, 1 -> keys 64-127 of each tile
    const int r = threadIdx.x & 127;    // query row == TMEM lane
    const uint32_t t_lane = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    bool ok = true;
    uint32_t g_base = 0;
    uint32_t mask_j = 0;
    for (int j = 0; j < n_items; ++j) {
      const int slot = j & 1;
      const Item it = item_of(static_cast<int>(blockIdx.x) + j * G, BH, QT, N);
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.sched_full[slot]), (j >> 1) & 1,
                                                              abort_flag, timeout_ns));
      const uint32_t n = ok ? ctl.n_live[slot] : 0u;
      const uint32_t* mrow =
          reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(smask0) + slot * mask_buf_bytes) + r * W;
      float m_run = -INFINITY, l_run = 0.f, l_out = 0.f;

      // Mask words (two per half-tile) of tile t for this row, bits >= N cleared.
      auto mask_words = [&](uint32_t t, uint32_t (&mw)[2]) {
        const int kt = ctl.live[slot][t];
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          const int cw = kt * 4 + wg * 2 + w;
          const int valid = N - cw * 32;
          uint32_t v = (cw < W) ? mrow[cw] : 0u;
          if (valid < 32) v = (valid <= 0) ? 0u : (v & ((1u << valid) - 1u));
          mw[w] = v;
        }
      };
      auto wait_s = [&](uint32_t g) -> bool {
        const bool all = __all_sync(
            0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.s_full[g & 1]), (g >> 1) & 1, abort_flag, timeout_ns));
        if (all) tc_fence_after();
        return all;
      };
      auto load_chunk = [&](uint32_t g, int c, float* dst) {
        tmem_ld32f(t_lane + kSCol + (g & 1) * kBN + wg * kHalf + c * 32, dst);
        tmem_wait_ld();
      };
      auto release_s = [&](uint32_t g) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl.s_free[g & 1]));
      };
      auto mask_max_chunk = [&](float* v, uint32_t word, float (&mx)[4]) {
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          const float v0 = (word & (1u << jj)) ? v[jj] : -INFINITY;
          const float v1 = (word & (2u << jj)) ? v[jj + 1] : -INFINITY;
          v[jj] = v0;
          v[jj + 1] = v1;
          mx[(jj >> 1) & 3] = max3f(mx[(jj >> 1) & 3], v0, v1);
        }
      };
      auto update_max = [&](const float (&mx)[4], float& alpha) -> bool {
        const float x_max = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
        alpha = 1.f;
        bool rescale = false;
        if (x_max > m_run + kRescaleThreshold) {
          if (m_run != -INFINITY) {
            alpha = ex2f(m_run - x_max);
            rescale = true;
          }
          l_run *= alpha;
          l_out *= alpha;
          m_run = x_max;
        }
        return rescale;
      };

      float buf[kHalf];
      float alpha_cur = 1.f;
      bool rescale_cur = false;
      if (ok && n > 0) {
        ok = wait_s(g_base);
        if (ok) {
          uint32_t mw[2];
          mask_words(0, mw);
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            load_chunk(g_base, c, buf + c * 32);
            mask_max_chunk(buf + c * 32, mw[c], mx);
          }
          release_s(g_base);
          rescale_cur = update_max(mx, alpha_cur);
        }
      }
      for (uint32_t t = 0; ok && t < n; ++t) {
        const uint32_t g = g_base + t;
        const bool has_next = t + 1 < n;
        const int pb = g & 1;
        if (has_next && !wait_s(g + 1)) {
          ok = false;
          break;
        }
        if (g >= 2) {
          // P buffer pb was last read by the PV of tile g-2.
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.pv_done[pb]), ((g - 2) >> 1) & 1, abort_flag,
                                                          timeout_ns))) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        uint32_t mwn[2];
        if (has_next) mask_words(t + 1, mwn);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        float la[4] = {0.f, 0.f, 0.f, 0.f};
        float lr[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const float p0 = ex2f(fmaf(buf[c * 32 + 2 * jj], scale_log2, -m_use));
            const float p1 = ex2f(fmaf(buf[c * 32 + 2 * jj + 1], scale_log2, -m_use));
            pk[jj] = pack2<BF16>(p0, p1);
            la[jj & 3] += p0 + p1;
            if constexpr (BF16) {
              lr[jj & 3] += __uint_as_float(pk[jj] << 16) + __uint_as_float(pk[jj] & 0xFFFF0000u);
            }
          }
          tmem_st16(t_lane + kPCol + pb * kHalf + wg * (kHalf / 2) + c * 16, pk);
          if (has_next) {
            load_chunk(g + 1, c, buf + c * 32);
            mask_max_chunk(buf + c * 32, mwn[c], mx);
          }
        }
        if (has_next) release_s(g + 1);
        const float l_tile = (la[0] + la[1]) + (la[2] + la[3]);
        l_run += l_tile;
        l_out += BF16 ? (lr[0] + lr[1]) + (lr[2] + lr[3]) : l_tile;
        if (t > 0 && __any_sync(0xffffffffu, rescale_cur)) {
          // Rare: this half's running max rose by more than the threshold.
          // Rescale its O once the PV of tile g-1 has finished.
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.pv_done[(g - 1) & 1]), ((g - 1) >> 1) & 1,
                                                          abort_flag, timeout_ns))) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < kD / 32; ++c) {
            uint32_t u[32];
            tmem_ld32(t_lane + kOCol + wg * kD + c * 32, u);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 32; ++q) u[q] = __float_as_uint(__uint_as_float(u[q]) * alpha_cur);
            tmem_st32(t_lane + kOCol + wg * kD + c * 32, u);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl.p_full[pb]));
        if (has_next) rescale_cur = update_max(mx, alpha_cur);
      }
      // Mask words of this item are no longer read.
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.mask_empty[slot]));
      ++mask_j;

      // ------------------------------------------------------------ epilogue
      if (threadIdx.x == 0) bulk_wait_group_read0();  // staging buffer free again
      if (ok && n > 0) {
        const uint32_t g_last = g_base + n - 1;
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.pv_done[g_last & 1]), (g_last >> 1) & 1,
                                                        abort_flag, timeout_ns));
        if (ok) tc_fence_after();
      }
      ctl.xm[wg][r] = m_run;
      ctl.xl[wg][r] = l_run;
      ctl.xo[wg][r] = l_out;
      named_bar_sync(1, 256);
      const float m0 = ctl.xm[0][r], m1 = ctl.xm[1][r];
      const float m = fmaxf(m0, m1);
      const float f0 = (m0 == -INFINITY) ? 0.f : ex2f(m0 - m);
      const float f1 = (m1 == -INFINITY) ? 0.f : ex2f(m1 - m);
      const float l_tot = ctl.xl[0][r] * f0 + ctl.xl[1][r] * f1;
      const float lo_tot = ctl.xo[0][r] * f0 + ctl.xo[1][r] * f1;
      const float inv = (lo_tot > 0.f) ? (1.f / lo_tot) : 0.f;
      // This WG writes output columns [32 wg, 32 wg + 32).
      {
        uint32_t u0[32], u1[32];
        if (ok && n > 0) {
          tmem_ld32(t_lane + kOCol + 0 * kD + wg * 32, u0);
          tmem_ld32(t_lane + kOCol + 1 * kD + wg * 32, u1);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) u0[q] = u1[q] = 0u;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctl.o_free));
        const float s0 = f0 * inv, s1 = f1 * inv;
        uint32_t h[16];
#pragma unroll
        for (int q = 0; q < 16; ++q)
          h[q] = pack2<BF16>(__uint_as_float(u0[2 * q]) * s0 + __uint_as_float(u1[2 * q]) * s1,
                             __uint_as_float(u0[2 * q + 1]) * s0 + __uint_as_float(u1[2 * q + 1]) * s1);
        uint8_t* row = out_ptr + r * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = (wg * 4 + q) ^ (r & 7);  // 128-byte swizzle of the O tensor map
          *reinterpret_cast<uint4*>(row + chunk * 16) = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
        }
      }
      if (wg == 0 && lse != nullptr && r < it.rows_valid) {
        lse[static_cast<int64_t>(it.bh) * N + it.q0 + r] = (l_tot > 0.f) ? (m + log2f(l_tot)) * kLn2 : -FLT_MAX;
      }
      fence_proxy_async_smem();
      named_bar_sync(1, 256);
      if (threadIdx.x == 0 && ctl.abort_flag == 0) {
        tma_store_3d(&tm_o, sOut, 0, it.q0, it.bh);
        bulk_commit_group();
      }
      g_base += n;
    }
    if (!ok && lane == 0) fail();
    if (threadIdx.x == 0) bulk_wait_group_read0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

bool map3d(CUtensorMap* m, const void* ptr, int dtype, int64_t BH, int64_t N, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD * 2), static_cast<cuuint64_t>(N * kD * 2)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(m, dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
            const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <bool BF16, int NS>
int launch(const AttnParams& p, const char** msg) {
  const int64_t BH = p.B * p.H;
  const int64_t N = p.N;
  const int64_t W = (N + 31) / 32;
  const int64_t KT = (N + kBN - 1) / kBN;
  const int64_t QT = (N + kBM - 1) / kBM;
  const int64_t total = QT * BH;
  if (total > 0x7FFFFFFFll) {
    *msg = "attention: batch*heads too large";
    return kErrArg;
  }
  CUtensorMap mq, mk, mv, mo;
  if (!map3d(&mq, p.q, p.dtype, BH, N, kBM) || !map3d(&mk, p.k, p.dtype, BH, N, kBN) ||
      !map3d(&mv, p.v, p.dtype, BH, N, kBN) || !map3d(&mo, p.out, p.dtype, BH, N, kBM)) {
    *msg = "attention: cuTensorMapEncodeTiled failed (pointer alignment or driver entry point)";
    return kErrCuda;
  }
  const size_t mask_buf = (static_cast<size_t>(kBM) * W * 4 + 15) / 16 * 16;
  // The kernel owns all of TMEM: the shared-memory request (> half an SM)
  // guarantees one resident CTA per SM whatever the sequence length.
  size_t smem = 2 * kQBytes + NS * kStageBytes + kStagingBytes + 2 * mask_buf + sizeof(Ctl);
  if (smem < kMinSmem) smem = kMinSmem;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *msg = "attention: no current CUDA device";
    return kErrCuda;
  }
  static int sms[kMaxDevices] = {};
  static size_t smem_set[kMaxDevices] = {};
  if (sms[dev] == 0 && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    *msg = "attention: cannot query the SM count";
    return kErrCuda;
  }
  auto kern = attn_fwd_persist_kernel<BF16, NS>;
  if (smem > smem_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) {
      *msg = cudaGetErrorString(e);
      return kErrLaunch;
    }
    smem_set[dev] = smem;
  }
  const int grid = static_cast<int>(total < sms[dev] ? total : sms[dev]);
  kern<<<grid, kThreads, smem, p.stream>>>(mq, mk, mv, mo, p.mask, p.lse, static_cast<int>(N),
                                           static_cast<int>(BH), static_cast<int>(W), static_cast<int>(KT),
                                           static_cast<int>(total), p.scale * kLog2e, p.err_word, p.timeout_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    static thread_local char buf[256];
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    snprintf(buf, sizeof(buf), "%s (persistent kernel: %d threads, %d regs/thread, max %d threads/block, %zu B dynamic smem)",
             cudaGetErrorString(e), kThreads, fa.numRegs, fa.maxThreadsPerBlock, smem);
    *msg = buf;
    return kErrLaunch;
  }
  return kOk;
}

}  // namespace

bool persist_supported(const AttnParams& p) { return p.D == kD && p.N <= kMaxTiles * kBN; }

int launch_attn_fwd_persist(const AttnParams& p, const char** msg) {
  // Four K/V stages while the two mask slots are small (N <= 1024), three above.
  if (p.N <= 1024) return p.dtype == 1 ? launch<true, 4>(p, msg) : launch<false, 4>(p, msg);
  return p.dtype == 1 ? launch<true, 3>(p, msg) : launch<false, 3>(p, msg);
}

}  // namespace sma
