// Fused masked-softmax attention forward for sm_100a (B200).
//
// Computes, per (batch*head, query row r):
//   s_j  = scale * <q_r, k_j>                     for every key j with mask bit set
//   O_r  = sum_j softmax(s)_j * v_j               (0 if the row has no set bit)
//   lse_r = log(sum_j exp(s_j))                   (-FLT_MAX if the row has no set bit)
// which is the reference forward (csrc/sparse_attention.cu:64-143; FP32 oracle
// python/sparse_attention.py:26-44).
//
// Work decomposition: one CTA per (batch*head, 128-row query tile).  Keys are
// processed in BN-wide tiles; a key tile whose packed-mask words are all zero
// for the 128 rows of the query tile is never loaded and never multiplied.
//
// Warp roles (192 threads):
//   warps 0-3  softmax / correction / epilogue; thread t owns query row t and
//              TMEM lane t (tcgen05.ld/st 32x32b shapes)
//   warp 4     producer: bulk-copies the query tile's packed-mask row block
//              into shared memory, scans it for live key tiles, then issues
//              the TMA loads of Q and of K/V for live tiles only
//   warp 5     TMEM allocator + single-thread tcgen05.mma issuer
//
// Per live key tile i the pipeline is
//   TMA K_i,V_i -> MMA S = Q K_i^T (TMEM) -> softmax: S -> P (fp16/bf16 in TMEM)
//   -> MMA O += P V_i (A operand straight from TMEM)
// with a K/V stage ring.  S is released as soon as the softmax warps have
// copied it to registers (and is double-buffered when TMEM allows), so QK^T
// of tile i+1 runs on the tensor core while tile i is exponentiated, and
// PV of tile i-1 runs while tile i's row maxima are reduced.
//
// Softmax: base-2 online softmax in FP32 registers.  The running maximum is
// only raised when a tile's maximum exceeds it by more than 8 (log2 units),
// so rescaling the O accumulator in TMEM is rare; values of P stay <= 2^8.
//
// TMEM columns (256 allocated, two CTAs per SM):
//   S buffers [0, kSBuf*BN)   P buffers [kSBuf*BN, +kPBuf*BN/2)   O [256-D, 256)
#include <cfloat>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "sma_internal.h"
#include "sma_ptx.cuh"

namespace sma {
namespace {

constexpr int kBM = 128;
constexpr int kThreads = 192;
constexpr int kTmemCols = 256;
constexpr int kMaxTiles = 128;  // kMaxSeqLen / 64
constexpr int kMaxStages = 4;
constexpr int kMaxDevices = 64;
constexpr size_t kMinSmemPerCta = 80 * 1024;  // > 228 KiB / 3
constexpr float kRescaleThreshold = 8.0f;
constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kLog2e = 1.44269504088896340736f;

template <int D, int BN>
struct Cfg {
  static_assert(D == 64 || D == 128, "head dim");
  static_assert(BN == 64, "key tile");
  static constexpr int kDChunks = D / 64;          // 128-byte swizzle chunks per row
  static constexpr int kQBytes = kBM * D * 2;
  static constexpr int kKBytes = BN * D * 2;
  static constexpr int kStageBytes = 2 * kKBytes;  // K + V
  // TMEM buffering within half of TMEM (two CTAs per SM): a second P buffer
  // first (the softmax then never waits for the previous PV before writing
  // P), then a second S buffer (QK^T may run two tiles ahead).
  static constexpr int kPBuf = (BN + 2 * (BN / 2) + D <= kTmemCols) ? 2 : 1;
  static constexpr int kSBuf = (2 * BN + kPBuf * (BN / 2) + D <= kTmemCols) ? 2 : 1;
  static constexpr int kSCol = 0;
  static constexpr int kPCol = kSBuf * BN;
  static constexpr int kOCol = kTmemCols - D;
  static_assert(kPCol + kPBuf * (BN / 2) <= kOCol, "TMEM budget");
  // K/V ring depth: as deep as 64 KiB of shared memory allows.
  static constexpr int kStages = (65536 / kStageBytes) < kMaxStages ? (65536 / kStageBytes) : kMaxStages;
  static_assert(kStages >= 2, "stages");
  static constexpr int kWordsPerTile = BN / 32;
};

struct SharedCtl {
  uint64_t q_full;
  uint64_t mask_full;
  uint64_t sched;
  uint64_t kv_full[kMaxStages];
  uint64_t kv_empty[kMaxStages];
  uint64_t s_full[2];
  uint64_t s_free[2];
  uint64_t p_full[2];
  uint64_t pv_done[2];
  uint64_t drain;
  uint32_t colbits[8];
  uint32_t tmem_base;
  uint32_t n_live;
  uint32_t abort_flag;
  uint16_t live[kMaxTiles];
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

__device__ __forceinline__ void record_abort(SharedCtl* ctl, uint32_t* err_word) {
  ctl->abort_flag = 1;
  atomicOr(err_word, kDevErrTimeout);
}

template <int D, int BN, bool BF16>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                    const uint32_t* __restrict__ mask, float* __restrict__ lse, int N, int BH, int W,
                    int KT, float scale_log2, uint32_t* err_word, uint64_t timeout_ns) {
  using C = Cfg<D, BN>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(1024) uint8_t dyn_smem[];

  // Carve-up (no static shared memory, so the dynamic window starts on a
  // 1024-byte boundary as the 128-byte-swizzled tiles require):
  //   Q | S x (K, V) | mask rows | control block
  const uint32_t base = smem_u32(dyn_smem);
  if ((base & 1023u) != 0u) {
    if (threadIdx.x == 0) atomicOr(err_word, kDevErrLayout);
    return;
  }
  uint8_t* base_ptr = dyn_smem;
  const uint32_t sQ = base;
  const uint32_t sStage = sQ + C::kQBytes;
  uint32_t* smask = reinterpret_cast<uint32_t*>(base_ptr + C::kQBytes + S * C::kStageBytes);
  SharedCtl& ctl = *reinterpret_cast<SharedCtl*>(base_ptr + C::kQBytes + S * C::kStageBytes +
                                                 ((static_cast<uint32_t>(kBM) * W * 4u + 15u) & ~15u));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Heaviest query tiles (largest index, most keys under a causal mask) first.
  const int QT = (N + kBM - 1) / kBM;
  const int qt = QT - 1 - static_cast<int>(blockIdx.x / BH);
  const int bh = static_cast<int>(blockIdx.x % BH);
  const int q0 = qt * kBM;
  const int rows_valid = min(kBM, N - q0);

  volatile uint32_t* abort_flag = &ctl.abort_flag;

  if (threadIdx.x == 128) {
    mbar_init(smem_u32(&ctl.q_full), 1);
    mbar_init(smem_u32(&ctl.mask_full), 1);
    mbar_init(smem_u32(&ctl.sched), 1);
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&ctl.kv_full[s]), 1);
      mbar_init(smem_u32(&ctl.kv_empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&ctl.s_full[b]), 1);
      mbar_init(smem_u32(&ctl.s_free[b]), 4);
      mbar_init(smem_u32(&ctl.p_full[b]), 4);
      mbar_init(smem_u32(&ctl.pv_done[b]), 1);
    }
    mbar_init(smem_u32(&ctl.drain), 1);
    ctl.abort_flag = 0;
    ctl.n_live = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;
  // Set-up above overlaps the previous kernel in the stream (see launch_pdl).
  pdl_wait_prior_grid();

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    const int64_t mask_row0 = static_cast<int64_t>(bh) * N + q0;
    const uint32_t* gmask = mask + mask_row0 * W;
    const uint32_t mask_bytes = static_cast<uint32_t>(rows_valid) * W * 4u;
    const bool bulk_ok = ((reinterpret_cast<uintptr_t>(gmask) & 15u) == 0) && ((mask_bytes & 15u) == 0);
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_o);
      if (bulk_ok) {
        mbar_arrive_expect_tx(smem_u32(&ctl.mask_full), mask_bytes);
        bulk_load(smem_u32(smask), gmask, mask_bytes, smem_u32(&ctl.mask_full));
      }
      mbar_arrive_expect_tx(smem_u32(&ctl.q_full), C::kQBytes);
      for (int dc = 0; dc < C::kDChunks; ++dc)
        tma_load_3d(sQ + dc * (kBM * 128), &tm_q, smem_u32(&ctl.q_full), dc * 64, q0, bh);
    }
    if (!bulk_ok) {
      for (uint32_t i = lane; i < static_cast<uint32_t>(rows_valid) * W; i += 32) smask[i] = gmask[i];
    }
    for (uint32_t i = rows_valid * W + lane; i < static_cast<uint32_t>(kBM) * W; i += 32) smask[i] = 0u;
    bool ok = true;
    if (bulk_ok) ok = mbar_wait_bounded(smem_u32(&ctl.mask_full), 0, abort_flag, timeout_ns);
    ok = __all_sync(0xffffffffu, ok);
    __syncwarp();

    uint32_t n_live = 0;
    if (ok) {
      // Column-word liveness: OR of each packed-mask column word over the
      // 128 rows.  Lanes read consecutive words of a row (no bank conflicts).
      if (W <= 32 && (32 % W) == 0) {
        const int c = lane % W, g = lane / W, G = 32 / W;
        uint32_t acc = 0;
#pragma unroll 8
        for (int r = g; r < kBM; r += G) acc |= smask[r * W + c];
        uint32_t nz = __ballot_sync(0xffffffffu, acc != 0u);
        for (int sh = W; sh < 32; sh <<= 1) nz |= nz >> sh;  // fold row groups onto columns
        if (lane == 0) ctl.colbits[0] = (W == 32) ? nz : (nz & ((1u << W) - 1u));
      } else {
        for (int c0 = 0; c0 < W; c0 += 32) {
          const int c = c0 + lane;
          uint32_t acc = 0;
          if (c < W) {
#pragma unroll 8
            for (int r = 0; r < kBM; ++r) acc |= smask[r * W + c];
          }
          const uint32_t nz = __ballot_sync(0xffffffffu, acc != 0u);
          if (lane == 0) ctl.colbits[c0 >> 5] = nz;
        }
      }
      __syncwarp();
      // A key tile is live when any of its column words is.
      if (lane == 0) {
        for (int t = 0; t < KT; ++t) {
          const int w0 = t * C::kWordsPerTile;
          const uint32_t bits = (ctl.colbits[w0 >> 5] >> (w0 & 31)) & ((1u << C::kWordsPerTile) - 1u);
          if (bits) ctl.live[n_live++] = static_cast<uint16_t>(t);
        }
      }
    } else if (lane == 0) {
      record_abort(&ctl, err_word);
    }
    if (lane == 0) {
      ctl.n_live = n_live;
      mbar_arrive(smem_u32(&ctl.sched));

      // K/V loads for live tiles through the stage ring.
      int issued = 0;
      for (uint32_t i = 0; i < n_live; ++i) {
        const int stage = i % S;
        if (i >= S) {
          if (!mbar_wait_bounded(smem_u32(&ctl.kv_empty[stage]), ((i / S) - 1) & 1, abort_flag, timeout_ns)) {
            record_abort(&ctl, err_word);
            break;
          }
        }
        const int kt = ctl.live[i];
        const uint32_t sK = sStage + stage * C::kStageBytes;
        const uint32_t sV = sK + C::kKBytes;
        const uint32_t bar = smem_u32(&ctl.kv_full[stage]);
        mbar_arrive_expect_tx(bar, C::kStageBytes);
        for (int dc = 0; dc < C::kDChunks; ++dc) {
          tma_load_3d(sK + dc * (BN * 128), &tm_k, bar, dc * 64, kt * BN, bh);
          tma_load_3d(sV + dc * (BN * 128), &tm_v, bar, dc * 64, kt * BN, bh);
        }
        ++issued;
      }
      if (ctl.abort_flag) {
        // Let every copy this thread started land before the CTA exits
        // (these waits ignore the abort flag; copies need no other role).
        uint32_t zero = 0;
        mbar_wait_bounded(smem_u32(&ctl.q_full), 0, &zero, timeout_ns);
        for (int j = (issued > S ? issued - S : 0); j < issued; ++j)
          mbar_wait_bounded(smem_u32(&ctl.kv_full[j % S]), (j / S) & 1, &zero, timeout_ns);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kBM, BN, BF16 ? 1 : 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBM, D, BF16 ? 1 : 0, 1);
      bool ok = mbar_wait_bounded(smem_u32(&ctl.sched), 0, abort_flag, timeout_ns);
      const uint32_t n = ok ? ctl.n_live : 0u;
      if (ok && n > 0) ok = mbar_wait_bounded(smem_u32(&ctl.q_full), 0, abort_flag, timeout_ns);
      auto issue_pv = [&](uint32_t j) {
        const int stage = j % S;
        const int pb = j % C::kPBuf;
        const uint32_t sV = sStage + stage * C::kStageBytes + C::kKBytes;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bdesc = smem_desc_sw128(sV + kk * 2048, BN * 128, 1024);
          mma_ts(tmem + C::kOCol, tmem + C::kPCol + pb * (BN / 2) + kk * 8, bdesc, idesc_pv,
                 (j > 0 || kk > 0) ? 1u : 0u);
        }
        // The producer only waits for a stage it will refill; the last S
        // tiles release nothing, so no asynchronous arrive can outlive the
        // CTA (pv_done of the last tile is awaited by the epilogue).
        if (j + S < n) mma_commit(smem_u32(&ctl.kv_empty[stage]));
        mma_commit(smem_u32(&ctl.pv_done[pb]));
      };
      // QK^T of tile j into S buffer j % kSBuf, once K_j has landed and the
      // softmax has copied out the S of tile j - kSBuf.
      auto issue_qk = [&](uint32_t j) -> bool {
        const int stage = j % S;
        const int sb = j % C::kSBuf;
        if (!mbar_wait_bounded(smem_u32(&ctl.kv_full[stage]), (j / S) & 1, abort_flag, timeout_ns)) return false;
        if (j >= static_cast<uint32_t>(C::kSBuf) &&
            !mbar_wait_bounded(smem_u32(&ctl.s_free[sb]), ((j - C::kSBuf) / C::kSBuf) & 1, abort_flag, timeout_ns))
          return false;
        tc_fence_after();
        const uint32_t sK = sStage + stage * C::kStageBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          const uint32_t qoff = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
          mma_ss(tmem + C::kSCol + sb * BN, smem_desc_sw128(sQ + qoff, 16, 1024),
                 smem_desc_sw128(sK + koff, 16, 1024), idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(smem_u32(&ctl.s_full[sb]));
        return true;
      };
      for (uint32_t j = 0; ok && j < n && j < static_cast<uint32_t>(C::kSBuf); ++j) ok = issue_qk(j);
      for (uint32_t i = 0; ok && i < n; ++i) {
        // Tile i + kSBuf's QK^T only needs tile i's S copied out (early in
        // the softmax of tile i), so it overlaps that softmax.
        if (i + C::kSBuf < n && !issue_qk(i + C::kSBuf)) {
          ok = false;
          break;
        }
        if (!mbar_wait_bounded(smem_u32(&ctl.p_full[i % C::kPBuf]), (i / C::kPBuf) & 1, abort_flag, timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(i);
      }
      if (!ok) {
        record_abort(&ctl, err_word);
        // Every MMA issued so far must finish before TMEM is released.
        mma_commit(smem_u32(&ctl.drain));
        uint32_t zero = 0;
        mbar_wait_bounded(smem_u32(&ctl.drain), 0, &zero, timeout_ns);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0-3
    // Software-pipelined over key tiles: while the exponentials of tile i
    // are computed (MUFU), tile i+1 is copied out of TMEM and its masked row
    // maximum is reduced (ALU), so both pipes stay busy in every warp.  Each
    // 32-column chunk of tile i+1 is loaded into the registers the same
    // chunk of tile i has just been consumed from.
    const int r = threadIdx.x;  // query row within the tile == TMEM lane
    const uint32_t t_lane = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float m_run = -INFINITY;  // running max of scale*log2(e)*s (may lag the true max by <= 8)
    float l_run = 0.f;        // sum of 2^(x - m_run), FP32 weights (for the LSE)
    float l_out = 0.f;        // the same over the weights as rounded for the PV MMA (normalises O)
    bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.sched), 0, abort_flag, timeout_ns));
    const uint32_t n = ok ? ctl.n_live : 0u;
    const uint32_t* mrow = smask + r * W;
    constexpr int kChunks = BN / 32;

    // Mask words of tile i for this row, bits past N cleared.
    auto mask_words = [&](uint32_t i, uint32_t (&mw)[C::kWordsPerTile]) {
      const int kt = ctl.live[i];
#pragma unroll
      for (int w = 0; w < C::kWordsPerTile; ++w) {
        const int cw = kt * C::kWordsPerTile + w;
        const int valid = N - cw * 32;
        uint32_t v = (cw < W) ? mrow[cw] : 0u;
        if (valid < 32) v = (valid <= 0) ? 0u : (v & ((1u << valid) - 1u));
        mw[w] = v;
      }
    };
    // Wait for S of tile i; copy column chunk c (32 columns) to registers.
    auto wait_s = [&](uint32_t i) -> bool {
      const bool w = mbar_wait_bounded(smem_u32(&ctl.s_full[i % C::kSBuf]), (i / C::kSBuf) & 1, abort_flag, timeout_ns);
      const bool all = __all_sync(0xffffffffu, w);
      if (all) tc_fence_after();
      return all;
    };
    auto load_chunk = [&](uint32_t i, int c, float* dst) {
      tmem_ld32f(t_lane + C::kSCol + (i % C::kSBuf) * BN + c * 32, dst);
      tmem_wait_ld();
    };
    auto release_s = [&](uint32_t i) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.s_free[i % C::kSBuf]));
    };
    // Masked values in place (-inf where the bit is clear) and their max.
    auto mask_max_chunk = [&](float* v, uint32_t word, float (&mx)[4]) {
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        const float v0 = (word & (1u << j)) ? v[j] : -INFINITY;
        const float v1 = (word & (2u << j)) ? v[j + 1] : -INFINITY;
        v[j] = v0;
        v[j + 1] = v1;
        mx[(j >> 1) & 3] = max3f(mx[(j >> 1) & 3], v0, v1);
      }
    };
    // Lazy running-max update from a tile maximum; returns whether the O
    // accumulator needs rescaling by `alpha` before the next PV.
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

    float buf[BN];
    float alpha_cur = 1.f;
    bool rescale_cur = false;
    if (ok && n > 0) {
      ok = wait_s(0);
      if (ok) {
        uint32_t mw[C::kWordsPerTile];
        mask_words(0, mw);
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < kChunks; ++c) {
          load_chunk(0, c, buf + c * 32);
          mask_max_chunk(buf + c * 32, mw[c], mx);
        }
        release_s(0);
        rescale_cur = update_max(mx, alpha_cur);
      }
    }

    // One pipelined step: exponentials of tile i (masked values in `buf`,
    // running max already settled) interleaved with loading and reducing
    // tile i+1 into the same registers.
    auto step = [&](uint32_t i) -> bool {
      const bool has_next = i + 1 < n;
      const int pb = i % C::kPBuf;
      if (has_next && !wait_s(i + 1)) return false;
      if (i >= static_cast<uint32_t>(C::kPBuf)) {
        // P buffer pb was last read by the PV of tile i - kPBuf.
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.pv_done[pb]), ((i - C::kPBuf) / C::kPBuf) & 1,
                                                        abort_flag, timeout_ns)))
          return false;
        tc_fence_after();
      }
      uint32_t mwn[C::kWordsPerTile];
      if (has_next) mask_words(i + 1, mwn);
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      float la[4] = {0.f, 0.f, 0.f, 0.f};
      float lr[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float p0 = ex2f(fmaf(buf[c * 32 + 2 * j], scale_log2, -m_use));
          const float p1 = ex2f(fmaf(buf[c * 32 + 2 * j + 1], scale_log2, -m_use));
          pk[j] = pack2<BF16>(p0, p1);
          la[j & 3] += p0 + p1;
          if constexpr (BF16) {
            // With 8-bit mantissas the rounding of a dominant weight would
            // show up directly in O: normalise by the weights the MMA uses.
            lr[j & 3] += __uint_as_float(pk[j] << 16) + __uint_as_float(pk[j] & 0xFFFF0000u);
          }
        }
        tmem_st16(t_lane + C::kPCol + pb * (BN / 2) + c * 16, pk);
        if (has_next) {
          load_chunk(i + 1, c, buf + c * 32);
          mask_max_chunk(buf + c * 32, mwn[c], mx);
        }
      }
      if (has_next) release_s(i + 1);
      const float l_tile = (la[0] + la[1]) + (la[2] + la[3]);
      l_run += l_tile;
      l_out += BF16 ? (lr[0] + lr[1]) + (lr[2] + lr[3]) : l_tile;
      if (i > 0 && __any_sync(0xffffffffu, rescale_cur)) {
        // Rare: the running max rose by more than the threshold at tile i.
        // Rescale O in place once the PV of tile i-1 has finished
        // accumulating into it; the PV of tile i waits for p_full below.
        if (C::kPBuf > 1) {
          if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.pv_done[(i - 1) % C::kPBuf]),
                                                          ((i - 1) / C::kPBuf) & 1, abort_flag, timeout_ns)))
            return false;
          tc_fence_after();
        }
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t u[32];
          tmem_ld32(t_lane + C::kOCol + c * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) u[j] = __float_as_uint(__uint_as_float(u[j]) * alpha_cur);
          tmem_st32(t_lane + C::kOCol + c * 32, u);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctl.p_full[pb]));
      if (has_next) rescale_cur = update_max(mx, alpha_cur);
      return true;
    };

    for (uint32_t i = 0; ok && i < n; ++i) ok = step(i);
    if (!ok && lane == 0) record_abort(&ctl, err_word);

    // ------------------------------------------------------------ epilogue
    if (ok && n > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.pv_done[(n - 1) % C::kPBuf]),
                                                      ((n - 1) / C::kPBuf) & 1, abort_flag, timeout_ns));
      if (ok) tc_fence_after();
    } else if (ok) {
      // No live tile: O is all zero; the Q buffer doubles as staging, so the
      // Q load must have landed before it is overwritten.
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&ctl.q_full), 0, abort_flag, timeout_ns));
    }
    if (!ok && lane == 0) record_abort(&ctl, err_word);
    if (ok) {
      const float inv = (l_out > 0.f) ? (1.f / l_out) : 0.f;
      uint8_t* stage_row = base_ptr + r * 128;  // row r of each 128-row x 64-col chunk
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t u[32];
        if (n > 0) {
          tmem_ld32(t_lane + C::kOCol + c * 32, u);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) u[j] = 0u;
        }
        uint32_t h[16];
#pragma unroll
        for (int j = 0; j < 16; ++j)
          h[j] = pack2<BF16>(__uint_as_float(u[2 * j]) * inv, __uint_as_float(u[2 * j + 1]) * inv);
        // columns [32c, 32c+32) = 64 bytes = four 16-byte chunks of row r,
        // stored at the 128-byte-swizzled positions the O tensor map expects
        const int dc = c >> 1;
        uint8_t* chunk_base = stage_row + dc * (kBM * 128);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = ((c & 1) * 4 + q) ^ (r & 7);
          *reinterpret_cast<uint4*>(chunk_base + chunk * 16) =
              make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
        }
      }
      if (lse != nullptr && r < rows_valid) {
        lse[static_cast<int64_t>(bh) * N + q0 + r] =
            (l_run > 0.f) ? (m_run + log2f(l_run)) * kLn2 : -FLT_MAX;
      }
      fence_proxy_async_smem();
    }
    tc_fence_before();
    named_bar_sync(1, 128);
    if (threadIdx.x == 0 && ctl.abort_flag == 0) {
      for (int dc = 0; dc < C::kDChunks; ++dc) tma_store_3d(&tm_o, sQ + dc * (kBM * 128), dc * 64, q0, bh);
      bulk_commit_group();
      bulk_wait_group_read0();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
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

// [BH, N, D] row-major 16-bit tensor viewed as a 3-D map, box {64, rows, 1},
// 128-byte swizzle; rows past N read as zero and are clipped on store.
bool make_map(CUtensorMap* m, const void* ptr, int dtype, int64_t BH, int64_t N, int64_t D, int box_rows) {
  auto fn = get_encode_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(N * D * 2)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(m, dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int D, int BN, bool BF16>
int launch_impl(const AttnParams& p, const char** msg) {
  using C = Cfg<D, BN>;
  const int64_t BH = p.B * p.H;
  const int64_t N = p.N;
  const int64_t W = (N + 31) / 32;
  const int64_t KT = (N + BN - 1) / BN;
  const int64_t QT = (N + kBM - 1) / kBM;
  if (QT * BH > 0x7FFFFFFFll || BH > 0x7FFFFFFFll) {
    *msg = "attention: batch*heads too large";
    return kErrArg;
  }
  CUtensorMap mq, mk, mv, mo;
  if (!make_map(&mq, p.q, p.dtype, BH, N, D, kBM) || !make_map(&mk, p.k, p.dtype, BH, N, D, BN) ||
      !make_map(&mv, p.v, p.dtype, BH, N, D, BN) || !make_map(&mo, p.out, p.dtype, BH, N, D, kBM)) {
    *msg = "attention: cuTensorMapEncodeTiled failed (pointer alignment or driver entry point)";
    return kErrCuda;
  }
  const size_t mask_bytes = static_cast<size_t>(kBM) * W * 4;
  // At most two CTAs may share an SM: each allocates half of TMEM, and a
  // third resident CTA would block in tcgen05.alloc.  Registers already cap
  // residency at two; the shared-memory floor makes that independent of the
  // register count.
  size_t smem = C::kQBytes + C::kStages * C::kStageBytes + ((mask_bytes + 15) / 16) * 16 + sizeof(SharedCtl);
  if (smem < kMinSmemPerCta) smem = kMinSmemPerCta;
  auto kern = attn_fwd_kernel<D, BN, BF16>;
  // The dynamic shared-memory opt-in is per device; remember the largest
  // value set on each device for this instantiation.
  static size_t smem_set[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *msg = "attention: no current CUDA device";
    return kErrCuda;
  }
  if (smem > smem_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) {
      *msg = cudaGetErrorString(e);
      return kErrLaunch;
    }
    smem_set[dev] = smem;
  }
  const float scale_log2 = p.scale * kLog2e;
  cudaError_t e = launch_pdl(kern, static_cast<unsigned>(QT * BH), kThreads, smem, p.stream, mq, mk, mv, mo, p.mask,
                             p.lse, static_cast<int>(N), static_cast<int>(BH), static_cast<int>(W),
                             static_cast<int>(KT), scale_log2, p.err_word, p.timeout_ns);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    *msg = cudaGetErrorString(e);
    return kErrLaunch;
  }
  return kOk;
}

__global__ void wait_probe_kernel(uint32_t* err_word, uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ uint32_t abort_word;
  if (threadIdx.x == 0) {
    abort_word = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nothing arrives on `bar`: the bounded wait must give up and report.
    if (!mbar_wait_bounded(smem_u32(&bar), 0, &abort_word, timeout_ns)) atomicOr(err_word, kDevErrTimeout);
  }
}

}  // namespace

int launch_attn_fwd(const AttnParams& p, const char** msg) {
  if (p.N > kMaxSeqLen || (p.D == 128 && p.N > kMaxSeqLenD128)) {
    *msg = "attention: sequence length above the supported maximum (16384 for head dim 64, 8192 for 128)";
    return kErrUnsupportedN;
  }
  if (p.occ != nullptr && p.N > kMaxSeqLenOcc) {
    *msg = "attention: occupancy map given for a sequence length above 8192";
    return kErrUnsupportedN;
  }
  const bool bf = p.dtype == 1;
  if (chain_supported(p)) return launch_attn_fwd_chain(p, msg);
  if (p.D == 64) return bf ? launch_impl<64, 64, true>(p, msg) : launch_impl<64, 64, false>(p, msg);
  if (p.D == 128) return bf ? launch_impl<128, 64, true>(p, msg) : launch_impl<128, 64, false>(p, msg);
  *msg = "attention: head dim must be 64 or 128";
  return kErrUnsupportedD;
}

int launch_wait_probe(uint32_t* err_word, uint64_t timeout_ns, cudaStream_t stream) {
  wait_probe_kernel<<<1, 32, 0, stream>>>(err_word, timeout_ns);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace sma
