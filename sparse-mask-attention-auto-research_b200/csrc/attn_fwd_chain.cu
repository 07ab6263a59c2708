// Persistent two-chain fused masked-softmax attention forward, head dims 64
// and 128 (sm_100a).
//
// O = softmax_masked(scale * Q K^T) V per (batch*head, query row), the
// reference forward (csrc/sparse_attention.cu:64-143); rows with no set mask
// bit give O = 0 and lse = -FLT_MAX.
//
// One CTA per SM runs two independent "chains".  A chain is one softmax
// warpgroup plus its own loader warp and MMA warp; it walks its own list of
// work items (batch*head, 128-row query tile) and has its own Q / K / V
// buffers in shared memory and its own S, P and O in TMEM.  Nothing couples
// the two chains except the SM's pipes, so while one chain waits on a
// tensor-core result, a copy or its epilogue, the other keeps the
// exponential unit busy.
//
// Per chain and live key tile g (BN = 128 keys for D = 64, 64 keys for
// D = 128; tiles with no set bit in the item's rows are skipped before their
// K/V are loaded):
//   MMA warp:  S = Q K_g^T            (D/16 x tcgen05.mma M=128 N=BN K=16)
//   softmax:   read S, mask, row max, P = 2^(S*scale*log2e - m), write P (fp16/bf16)
//   MMA warp:  O += P V_g             (BN/16 x tcgen05.mma M=128 N=D K=16, P from TMEM)
// S and P occupy separate TMEM columns: as soon as the softmax has copied S
// into registers, the MMA warp issues Q K_{g+1}^T into the same columns, so
// the next S is ready when the current exponentials are done.
//
// Warps (384 threads):
//   0-3  softmax chain 0     4-7  softmax chain 1   (thread t of a warpgroup owns query row t)
//        besides the softmax, each warpgroup scans the packed-mask rows of
//        the item two ahead for live key tiles during its epilogue and
//        publishes the list (or, given the packer's occupancy map, reads the
//        item's two words of live-tile bits from it instead; D = 64 only)
//   8    loader chain 0      9    loader chain 1
//        TMA loads: Q, K and V (two-stage rings), K one tile ahead of V so
//        that a K copy never queues behind a V slot
//   10   MMA chain 0 (+ TMEM allocation)   11  MMA chain 1
//
// TMEM (512 columns): chain c at 256c: S [0,BN) | P [BN,3BN/2) | O [3BN/2, 3BN/2+D)
// Shared memory per chain: D = 64: Q[2] K[2] V[2] and an O staging tile,
// 16 KiB each (O leaves by TMA store); D = 128: Q (32 KiB) K[2] V[2] (16
// KiB each; O is stored from registers).  Plus the control block.
// The softmax reads its row's mask words of the next tile with one 16- or
// 8-byte global load issued a tile ahead.
// Every wait is bounded (mbar_wait_bounded) and reports through err_word.
#include <algorithm>
#include <cfloat>
#include <cstdio>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "mask_bits.cuh"
#include "sma_internal.h"
#include "sma_ptx.cuh"

namespace sma {
namespace {

constexpr int kBM = 128;
constexpr int kThreads = 384;
// Register split after start-up: the launch gives every thread 168 (384 x
// 168 = 64512); the loader and MMA warps (one warpgroup) drop to 64 and the
// two softmax warpgroups rise to 216: 128 x 64 + 256 x 216 = 63488 <= 64512.
constexpr int kRegsLaunch = 168;
constexpr int kRegsOther = 64;
constexpr int kRegsSoftmax = 216;
static_assert(128 * kRegsOther + 256 * kRegsSoftmax <= kThreads * kRegsLaunch, "register split");
constexpr int kSlots = 4;          // live-list slots per chain
constexpr int kMaxSeq = 65536;     // longest sequence the live-tile bitsets cover
constexpr int kLiveWords = kMaxSeq / 64 / 32;  // bit words per item: one bit per key tile (64 keys or more)
constexpr int kStages = 2;         // K ring and V ring depth per chain
constexpr int kTmemCols = 512;
constexpr int kChainCols = 256;
constexpr int kScanBatch = 4;      // 16-byte mask loads in flight per thread while scanning
constexpr int kSplitMinTiles = 32;  // key tiles per piece, at least, of an item split along keys
constexpr int kPackBatch = 8;      // bool input: packed words (32 mask bytes each) per batch of loads in flight
constexpr int kEpiGroups = 8;      // D = 128: mask rows of up to 8 16-byte groups (N <= 1024) scanned from registers

// Per head dim: D = 64 takes 128-key tiles, D = 128 takes 64-key tiles, so a
// K or V tile is 16 KiB either way and S + P + O of a chain fit its 256 TMEM
// columns.  Q (and O) rows are D / 64 swizzle chunks of 128 bytes.
template <int D>
struct ChainCfg {
  static_assert(D == 64 || D == 128, "head dim");
  static constexpr int kBN = D == 64 ? 128 : 64;       // keys per tile
  static constexpr int kWords = kBN / 32;              // packed-mask words of a row per tile
  static constexpr int kTilesPerGroup = 4 / kWords;    // tiles per 16-byte group of a mask row
  static constexpr int kGroupsPerWord = 32 / kTilesPerGroup;  // groups per 32-tile bit word
  static constexpr int kDChunks = D / 64;
  static constexpr int kQBytes = kBM * D * 2;          // 16 / 32 KiB
  static constexpr int kKVBytes = kBN * D * 2;         // 16 KiB
  static constexpr int kQBufs = D == 64 ? 2 : 1;
  // O leaves through a TMA store from a staging tile (D = 64) or straight
  // from registers (D = 128, which has no shared memory left for staging).
  static constexpr bool kStageO = D == 64;
  static constexpr int kChainBytes = kQBufs * kQBytes + 2 * kStages * kKVBytes + (kStageO ? kQBytes : 0);
  static constexpr int kSCol = 0;
  static constexpr int kPCol = kBN;
  static constexpr int kOCol = kBN + kBN / 2;
  static_assert(kOCol + D <= kChainCols, "TMEM budget");
  static constexpr int kMaxN = kMaxSeq;
};
constexpr float kRescaleThreshold = 8.0f;
constexpr float kLn2 = 0.69314718055994530942f;
constexpr float kLog2e = 1.44269504088896340736f;

struct ChainCtl {
  uint64_t sched_full[kSlots];
  uint64_t sched_empty[kSlots];  // 4 softmax warps + MMA warp + loader
  uint64_t q_full[2];   // per Q buffer (one or two)
  uint64_t q_empty[2];
  uint64_t k_full[kStages];
  uint64_t k_empty[kStages];
  uint64_t v_full[kStages];
  uint64_t v_empty[kStages];
  uint64_t s_full;
  uint64_t s_free;
  uint64_t p_full;
  uint64_t pv_done;
  uint64_t drain;
  // Live key tiles of the items in flight, one bit per tile: the scan ORs
  // each warp's bits into scan_bits, the publisher moves them to live_bits
  // (clearing scan_bits) once the slot's previous item has been released.
  uint32_t scan_bits[kSlots][kLiveWords];
  uint32_t live_bits[kSlots][kLiveWords];
  uint32_t n_live[kSlots];
  uint32_t split_last;  // kSplitK: this chain's unit completed its item (broadcast to the warpgroup)
};

struct Ctl {
  ChainCtl ch[2];
  uint32_t tmem_base;
  uint32_t abort_flag;
};

// Split along keys (kSplitK kernels), for workloads with fewer items than
// chains: every item is cut into `pieces` units that share its live key tiles
// evenly (by rank), run on different chains and leave their unnormalised O
// (FP32) and (max, sums) in `ws`; the unit that completes its item's count in
// `cnt` merges the item's pieces in piece order and writes O and the LSE.
struct SplitParams {
  int pieces;                // units per item (>= 2 in kSplitK kernels)
  float* ws;                 // [units][128][4] (max, l, l_out, -) then [units][128][D]
  unsigned long long* cnt;   // [items]: launch epoch << 8 | pieces finished
  unsigned long long epoch;  // distinct per launch, < 2^56, never 0
};

// Counts one finished piece of an item; a counter left by an earlier launch
// (another epoch, or whatever the memory held) counts as zero, so counters
// need no clearing.  True for the piece that completes the item.
__device__ __forceinline__ bool claim_last_piece(unsigned long long* cnt, unsigned long long epoch, int pieces) {
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(cnt);
  for (;;) {
    const unsigned long long want = ((cur >> 8) == epoch) ? cur + 1ull : ((epoch << 8) | 1ull);
    const unsigned long long prev = atomicCAS(cnt, cur, want);
    if (prev == cur) return static_cast<int>(want & 0xFFull) == pieces;
    cur = prev;
  }
}

template <int D>
constexpr size_t smem_bytes() {
  return 2 * static_cast<size_t>(ChainCfg<D>::kChainBytes) + sizeof(Ctl);
}
static_assert(smem_bytes<64>() <= 227 * 1024 && smem_bytes<128>() <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed FP32 pairs (sm_100a f32x2 instructions): one issue slot for two lanes' worth of FMA / add.
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
  int bh, q0, rows_valid;
};

// Item w.  Query tiles run in decreasing index order: under a causal mask
// the last query tiles see the most keys.
//   head_major == 0: batch*head fastest, so all chains of a round work on the
//     same query tile index and causal rounds are even.  Used when K and V of
//     all heads fit in L2 together.
//   head_major != 0: the query tiles of one batch*head are consecutive, so the
//     chains working on them at the same time share that head's K and V in
//     L2 (the serpentine walk still pairs a chain's heavy tiles with light
//     ones).  Used when K and V would not stay in L2 between rounds.
__device__ __forceinline__ Item item_of(int w, int BH, int QT, int N, int head_major) {
  Item it;
  const int fast_n = head_major ? QT : BH;  // one division for either order
  const int slow = w / fast_n, fast = w - slow * fast_n;
  const int qt = QT - 1 - (head_major ? fast : slow);
  it.bh = head_major ? slow : fast;
  it.q0 = qt * kBM;
  it.rows_valid = min(kBM, N - it.q0);
  return it;
}

// Bits of word `cw` of a packed-mask row that address columns < N.
__device__ __forceinline__ uint32_t valid_bits(int cw, int N) {
  const int valid = N - cw * 32;
  return valid >= 32 ? 0xFFFFFFFFu : (valid <= 0 ? 0u : ((1u << valid) - 1u));
}

// The mask words of key tile kt (kWords of them) for one query row, columns
// >= N cleared.
// kOwn: the words were written earlier in this kernel by the same thread
// (bool-mask input), so they are read with plain loads, not the read-only path.
template <int D, bool kOwn>
__device__ __forceinline__ void load_tile_words(const uint32_t* mrow, int kt, int W, int N, bool vec,
                                                uint32_t (&mw)[ChainCfg<D>::kWords]) {
  using C = ChainCfg<D>;
  const int w0 = kt * C::kWords;
  if (vec) {
    if constexpr (C::kWords == 4) {
      const uint4 v = kOwn ? ld_global_v4(mrow + w0) : __ldg(reinterpret_cast<const uint4*>(mrow + w0));
      mw[0] = v.x;
      mw[1] = v.y;
      mw[2] = v.z;
      mw[3] = v.w;
    } else {
      const uint2 v = kOwn ? ld_global_v2(mrow + w0) : __ldg(reinterpret_cast<const uint2*>(mrow + w0));
      mw[0] = v.x;
      mw[1] = v.y;
    }
  } else {
#pragma unroll
    for (int w = 0; w < C::kWords; ++w)
      mw[w] = (w0 + w < W) ? (kOwn ? ld_global_u32(mrow + w0 + w) : __ldg(mrow + w0 + w)) : 0u;
  }
  if (N - kt * C::kBN < C::kBN) {
#pragma unroll
    for (int w = 0; w < C::kWords; ++w) mw[w] &= valid_bits(w0 + w, N);
  }
}

// Eight 32-bit words r[o .. o+7] to a 32-byte aligned global address.
__device__ __forceinline__ void st_global_v8(void* dst, const uint32_t (&r)[16], int o) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(dst), "r"(r[o]), "r"(r[o + 1]),
               "r"(r[o + 2]), "r"(r[o + 3]), "r"(r[o + 4]), "r"(r[o + 5]), "r"(r[o + 6]), "r"(r[o + 7])
               : "memory");
}

// Live bits, relative to tile 32k, of the key tiles in 16-byte group g of a
// mask row (words 4g .. 4g+3: one 128-key tile, or two 64-key tiles),
// columns >= N cleared.
template <int D>
__device__ __forceinline__ uint32_t group_live(const uint4& v, int g, int k, int N) {
  const uint32_t x0 = v.x & valid_bits(g * 4, N), x1 = v.y & valid_bits(g * 4 + 1, N);
  const uint32_t x2 = v.z & valid_bits(g * 4 + 2, N), x3 = v.w & valid_bits(g * 4 + 3, N);
  if constexpr (ChainCfg<D>::kWords == 4) {
    return ((x0 | x1 | x2 | x3) != 0u ? 1u : 0u) << (g - 32 * k);
  } else {
    const int t = 2 * g - 32 * k;
    return (((x0 | x1) != 0u ? 1u : 0u) << t) | (((x2 | x3) != 0u ? 1u : 0u) << (t + 1));
  }
}

// The unit that completed a split item merges the item's pieces p0 ..
// p0+pieces-1 for its row r, in piece order: weights 2^(m_p - M) against the
// row's overall max M, O = sum w_p O_p / sum w_p l_out_p, LSE from
// sum w_p l_p (M = -inf: an empty row, O = 0 and LSE = -FLT_MAX).
template <int D, bool BF16>
__device__ __noinline__ void merge_pieces(const SplitParams sp, int64_t n_units, int64_t p0, int r, uint16_t* orow,
                                          float* lse_r, bool write_o) {
  const float* ml_base = sp.ws;                    // [unit][row][4]
  const float* po_base = sp.ws + n_units * kBM * 4;  // [unit][row][D]
  float M = -INFINITY;
  for (int pc = 0; pc < sp.pieces; ++pc) M = fmaxf(M, __ldcg(ml_base + ((p0 + pc) * kBM + r) * 4));
  float lr = 0.f, lo = 0.f;
  for (int pc = 0; pc < sp.pieces; ++pc) {
    const float4 v = __ldcg(reinterpret_cast<const float4*>(ml_base + ((p0 + pc) * kBM + r) * 4));
    const float w = (v.x == -INFINITY) ? 0.f : ex2f(v.x - M);
    lr += w * v.y;
    lo += w * v.z;
  }
  const float inv = (lo > 0.f) ? (1.f / lo) : 0.f;
#pragma unroll 1
  for (int dc = 0; dc < D / 32; ++dc) {
    float acc[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) acc[q] = 0.f;
    for (int pc = 0; pc < sp.pieces; ++pc) {
      const float mp = __ldcg(ml_base + ((p0 + pc) * kBM + r) * 4);
      const float w = (mp == -INFINITY) ? 0.f : ex2f(mp - M);
      const float4* src = reinterpret_cast<const float4*>(po_base + ((p0 + pc) * kBM + r) * D + dc * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 o = __ldcg(src + q);
        acc[4 * q] += w * o.x;
        acc[4 * q + 1] += w * o.y;
        acc[4 * q + 2] += w * o.z;
        acc[4 * q + 3] += w * o.w;
      }
    }
    uint32_t hw[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) hw[q] = pack2<BF16>(acc[2 * q] * inv, acc[2 * q + 1] * inv);
    if (write_o) {
      uint4* dst = reinterpret_cast<uint4*>(orow + dc * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q) dst[q] = make_uint4(hw[4 * q], hw[4 * q + 1], hw[4 * q + 2], hw[4 * q + 3]);
    }
  }
  if (lse_r != nullptr) *lse_r = (lr > 0.f) ? (M + log2f(lr)) * kLn2 : -FLT_MAX;
}

// Position of one chain in the flattened sequence of its live tiles.
struct Cursor {
  int i;       // item index (-1 before the first item, n_items when exhausted)
  uint32_t t;  // live tile within the item
  uint32_t n;  // live tiles of item i
  int w;       // bit word of the current tile
  uint32_t x;  // live bits of word w above the current tile
  int kt;      // current key tile
};

// Steps (w, x) to the next set bit of a slot's live bitset and returns its
// tile index.  The caller knows such a bit exists (it counts tiles against
// n_live).
__device__ __forceinline__ int next_live(const uint32_t* bits, int& w, uint32_t& x) {
  while (x == 0u) x = bits[++w];
  const int b = __ffs(x) - 1;
  x &= x - 1u;
  return w * 32 + b;
}

// kBoolIn: the mask arrives as bool bytes (`bmask`, [BH, N, N]) instead of
// packed words; the softmax warps pack each item's rows into `pk` while they
// scan them (pk then holds exactly what the mask packer writes) and the tile
// loop reads its words back from there.  `mask` is unused then.
template <int D, bool BF16, bool kBoolIn, bool kSplitK>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_chain_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                          uint16_t* __restrict__ out, const uint32_t* __restrict__ mask,
                          const uint8_t* __restrict__ bmask, uint32_t* pk,
                          const uint32_t* __restrict__ occ, float* __restrict__ lse, int N, int BH, int W,
                          int KT, int total_items, int vec, int o_wide, int head_major, int pf_early,
                          float scale_log2, const SplitParams sp, uint32_t* err_word,
                          uint64_t timeout_ns) {
  using C = ChainCfg<D>;
  constexpr int kBN = C::kBN;
  constexpr int kWords = C::kWords;
  constexpr int kGroupsPerWord = C::kGroupsPerWord;
  constexpr int kSCol = C::kSCol, kPCol = C::kPCol, kOCol = C::kOCol;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t base = smem_u32(smem);
  if ((base & 1023u) != 0u) {
    if (threadIdx.x == 0) atomicOr(err_word, kDevErrLayout);
    return;
  }
  Ctl& ctl = *reinterpret_cast<Ctl*>(smem + 2 * C::kChainBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int QT = (N + kBM - 1) / kBM;
  const int G = gridDim.x;
  volatile uint32_t* abort_flag = &ctl.abort_flag;

  // The 2G chains (chain c of CTA b is k = c*G + b) take the items round by
  // round, serpentine: in round i chain k takes item 2G*i + k (i even) or
  // 2G*i + 2G-1-k (i odd), which evens out per-SM work when item sizes fall
  // with the item index (causal masks).
  auto chain_item = [&](int c, int i) {
    const int k = c * G + static_cast<int>(blockIdx.x);
    return 2 * G * i + ((i & 1) ? 2 * G - 1 - k : k);
  };
  auto chain_items = [&](int c) {
    const int k = c * G + static_cast<int>(blockIdx.x);
    const int full = total_items / (2 * G), rem = total_items % (2 * G);
    const int off = (full & 1) ? 2 * G - 1 - k : k;
    return full + (off < rem ? 1 : 0);
  };
  // The item of chain c's unit i (kSplitK: units are pieces of items) and
  // the piece it is (-1: a whole item).
  auto item_at = [&](int c, int i) {
    const int w = chain_item(c, i);
    return item_of(kSplitK ? w / sp.pieces : w, BH, QT, N, head_major);
  };
  auto piece_at = [&](int c, int i) { return kSplitK ? chain_item(c, i) % sp.pieces : -1; };

  if (threadIdx.x == 256) {
    for (int c = 0; c < 2; ++c) {
      ChainCtl& cc = ctl.ch[c];
      for (int s = 0; s < kSlots; ++s) {
        mbar_init(smem_u32(&cc.sched_full[s]), 1);
        mbar_init(smem_u32(&cc.sched_empty[s]), 6);
      }
      for (int b = 0; b < 2; ++b) {
        mbar_init(smem_u32(&cc.q_full[b]), 1);
        mbar_init(smem_u32(&cc.q_empty[b]), 1);
      }
      for (int s = 0; s < kStages; ++s) {
        mbar_init(smem_u32(&cc.k_full[s]), 1);
        mbar_init(smem_u32(&cc.k_empty[s]), 1);
        mbar_init(smem_u32(&cc.v_full[s]), 1);
        mbar_init(smem_u32(&cc.v_empty[s]), 1);
      }
      mbar_init(smem_u32(&cc.s_full), 1);
      mbar_init(smem_u32(&cc.s_free), 4);
      mbar_init(smem_u32(&cc.p_full), 4);
      mbar_init(smem_u32(&cc.pv_done), 1);
      mbar_init(smem_u32(&cc.drain), 1);
    }
    for (int c = 0; c < 2; ++c)
      for (int sl = 0; sl < kSlots; ++sl)
        for (int k = 0; k < kLiveWords; ++k) ctl.ch[c].scan_bits[sl][k] = 0u;
    ctl.abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 10) {
    tmem_alloc(smem_u32(&ctl.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl.tmem_base;
  // Set-up above overlaps the previous kernel (the mask packer); its outputs
  // and everything else earlier in the stream are read only after this.
  pdl_wait_prior_grid();

  auto fail = [&]() {
    ctl.abort_flag = 1;
    atomicOr(err_word, kDevErrTimeout);
  };

  // Moves a cursor to the next live tile (one thread): 1 = found, 0 = no
  // tiles left, -1 = a wait gave up.  With `release`, the cursor arrives on
  // sched_empty of every item it leaves.
  auto advance = [&](ChainCtl& cc, Cursor& cu, int n_items, bool release) -> int {
    if (cu.i >= 0 && cu.i < n_items && cu.t + 1 < cu.n) {
      ++cu.t;
      cu.kt = next_live(cc.live_bits[cu.i % kSlots], cu.w, cu.x);
      return 1;
    }
    if (release && cu.i >= 0 && cu.i < n_items) mbar_arrive(smem_u32(&cc.sched_empty[cu.i % kSlots]));
    for (int i = cu.i + 1; i < n_items; ++i) {
      const int slot = i % kSlots;
      if (!mbar_wait_bounded(smem_u32(&cc.sched_full[slot]), (i / kSlots) & 1, abort_flag, timeout_ns)) return -1;
      const uint32_t n = cc.n_live[slot];
      if (n == 0) {
        if (release) mbar_arrive(smem_u32(&cc.sched_empty[slot]));
        continue;
      }
      cu.i = i;
      cu.t = 0;
      cu.n = n;
      cu.w = 0;
      cu.x = cc.live_bits[slot][0];
      cu.kt = next_live(cc.live_bits[slot], cu.w, cu.x);
      return 1;
    }
    cu.i = n_items;
    return 0;
  };

  // The loader and the MMA warp look one live tile ahead: the next K copy
  // and QK^T go before this tile's V copy and PV.  Past an item with no live
  // tile, though, the next live tile lies in an item whose list the softmax
  // publishes only after this tile's PV, so waiting for it first would
  // deadlock.  look_ahead() decides, without changing the cursor: 1 = the
  // next live tile needs no list that is not out (same item, or the next
  // item's list is published with a live tile, or no items left); -1 = the
  // next item's list is out and has no live tile (finish this tile first);
  // 0 = not known yet.  Callers poll it together with the readiness of
  // their own next step and take whichever comes first.
  auto look_ahead = [&](ChainCtl& cc, const Cursor& cu, int n_items) -> int {
    if (cu.i >= 0 && cu.i < n_items && cu.t + 1 < cu.n) return 1;
    const int j = cu.i + 1;
    if (j >= n_items) return 1;
    const int slot = j % kSlots;
    if (!mbar_test_wait(smem_u32(&cc.sched_full[slot]), (j / kSlots) & 1)) return 0;
    return cc.n_live[slot] != 0u ? 1 : -1;
  };
  // Polls look_ahead() and `own_ready` (the caller's own next step can go
  // without waiting) until one decides: true = look ahead first, false =
  // finish this tile first.  Bounded like every wait; `ok` turns false when
  // it gives up.
  auto decide_ahead = [&](ChainCtl& cc, const Cursor& cu, int n_items, auto own_ready, bool& ok) -> bool {
    const int a0 = look_ahead(cc, cu, n_items);  // the common case decides at once
    if (a0 != 0) return a0 > 0;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
      const int a = look_ahead(cc, cu, n_items);
      if (a != 0) return a > 0;
      if (own_ready()) return false;
      if (*abort_flag != 0u || global_timer_ns() - t0 > timeout_ns) {
        ok = false;
        return false;
      }
      __nanosleep(32);
    }
  };

  if (warp == 8 || warp == 9) {
    // ================================================================ loader
    regs_dec<kRegsOther>();
    const int c = warp - 8;
    ChainCtl& cc = ctl.ch[c];
    if (lane == 0) {
      const uint32_t sQ = base + c * C::kChainBytes;
      const uint32_t sK = sQ + C::kQBufs * C::kQBytes;
      const uint32_t sV = sK + kStages * C::kKVBytes;
      const int n_items = chain_items(c);
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      if constexpr (C::kStageO) tma_prefetch_desc(&tm_o);
      Cursor kc{-1, 0u, 0u, 0, 0u, 0}, vc{-1, 0u, 0u, 0, 0u, 0};
      uint32_t gk = 0, gv = 0, q_count = 0;  // K, V and Q copies issued
      bool ok = true;
      auto issue_k = [&]() -> bool {
        const Item it = item_at(c, kc.i);
        if (kc.t == 0) {
          // First tile of an item: its Q, into the buffer the item kQBufs back used.
          const int qb = q_count % C::kQBufs;
          if (q_count >= static_cast<uint32_t>(C::kQBufs) &&
              !mbar_wait_bounded(smem_u32(&cc.q_empty[qb]), ((q_count / C::kQBufs) - 1) & 1, abort_flag,
                                 timeout_ns))
            return false;
          mbar_arrive_expect_tx(smem_u32(&cc.q_full[qb]), C::kQBytes);
#pragma unroll
          for (int dc = 0; dc < C::kDChunks; ++dc)
            tma_load_3d(sQ + qb * C::kQBytes + dc * (kBM * 128), &tm_q, smem_u32(&cc.q_full[qb]), dc * 64, it.q0,
                        it.bh);
          ++q_count;
        }
        const int stage = gk % kStages;
        if (gk >= static_cast<uint32_t>(kStages) &&
            !mbar_wait_bounded(smem_u32(&cc.k_empty[stage]), ((gk / kStages) - 1) & 1, abort_flag, timeout_ns))
          return false;
        const int kt = kc.kt;
        mbar_arrive_expect_tx(smem_u32(&cc.k_full[stage]), C::kKVBytes);
#pragma unroll
        for (int dc = 0; dc < C::kDChunks; ++dc)
          tma_load_3d(sK + stage * C::kKVBytes + dc * (kBN * 128), &tm_k, smem_u32(&cc.k_full[stage]), dc * 64,
                      kt * kBN, it.bh);
        ++gk;
        return true;
      };
      auto issue_v = [&]() -> bool {
        const Item it = item_at(c, vc.i);
        const int stage = gv % kStages;
        if (gv >= static_cast<uint32_t>(kStages) &&
            !mbar_wait_bounded(smem_u32(&cc.v_empty[stage]), ((gv / kStages) - 1) & 1, abort_flag, timeout_ns))
          return false;
        const int kt = vc.kt;
        mbar_arrive_expect_tx(smem_u32(&cc.v_full[stage]), C::kKVBytes);
#pragma unroll
        for (int dc = 0; dc < C::kDChunks; ++dc)
          tma_load_3d(sV + stage * C::kKVBytes + dc * (kBN * 128), &tm_v, smem_u32(&cc.v_full[stage]), dc * 64,
                      kt * kBN, it.bh);
        ++gv;
        return true;
      };
      // The K cursor walks the live tiles and releases every item it leaves
      // (so no list slot is reused before it has passed); the V copy of a
      // tile uses the K cursor's position saved when that tile's K was issued.
      int rk = advance(cc, kc, n_items, true);
      if (rk < 0 || (rk == 1 && !issue_k())) ok = false;
      while (ok && rk == 1) {
        vc = kc;  // tile g: its K is out, its V is next
        // K of the next live tile before this V, unless that waits on the softmax.
        const bool k_first = decide_ahead(cc, kc, n_items, [&]() {
          return gv < static_cast<uint32_t>(kStages) ||
                 mbar_test_wait(smem_u32(&cc.v_empty[gv % kStages]), ((gv / kStages) - 1) & 1);
        }, ok);
        if (!ok) break;
        if (k_first) {
          rk = advance(cc, kc, n_items, true);
          if (rk < 0 || (rk == 1 && !issue_k())) {
            ok = false;
            break;
          }
        }
        if (!issue_v()) {
          ok = false;
          break;
        }
        if (!k_first) {
          rk = advance(cc, kc, n_items, true);
          if (rk < 0 || (rk == 1 && !issue_k())) {
            ok = false;
            break;
          }
        }
      }
      if (rk < 0) ok = false;
      if (!ok) {
        fail();
        // Let the copies this thread started land before the CTA exits.
        uint32_t zero = 0;
        for (uint32_t x = (gk > static_cast<uint32_t>(kStages) ? gk - kStages : 0u); x < gk; ++x)
          mbar_wait_bounded(smem_u32(&cc.k_full[x % kStages]), (x / kStages) & 1, &zero, timeout_ns);
        for (uint32_t x = (gv > static_cast<uint32_t>(kStages) ? gv - kStages : 0u); x < gv; ++x)
          mbar_wait_bounded(smem_u32(&cc.v_full[x % kStages]), (x / kStages) & 1, &zero, timeout_ns);
        for (uint32_t q = (q_count > static_cast<uint32_t>(C::kQBufs) ? q_count - C::kQBufs : 0u); q < q_count; ++q)
          mbar_wait_bounded(smem_u32(&cc.q_full[q % C::kQBufs]), (q / C::kQBufs) & 1, &zero, timeout_ns);
      }
    }
  } else if (warp == 10 || warp == 11) {
    // ================================================================ MMA issuer
    regs_dec<kRegsOther>();
    const int c = warp - 10;
    ChainCtl& cc = ctl.ch[c];
    if (lane == 0) {
      const uint32_t sQ = base + c * C::kChainBytes;
      const uint32_t sK = sQ + C::kQBufs * C::kQBytes;
      const uint32_t sV = sK + kStages * C::kKVBytes;
      const uint32_t tS = tmem + c * kChainCols + kSCol;
      const uint32_t tP = tmem + c * kChainCols + kPCol;
      const uint32_t tO = tmem + c * kChainCols + kOCol;
      constexpr uint32_t idesc_qk = make_idesc_f16(kBM, kBN, BF16 ? 1 : 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBM, D, BF16 ? 1 : 0, 1);
      const int n_items = chain_items(c);
      bool ok = true;

      Cursor qc{-1, 0u, 0u, 0, 0u, 0};  // next tile to multiply by K^T
      uint32_t q_count = 0;
      int qqb = 0;            // Q buffer of the cursor's item
      auto advance_qk = [&]() -> int {
        const int res = advance(cc, qc, n_items, true);
        if (res == 1 && qc.t == 0) {
          qqb = q_count % C::kQBufs;
          if (!mbar_wait_bounded(smem_u32(&cc.q_full[qqb]), (q_count / C::kQBufs) & 1, abort_flag, timeout_ns))
            return -1;
          ++q_count;
        }
        return res;
      };
      bool first_of[2] = {false, false};  // tile g is the first of its item (O overwritten)
      auto issue_qk = [&](uint32_t g) -> bool {
        const int stage = g % kStages;
        if (!mbar_wait_bounded(smem_u32(&cc.k_full[stage]), (g / kStages) & 1, abort_flag, timeout_ns))
          return false;
        // S is free once the softmax has copied S of tile g-1 into registers.
        if (g > 0 && !mbar_wait_bounded(smem_u32(&cc.s_free), (g - 1) & 1, abort_flag, timeout_ns)) return false;
        tc_fence_after();
        const uint32_t sQb = sQ + qqb * C::kQBytes;
        const uint32_t sKb = sK + stage * C::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          // 16 head dims: swizzle chunk kk / 4 of the rows, 32 bytes into it.
          const uint32_t qoff = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
          mma_ss(tS, smem_desc_sw128(sQb + qoff, 16, 1024), smem_desc_sw128(sKb + koff, 16, 1024), idesc_qk,
                 kk > 0 ? 1u : 0u);
        }
        mma_commit(smem_u32(&cc.s_full));
        mma_commit(smem_u32(&cc.k_empty[stage]));
        if (qc.t + 1 == qc.n) mma_commit(smem_u32(&cc.q_empty[qqb]));  // last QK^T of the item
        first_of[g & 1] = (qc.t == 0);
        return true;
      };

      uint32_t n_qk = 0;
      int res = advance_qk();
      if (res < 0 || (res == 1 && !issue_qk(0))) ok = false;
      if (ok && res == 1) n_qk = 1;
      // QK^T of the next live tile; returns false if a wait gave up.
      auto qk_ahead = [&](uint32_t g) -> bool {
        res = advance_qk();
        if (res < 0 || (res == 1 && !issue_qk(g + 1))) return false;
        if (res == 1) ++n_qk;
        return true;
      };
      for (uint32_t g = 0; ok && g < n_qk; ++g) {
        // The next QK^T before this PV, unless that waits on the softmax.
        const bool qk_first = decide_ahead(cc, qc, n_items, [&]() {
          return mbar_test_wait(smem_u32(&cc.p_full), g & 1);
        }, ok);
        if (!ok) break;
        if (qk_first && !qk_ahead(g)) {
          ok = false;
          break;
        }
        const int stage = g % kStages;
        if (!mbar_wait_bounded(smem_u32(&cc.p_full), g & 1, abort_flag, timeout_ns) ||
            !mbar_wait_bounded(smem_u32(&cc.v_full[stage]), (g / kStages) & 1, abort_flag, timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sVb = sV + stage * C::kKVBytes;
        const bool fresh = first_of[g & 1];
        // V is MN-major: 16 keys are 2048 bytes into each 64-dim chunk; the
        // chunks (D = 128) are kBN * 128 bytes apart.
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          mma_ts(tO, tP + kk * 8, smem_desc_sw128(sVb + kk * 2048, kBN * 128, 1024), idesc_pv,
                 (fresh && kk == 0) ? 0u : 1u);
        mma_commit(smem_u32(&cc.pv_done));
        mma_commit(smem_u32(&cc.v_empty[stage]));
        if (!qk_first && !qk_ahead(g)) {
          ok = false;
          break;
        }
      }
      if (!ok) fail();
      // Every MMA this thread issued must complete before TMEM is released.
      mma_commit(smem_u32(&cc.drain));
      uint32_t zero = 0;
      mbar_wait_bounded(smem_u32(&cc.drain), 0, &zero, timeout_ns);
    }
  } else {
    // ================================================================ softmax
    regs_inc<kRegsSoftmax>();
    const int c = warp >> 2;
    const int wq = warp & 3;
    ChainCtl& cc = ctl.ch[c];
    const int r = threadIdx.x & 127;  // query row == TMEM lane
    const uint32_t t_lane = tmem + c * kChainCols + (static_cast<uint32_t>(wq * 32) << 16);
    // O staging tile (D = 64 only): after Q, K and V of the chain.
    constexpr int kStageOff = C::kQBufs * C::kQBytes + 2 * kStages * C::kKVBytes;
    const uint32_t sO = base + c * C::kChainBytes + kStageOff;
    uint8_t* out_row = smem + c * C::kChainBytes + kStageOff + r * 128;
    const int n_items = chain_items(c);
    const int bar_id = 1 + c;
    const int G4 = W >> 2;  // 16-byte groups per mask row (vec path)
    bool ok = true;
    uint32_t g = 0;  // tiles processed by this chain

    auto wait_all = [&](uint64_t& bar, uint32_t parity) -> bool {
      const bool all =
          __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&bar), parity, abort_flag, timeout_ns));
      if (all) tc_fence_after();
      return all;
    };
    auto arrive_warp = [&](uint64_t& bar) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar));
    };
    // Packed words of the tile loop: the caller's, or (bool input) this
    // kernel's own, written by the scan of the item.
    const uint32_t* words = kBoolIn ? pk : mask;
    auto row_ptr = [&](const Item& it) {
      return words + (static_cast<int64_t>(it.bh) * N + it.q0 + r) * W;
    };
    // Mask words of key tile kt for this thread's row of `it` (0 for padding rows).
    auto fetch_words = [&](const Item& it, int kt, uint32_t (&mw)[kWords]) {
      if (r < it.rows_valid) {
        load_tile_words<D, kBoolIn>(row_ptr(it), kt, W, N, vec != 0, mw);
      } else {
#pragma unroll
        for (int w = 0; w < kWords; ++w) mw[w] = 0u;
      }
    };
    // This thread's packed-mask row of `it` into L1 (a prefetch holds no registers).
    auto prefetch_rows_l1 = [&](const Item& it) {
      if (r >= it.rows_valid) return;
      const uintptr_t a0 = reinterpret_cast<uintptr_t>(row_ptr(it));
      const uintptr_t a1 = a0 + static_cast<uintptr_t>(W) * 4u;
      for (uintptr_t a = a0 & ~static_cast<uintptr_t>(127); a < a1; a += 128)
        asm volatile("prefetch.global.L1 [%0];" ::"l"(a));
    };
    // ORs this thread's packed-mask row of `it` into live-tile words (bit t of
    // word k = key tile 32k + t) and adds each warp's words to item j's
    // scan_bits; the WG barrier after it completes them for the publisher.
    auto scan_post = [&](const Item& it, int j) {
      const uint32_t* mrow = row_ptr(it);
      const bool row_ok = r < it.rows_valid;
      const int nw = (KT + 31) >> 5;
      for (int k = 0; k < nw; ++k) {
        uint32_t bits = 0u;
        if (row_ok) {
          if (vec) {
            const int g_lo = k * kGroupsPerWord;
            const int g_hi = min(G4, g_lo + kGroupsPerWord);
            for (int gb = g_lo; gb < g_hi; gb += kScanBatch) {
              uint4 v[kScanBatch];
#pragma unroll
              for (int u = 0; u < kScanBatch; ++u)
                v[u] = (gb + u < g_hi) ? __ldg(reinterpret_cast<const uint4*>(mrow) + gb + u)
                                       : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
              for (int u = 0; u < kScanBatch; ++u)
                if (gb + u < g_hi) bits |= group_live<D>(v[u], gb + u, k, N);
            }
          } else {
            const int w_lo = k * 32 * kWords;
            const int w_hi = min(W, w_lo + 32 * kWords);
            for (int cw = w_lo; cw < w_hi; ++cw)
              if ((__ldg(mrow + cw) & valid_bits(cw, N)) != 0u) bits |= 1u << (cw / kWords - 32 * k);
          }
        }
        const uint32_t x = __reduce_or_sync(0xffffffffu, bits);
        if (lane == 0 && x != 0u) atomicOr(&cc.scan_bits[j % kSlots][k], x);
      }
    };
    // Bool input: this thread's bool row of `it` into L2 (N bytes, a hint:
    // no registers, nothing to wait for).
    auto prefetch_bool_row = [&](const Item& it) {
      if (r < it.rows_valid)
        bulk_prefetch_l2(bmask + (static_cast<int64_t>(it.bh) * N + it.q0 + r) * N, static_cast<uint32_t>(N));
    };
    // Bool input: packs this thread's bool row of `it` into its packed row
    // (32 bytes -> one word, N % 32 == 0) and ORs live-tile bits into item
    // j's scan_bits like scan_post.  Rows of 0/1 bytes (what torch writes
    // for bool) take the multiply packing; a batch holding any other byte
    // value is packed with the exact any-non-zero rule instead.
    auto scan_pack = [&](const Item& it, int j) {
      const bool row_ok = r < it.rows_valid;
      const int64_t row = static_cast<int64_t>(it.bh) * N + it.q0 + r;
      const uint4* brow = reinterpret_cast<const uint4*>(bmask + row * N);
      uint32_t* prow = pk + row * W;
      const int nw = (KT + 31) >> 5;
      for (int k = 0; k < nw; ++k) {
        uint32_t bits = 0u;
        if (row_ok) {
          const int w_lo = k * 32 * kWords;  // a multiple of 64 words
          const int w_hi = min(W, w_lo + 32 * kWords);
          for (int wb = w_lo; wb < w_hi; wb += kPackBatch) {
            uint4 v[2 * kPackBatch];
#pragma unroll
            for (int u = 0; u < kPackBatch; ++u) {
              const bool in = wb + u < w_hi;
              v[2 * u] = in ? __ldcs(brow + 2 * (wb + u)) : make_uint4(0u, 0u, 0u, 0u);
              v[2 * u + 1] = in ? __ldcs(brow + 2 * (wb + u) + 1) : make_uint4(0u, 0u, 0u, 0u);
            }
            bool all01 = true;
#pragma unroll
            for (int u = 0; u < kPackBatch; ++u) all01 = all01 && bytes_are_01(v[2 * u], v[2 * u + 1]);
            uint32_t wd[kPackBatch];
            if (all01) {
#pragma unroll
              for (int u = 0; u < kPackBatch; ++u) wd[u] = pack32_01(v[2 * u], v[2 * u + 1]);
            } else {
#pragma unroll
              for (int u = 0; u < kPackBatch; ++u) wd[u] = pack32_any(v[2 * u], v[2 * u + 1]);
            }
            if (vec && wb + kPackBatch <= w_hi) {
#pragma unroll
              for (int u = 0; u < kPackBatch; u += 4)
                *reinterpret_cast<uint4*>(prow + wb + u) = make_uint4(wd[u], wd[u + 1], wd[u + 2], wd[u + 3]);
            } else {
#pragma unroll
              for (int u = 0; u < kPackBatch; ++u)
                if (wb + u < w_hi) prow[wb + u] = wd[u];
            }
#pragma unroll
            for (int u = 0; u < kPackBatch; ++u)
              if (wd[u] != 0u) bits |= 1u << ((wb + u) / kWords - 32 * k);
          }
        }
        const uint32_t x = __reduce_or_sync(0xffffffffu, bits);
        if (lane == 0 && x != 0u) atomicOr(&cc.scan_bits[j % kSlots][k], x);
      }
    };
    auto scan_item = [&](const Item& it, int j) {
      if constexpr (kBoolIn) {
        scan_pack(it, j);
      } else {
        scan_post(it, j);
      }
    };
    // Warp 0 of the WG, after a WG barrier: moves item j's scanned bits (lane
    // k: word k) into its slot's live bits, counts them and publishes them.
    auto publish = [&](int j) {
      const int slot = j % kSlots;
      if (j >= kSlots && !wait_all(cc.sched_empty[slot], ((j / kSlots) - 1) & 1)) {
        if (lane == 0) fail();
        return;
      }
      // Live key tiles straight from the packer's occupancy map when there is
      // one (two words per item: the map is only made for N <= 8192).
      const uint32_t* occ_j = nullptr;
      if (occ != nullptr) {
        const Item itj = item_at(c, j);
        occ_j = occ + 2 * (static_cast<int64_t>(itj.bh) * QT + itj.q0 / kBM);
      }
      const int nw = (KT + 31) >> 5;  // <= 32: one word per lane
      uint32_t x = 0u;
      if (lane < nw) {
        if (occ_j != nullptr) {
          x = lane < 2 ? occ_j[lane] : 0u;
        } else {
          x = cc.scan_bits[slot][lane];
          cc.scan_bits[slot][lane] = 0u;  // ready for the item four later
        }
        if (KT - lane * 32 < 32) x &= (1u << (KT - lane * 32)) - 1u;
      }
      if constexpr (kSplitK) {
        // This unit's share of the item's L live tiles: those of rank
        // [pj * L / pieces, (pj + 1) * L / pieces) in key order.
        const int pj = piece_at(c, j);
        const uint32_t cnt = static_cast<uint32_t>(__popc(x));
        uint32_t incl = cnt;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const uint32_t t = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += t;
        }
        const int live = static_cast<int>(__shfl_sync(0xffffffffu, incl, 31));
        const int pre = static_cast<int>(incl - cnt);
        const int a = max(pj * live / sp.pieces - pre, 0);
        const int b = min((pj + 1) * live / sp.pieces - pre, static_cast<int>(cnt));
        uint32_t keep = 0u;
        if (b > a) {
          keep = x;
          for (int t = 0; t < a; ++t) keep &= keep - 1u;  // drop the a lowest
          uint32_t above = keep;
          for (int t = 0; t < b - a; ++t) above &= above - 1u;
          keep &= ~above;  // the next b - a
        }
        x = keep;
      }
      if (lane < nw) cc.live_bits[slot][lane] = x;
      const uint32_t n = __reduce_add_sync(0xffffffffu, static_cast<uint32_t>(__popc(x)));
      __syncwarp();
      if (lane == 0) {
        cc.n_live[slot] = n;
        mbar_arrive(smem_u32(&cc.sched_full[slot]));
      }
    };

    // Prologue: the live lists of the first two items.  The second item's
    // mask rows are prefetched into L1 first, so both rows are fetched from
    // HBM at once, and the first list is published before the second is built.
    const int n_pre = n_items < 2 ? n_items : 2;
    if constexpr (kBoolIn) {
      for (int j = 0; j < n_pre; ++j) prefetch_bool_row(item_at(c, j));
    } else {
      if (n_pre > 1 && occ == nullptr) prefetch_rows_l1(item_at(c, 1));
    }
    for (int j = 0; j < n_pre; ++j) {
      if (occ == nullptr) scan_item(item_at(c, j), j);
      named_bar_sync(bar_id, 128);
      if (wq == 0) publish(j);
    }

    uint32_t mw[kWords] = {};
    bool have_mw = false;  // mw already holds tile 0 of the current item
    for (int i = 0; i < n_items; ++i) {
      const int slot = i % kSlots;
      const Item it = item_at(c, i);
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&cc.sched_full[slot]), (i / kSlots) & 1,
                                                              abort_flag, timeout_ns));
      const uint32_t n = ok ? cc.n_live[slot] : 0u;
      // Bool input: item i+2's rows head for L2 an item before their scan
      // (at the item's last tile instead when the rows of a round of items
      // would not fit in L2 together).
      if constexpr (kBoolIn) {
        if (pf_early && i + 2 < n_items) prefetch_bool_row(item_at(c, i + 2));
      }
      // Walk over the item's live bits (word lw, bits above the current tile lx).
      int lw = 0;
      uint32_t lx = cc.live_bits[slot][0];
      const int kt0 = n > 0 ? next_live(cc.live_bits[slot], lw, lx) : 0;
      if (n > 0 && !have_mw) fetch_words(it, kt0, mw);
      have_mw = false;
      float m_run = -INFINITY, l_run = 0.f, l_out = 0.f;

      for (uint32_t t = 0; ok && t < n; ++t, ++g) {
        // At the last tile, look up the next item's first live tile (its
        // list was published an item ago) so its mask words can be fetched early.
        int next_kt = -1;
        if constexpr (kBoolIn) {
          if (!pf_early && t + 1 == n && i + 2 < n_items)
            prefetch_bool_row(item_at(c, i + 2));
        }
        if (t + 1 == n && i + 1 < n_items) {
          const int slot2 = (i + 1) % kSlots;
          if (__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&cc.sched_full[slot2]), ((i + 1) / kSlots) & 1,
                                                         abort_flag, timeout_ns)) &&
              cc.n_live[slot2] > 0) {
            int w2 = 0;
            uint32_t x2 = cc.live_bits[slot2][0];
            next_kt = next_live(cc.live_bits[slot2], w2, x2);
          }
        }
        if (!wait_all(cc.s_full, g & 1)) {
          ok = false;
          break;
        }
        float s[kBN];
#pragma unroll
        for (int ch = 0; ch < kWords; ++ch) tmem_ld32f(t_lane + kSCol + ch * 32, s + ch * 32);
        tmem_wait_ld();
        arrive_warp(cc.s_free);  // the next QK^T may overwrite S now

        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        // A tile every row of the warp keeps whole (dense or prefix-shaped
        // masks) needs the max only.
        uint32_t all_words = mw[0];
#pragma unroll
        for (int ch = 1; ch < kWords; ++ch) all_words &= mw[ch];
        if (__all_sync(0xffffffffu, all_words == 0xFFFFFFFFu)) {
#pragma unroll
          for (int e = 0; e < kBN; e += 2) mx[(e >> 1) & 3] = max3f(mx[(e >> 1) & 3], s[e], s[e + 1]);
        } else {
#pragma unroll
          for (int ch = 0; ch < kWords; ++ch) {
            const uint32_t word = mw[ch];
#pragma unroll
            for (int jj = 0; jj < 32; jj += 2) {
              const float v0 = (word & (1u << jj)) ? s[ch * 32 + jj] : -INFINITY;
              const float v1 = (word & (2u << jj)) ? s[ch * 32 + jj + 1] : -INFINITY;
              s[ch * 32 + jj] = v0;
              s[ch * 32 + jj + 1] = v1;
              mx[(jj >> 1) & 3] = max3f(mx[(jj >> 1) & 3], v0, v1);
            }
          }
        }
        // The next tile's mask words, a whole tile of exponentials ahead of their use.
        if (t + 1 < n) {
          fetch_words(it, next_live(cc.live_bits[slot], lw, lx), mw);
        } else if (next_kt >= 0) {
          fetch_words(item_at(c, i + 1), next_kt, mw);
          have_mw = true;
        }

        // Lazy rescale: the running max only moves when it rises by more than
        // the threshold, so O needs correcting rarely.
        const float x_max = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * scale_log2;
        float alpha = 1.f;
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
        // P (single buffer) was last read by the PV of tile g-1.
        if (g > 0 && !wait_all(cc.pv_done, (g - 1) & 1)) {
          ok = false;
          break;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        const uint64_t scale2 = f2(scale_log2, scale_log2);
        const uint64_t negm2 = f2(-m_use, -m_use);
        // Row sums, two keys per add (f32x2): la2 of P as computed, lr2
        // (bf16) of P as rounded for the PV product.
        uint64_t la2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
        uint64_t lr2[2] = {f2(0.f, 0.f), f2(0.f, 0.f)};
#pragma unroll
        for (int ch = 0; ch < kWords; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            float x0, x1;
            f2_split(fma2(f2(s[ch * 32 + 2 * jj], s[ch * 32 + 2 * jj + 1]), scale2, negm2), x0, x1);
            const float p0 = ex2f(x0);
            const float p1 = ex2f(x1);
            pk[jj] = pack2<BF16>(p0, p1);
            la2[jj & 1] = add2(la2[jj & 1], f2(p0, p1));
            if constexpr (BF16) {
              lr2[jj & 1] = add2(lr2[jj & 1], f2(__uint_as_float(pk[jj] << 16), __uint_as_float(pk[jj] & 0xFFFF0000u)));
            }
          }
          tmem_st16(t_lane + kPCol + ch * 16, pk);
        }
        float la[2], lr[2];
        f2_split(add2(la2[0], la2[1]), la[0], la[1]);
        f2_split(add2(lr2[0], lr2[1]), lr[0], lr[1]);
        if (__any_sync(0xffffffffu, rescale)) {
          // Rare: the running max rose by more than the threshold; bring O
          // (PV of tiles before g, complete) to the new max before PV of g.
#pragma unroll 1
          for (int ch = 0; ch < D / 16; ++ch) {
            uint32_t u[16];
            tmem_ld16(t_lane + kOCol + ch * 16, u);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 16; ++q) u[q] = __float_as_uint(__uint_as_float(u[q]) * alpha);
            tmem_st16(t_lane + kOCol + ch * 16, u);
          }
        }
        tmem_wait_st();
        arrive_warp(cc.p_full);
        const float l_tile = la[0] + la[1];
        l_run += l_tile;
        l_out += BF16 ? lr[0] + lr[1] : l_tile;
      }
      // This item's live list is no longer read.
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&cc.sched_empty[slot]));

      // ------------------------------------------------------------ epilogue
      // Scan of item i+2: its mask rows are prefetched into L1 before the
      // wait for the last PV, so the loads after it hit (a prefetch holds no
      // registers).
      const bool do_scan = i + 2 < n_items;
      const Item itn = item_at(c, do_scan ? i + 2 : i);
      // D = 128 loads short rows (up to kEpiGroups 16-byte groups) outright
      // below, before it writes O.
      const bool scan_regs = !kBoolIn && !C::kStageO && vec && G4 <= kEpiGroups;
      if (!kBoolIn && do_scan && occ == nullptr && !scan_regs) prefetch_rows_l1(itn);
      const float inv = (l_out > 0.f) ? (1.f / l_out) : 0.f;
      const float lse_row = (l_run > 0.f) ? (m_run + log2f(l_run)) * kLn2 : -FLT_MAX;
      // The last PV of the item (O complete); a warp-wide wait.
      auto wait_o = [&]() -> bool {
        const bool ready = ok && n > 0 && wait_all(cc.pv_done, (g - 1) & 1);
        if (n > 0 && !ready) ok = false;
        return ready;
      };
      if constexpr (kSplitK) {
        // A piece of a split item (no O staging, no scan ahead: i+2 is
        // scanned below like any unit).  Its unnormalised O (FP32) and (max,
        // sums) go to the workspace; the piece that completes the item's
        // count merges the item's pieces in piece order, so the result does
        // not depend on which piece finishes last.
        if (do_scan && occ == nullptr) scan_item(itn, i + 2);
        named_bar_sync(bar_id, 128);
        if (wq == 0 && do_scan) publish(i + 2);
        const int w = chain_item(c, i);
        const int item = w / sp.pieces;
        const int64_t n_units = static_cast<int64_t>(total_items);
        float* ml = sp.ws + (static_cast<int64_t>(w) * kBM + r) * 4;
        float* po = sp.ws + n_units * kBM * 4 + (static_cast<int64_t>(w) * kBM + r) * D;
        const bool o_ready = wait_o();
#pragma unroll 1
        for (int dc = 0; dc < D / 32; ++dc) {
          uint32_t u[32];
          if (o_ready) {
            tmem_ld32(t_lane + kOCol + dc * 32, u);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q) u[q] = 0u;
          }
#pragma unroll
          for (int q = 0; q < 8; ++q)
            reinterpret_cast<uint4*>(po + dc * 32)[q] = make_uint4(u[4 * q], u[4 * q + 1], u[4 * q + 2], u[4 * q + 3]);
        }
        *reinterpret_cast<float4*>(ml) = make_float4(m_run, l_run, l_out, 0.f);
        __threadfence();
        named_bar_sync(bar_id, 128);
        if (r == 0) {
          const bool last = claim_last_piece(sp.cnt + item, sp.epoch, sp.pieces);
          // The item's count starts from zero again, so a replay of the same
          // launch (a CUDA graph: same workspace, same epoch) counts afresh.
          if (last) atomicExch(sp.cnt + item, 0ull);
          cc.split_last = last ? 1u : 0u;
        }
        named_bar_sync(bar_id, 128);
        if (cc.split_last != 0u && r < it.rows_valid) {
          __threadfence();
          merge_pieces<D, BF16>(sp, n_units, static_cast<int64_t>(item) * sp.pieces, r,
                                out + (static_cast<int64_t>(it.bh) * N + it.q0 + r) * D,
                                lse != nullptr ? lse + static_cast<int64_t>(it.bh) * N + it.q0 + r : nullptr,
                                ctl.abort_flag == 0);
        }
      } else if constexpr (C::kStageO) {
        // The work that does not need O goes first, under the last PV's
        // latency: the scan of item i+2, the barrier that also frees the
        // staging tile (the previous item's O store has read it), and the
        // publication of item i+2's list.
        if (do_scan && occ == nullptr) scan_item(itn, i + 2);
        if (r == 0) bulk_wait_group_read0();
        named_bar_sync(bar_id, 128);
        if (wq == 0 && do_scan) publish(i + 2);
        // O of the item, normalised and packed to 16-bit pairs (32 words per
        // row), through the staging tile and one TMA store.
        const bool o_ready = wait_o();
        uint32_t u0[32], u1[32];
        if (o_ready) {
          tmem_ld32(t_lane + kOCol, u0);
          tmem_ld32(t_lane + kOCol + 32, u1);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) u0[e] = u1[e] = 0u;
        }
        uint32_t h[32];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          h[e] = pack2<BF16>(__uint_as_float(u0[2 * e]) * inv, __uint_as_float(u0[2 * e + 1]) * inv);
          h[16 + e] = pack2<BF16>(__uint_as_float(u1[2 * e]) * inv, __uint_as_float(u1[2 * e + 1]) * inv);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int chunk = q ^ (r & 7);  // 128-byte swizzle of the O tensor map
          *reinterpret_cast<uint4*>(out_row + chunk * 16) =
              make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
        }
        if (lse != nullptr && r < it.rows_valid) lse[static_cast<int64_t>(it.bh) * N + it.q0 + r] = lse_row;
        fence_proxy_async_smem();
        named_bar_sync(bar_id, 128);
        if (r == 0 && ctl.abort_flag == 0) {
          tma_store_3d(&tm_o, sO, 0, it.q0, it.bh);
          bulk_commit_group();
        }
      } else {
        const bool o_ready = wait_o();
        // The scan loads of item i+2 go first and land while O is written.
        uint4 sv[kEpiGroups];
        const bool load_sv = scan_regs && do_scan && occ == nullptr && r < itn.rows_valid;
#pragma unroll
        for (int u = 0; u < kEpiGroups; ++u)
          sv[u] = (load_sv && u < G4) ? __ldg(reinterpret_cast<const uint4*>(row_ptr(itn)) + u)
                                      : make_uint4(0u, 0u, 0u, 0u);
        // O of the item, normalised, stored from registers 32 columns (64
        // bytes of the row) at a time, as two 32-byte stores when `out` allows.
        uint16_t* orow = out + (static_cast<int64_t>(it.bh) * N + it.q0 + r) * D;
        const bool store = r < it.rows_valid && ctl.abort_flag == 0;
#pragma unroll 1
        for (int dc = 0; dc < D / 32; ++dc) {
          uint32_t u[32];
          if (o_ready) {
            tmem_ld32(t_lane + kOCol + dc * 32, u);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) u[e] = 0u;
          }
          uint32_t hw[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            hw[e] = pack2<BF16>(__uint_as_float(u[2 * e]) * inv, __uint_as_float(u[2 * e + 1]) * inv);
          if (store) {
            if (o_wide) {
              st_global_v8(orow + dc * 32, hw, 0);
              st_global_v8(orow + dc * 32 + 16, hw, 8);
            } else {
              uint4* dst = reinterpret_cast<uint4*>(orow + dc * 32);
#pragma unroll
              for (int q = 0; q < 4; ++q) dst[q] = make_uint4(hw[4 * q], hw[4 * q + 1], hw[4 * q + 2], hw[4 * q + 3]);
            }
          }
        }
        if (lse != nullptr && r < it.rows_valid) lse[static_cast<int64_t>(it.bh) * N + it.q0 + r] = lse_row;
        if (do_scan && occ == nullptr) {
          if (scan_regs) {  // kEpiGroups groups: tiles 0 .. 15, word 0
            uint32_t bits = 0u;
#pragma unroll
            for (int u = 0; u < kEpiGroups; ++u)
              if (u < G4) bits |= group_live<D>(sv[u], u, 0, N);
            const uint32_t x = __reduce_or_sync(0xffffffffu, bits);
            if (lane == 0 && x != 0u) atomicOr(&cc.scan_bits[(i + 2) % kSlots][0], x);
          } else {
            scan_item(itn, i + 2);
          }
        }
        named_bar_sync(bar_id, 128);
        if (wq == 0 && do_scan) publish(i + 2);
      }
    }
    if (!ok && lane == 0) fail();
    if constexpr (C::kStageO) {
      if (r == 0) bulk_wait_group_read0();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 10) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side

template <int D, bool BF16, bool kBoolIn, bool kSplitK>
int launch(const AttnParams& p, int pieces, const char** msg) {
  using C = ChainCfg<D>;
  constexpr size_t kSmemBytes = smem_bytes<D>();
  const int64_t BH = p.B * p.H;
  const int64_t N = p.N;
  const int64_t W = (N + 31) / 32;
  const int64_t KT = (N + C::kBN - 1) / C::kBN;
  const int64_t QT = (N + kBM - 1) / kBM;
  const int64_t items = QT * BH;
  const int64_t total = kSplitK ? items * pieces : items;  // work units
  if (total > 0x3FFFFFFFll) {
    *msg = "attention: batch*heads too large";
    return kErrArg;
  }
  CUtensorMap mq, mk, mv, mo;
  CUresult rc = make_tensor_map_3d(&mq, p.q, p.dtype, D, BH, N, kBM);
  if (rc == CUDA_SUCCESS) rc = make_tensor_map_3d(&mk, p.k, p.dtype, D, BH, N, C::kBN);
  if (rc == CUDA_SUCCESS) rc = make_tensor_map_3d(&mv, p.v, p.dtype, D, BH, N, C::kBN);
  if (rc == CUDA_SUCCESS) rc = make_tensor_map_3d(&mo, p.out, p.dtype, D, BH, N, kBM);
  if (rc != CUDA_SUCCESS) {
    *msg = tensor_map_error("attention", rc);
    return kErrCuda;
  }
  DeviceProps dp;
  if (!device_props(&dp, msg)) return kErrCuda;
  static std::atomic<bool> smem_set[kMaxDevices] = {};
  auto kern = attn_fwd_chain_kernel<D, BF16, kBoolIn, kSplitK>;
  {
    cudaError_t e = ensure_smem_limit(kern, kSmemBytes, dp.device, smem_set);
    if (e != cudaSuccess) {
      *msg = cudaGetErrorString(e);
      return kErrLaunch;
    }
  }
  // Bool input: the kernel packs into p.packed_out and reads its words back.
  const uint32_t* words = kBoolIn ? p.packed_out : p.mask;
  const int vec = (W % 4 == 0 && (reinterpret_cast<uintptr_t>(words) & 15u) == 0) ? 1 : 0;
  const int o_wide = (reinterpret_cast<uintptr_t>(p.out) & 31u) == 0 ? 1 : 0;  // 32-byte O stores (D = 128)
  // Head-major item order once K and V of all heads exceed half of L2.
  const int head_major = 2 * BH * N * D * 2 > dp.l2_bytes / 2 ? 1 : 0;
  const int grid = static_cast<int>(total < dp.sms ? total : dp.sms);
  // The occupancy map describes 128-key tiles: only the D = 64 kernel uses it.
  const uint32_t* occ = (D == 64 && !kBoolIn) ? p.occ : nullptr;
  // Bool input: item i+2's bool rows are prefetched into L2 when item i
  // starts if two rounds of items' rows (2 chains per CTA) take at most 48
  // MB of L2, else at item i's last tile.
  const int pf_early = 2 * static_cast<int64_t>(grid) * 2 * kBM * N <= (int64_t{48} << 20) ? 1 : 0;
  SplitParams sp{};
  void* ws = nullptr;
  if constexpr (kSplitK) {
    // Counters (one per item), then (max, sums) and the FP32 O of every unit.
    const size_t cnt_bytes = (static_cast<size_t>(items) * 8 + 255) / 256 * 256;
    const size_t rows = static_cast<size_t>(total) * kBM;
    cudaError_t ea = scratch_alloc_async(&ws, cnt_bytes + rows * (4 + D) * sizeof(float), p.stream);
    if (ea != cudaSuccess) {
      *msg = cudaGetErrorString(ea);
      return kErrCuda;
    }
    sp.pieces = pieces;
    sp.cnt = static_cast<unsigned long long*>(ws);
    sp.ws = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + cnt_bytes);
    sp.epoch = next_launch_epoch();
  }
  cudaError_t e = launch_pdl(kern, static_cast<unsigned>(grid), kThreads, kSmemBytes, p.stream, mq, mk, mv, mo,
                             static_cast<uint16_t*>(p.out), kBoolIn ? nullptr : p.mask, kBoolIn ? p.bmask : nullptr,
                             kBoolIn ? p.packed_out : nullptr, occ, p.lse, static_cast<int>(N), static_cast<int>(BH),
                             static_cast<int>(W), static_cast<int>(KT), static_cast<int>(total), vec, o_wide,
                             head_major, pf_early, p.scale * kLog2e, sp, p.err_word, p.timeout_ns);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (ws != nullptr) {
    cudaError_t ef = cudaFreeAsync(ws, p.stream);
    if (e == cudaSuccess) e = ef;
  }
  if (e != cudaSuccess) {
    static thread_local char buf[256];
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, kern);
    snprintf(buf, sizeof(buf), "%s (chain kernel: %d threads, %d regs/thread, max %d threads/block, %zu B dynamic smem)",
             cudaGetErrorString(e), kThreads, fa.numRegs, fa.maxThreadsPerBlock, kSmemBytes);
    *msg = buf;
    return kErrLaunch;
  }
  return kOk;
}

}  // namespace

bool chain_supported(const AttnParams& p) {
  return (p.D == 64 && p.N <= ChainCfg<64>::kMaxN) || (p.D == 128 && p.N <= ChainCfg<128>::kMaxN);
}

template <bool kBoolIn>
int launch_any(const AttnParams& p, int pieces, const char** msg) {
  if (pieces >= 2) {
    if (p.D == 128)
      return p.dtype == 1 ? launch<128, true, kBoolIn, true>(p, pieces, msg) : launch<128, false, kBoolIn, true>(p, pieces, msg);
    return p.dtype == 1 ? launch<64, true, kBoolIn, true>(p, pieces, msg) : launch<64, false, kBoolIn, true>(p, pieces, msg);
  }
  if (p.D == 128)
    return p.dtype == 1 ? launch<128, true, kBoolIn, false>(p, 1, msg) : launch<128, false, kBoolIn, false>(p, 1, msg);
  return p.dtype == 1 ? launch<64, true, kBoolIn, false>(p, 1, msg) : launch<64, false, kBoolIn, false>(p, 1, msg);
}

int launch_attn_fwd_chain(const AttnParams& p, const char** msg) {
  // Split along keys when the items (batch*head x 128-row query tiles) leave
  // chains idle and are long: as many pieces per item as fill the chains,
  // each of at least kSplitMinTiles key tiles (shorter pieces lose to the
  // merge and the per-unit fixed costs).
  DeviceProps dp;
  if (!device_props(&dp, msg)) return kErrCuda;
  const int64_t items = (p.N + kBM - 1) / kBM * p.B * p.H;
  const int64_t kt = p.D == 64 ? (p.N + 127) / 128 : (p.N + 63) / 64;
  const int64_t chains = 2 * static_cast<int64_t>(dp.sms);
  int pieces = 1;
  if (items > 0 && items < chains)
    pieces = static_cast<int>(std::min<int64_t>({kt / kSplitMinTiles, chains / items, 255}));
  return p.bmask != nullptr ? launch_any<true>(p, pieces, msg) : launch_any<false>(p, pieces, msg);
}

}  // namespace sma
