// Internal launcher interface shared by the kernel translation units and the
// C-ABI layer (sma_capi.cu).  Nothing here is exported from the library.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace sma {

// Status codes (mirrored by the public SMA_* values in include/sma_capi.h).
enum : int {
  kOk = 0,
  kErrArg = 1,
  kErrDtype = 2,
  kErrUnsupportedD = 3,
  kErrLaunch = 4,
  kErrTimeout = 5,
  kErrUnsupportedN = 6,
  kErrCuda = 7,
};

struct AttnParams {
  int dtype;                  // 0 = fp16, 1 = bf16
  const void* q;              // [B, H, N, D] contiguous
  const void* k;
  const void* v;
  const uint32_t* mask;       // [B, H, N, ceil(N/32)] packed bits, LSB = lowest column
  void* out;                  // [B, H, N, D] contiguous
  float* lse;                 // [B, H, N] or nullptr
  int64_t B, H, N, D;
  float scale;
  const uint32_t* occ;        // [B*H, ceil(N/128), 2] live key-tile bits per query tile, or nullptr
  // Bool-mask input instead of `mask`: [B, H, N, N] bytes (non-zero = attend),
  // N % 32 == 0, 16-byte aligned; the kernel writes the packed words to
  // packed_out ([B, H, N, N/32], 16-byte aligned) and reads them back.
  const uint8_t* bmask;
  uint32_t* packed_out;
  uint32_t* err_word;         // device word the kernel ORs error bits into
  uint64_t timeout_ns;        // bound on every device-side wait
  cudaStream_t stream;
};

// Largest sequence length: the attention kernel keeps one live bit per key
// tile in 32 words per item (1024 tiles of 64 keys); the occupancy map holds
// two 32-bit words (64 key tiles of 128) per query tile.
constexpr int64_t kMaxSeqLen = 65536;
constexpr int64_t kMaxSeqLenOcc = 8192;

int launch_pack_mask(const uint8_t* mask, uint32_t* packed, int64_t rows, int64_t n,
                     cudaStream_t stream, const char** msg);

// Packs like launch_pack_mask and writes the occupancy map `occ`
// ([bh, ceil(n/128), 2] uint32: bit t = key tile t has a set bit in the
// 128-row query tile).  Needs n % 32 == 0, n <= kMaxSeqLenOcc, aligned pointers.
int launch_pack_mask_occ(const uint8_t* mask, uint32_t* packed, uint32_t* occ, int64_t bh, int64_t n,
                         cudaStream_t stream, const char** msg);

int launch_attn_fwd(const AttnParams& p, const char** msg);

struct BwdParams {
  int dtype;                  // 0 = fp16, 1 = bf16
  const void* q;              // [B, H, N, D] contiguous, as for the forward
  const void* k;
  const void* v;
  const void* out;            // the forward's O
  const void* dout;           // upstream gradient of O
  const float* lse;           // [B, H, N] the forward's LSE (natural log, -FLT_MAX for empty rows)
  const uint32_t* mask;       // packed mask
  void* dq;                   // [B, H, N, D] outputs
  void* dk;
  void* dv;
  float* dq_accum;            // [B, H, N, D] FP32 scratch
  float* delta;               // [B, H, N] FP32 scratch
  int64_t B, H, N, D;
  float scale;
  uint32_t* err_word;
  uint64_t timeout_ns;
  cudaStream_t stream;
};

// Backward (attn_bwd.cu): head dims 64 and 128.
int launch_attn_bwd(const BwdParams& p, const char** msg);

// TMA map of the [BH, N, D] view of a contiguous [B, H, N, D] fp16/bf16
// tensor: boxes of 64 head dims (one 128-byte swizzle span) by `rows` rows,
// 128-byte swizzle (tma_map.cu).  Returns the driver's status
// (CUDA_ERROR_NOT_FOUND when the entry point is missing).
CUresult make_tensor_map_3d(CUtensorMap* m, const void* ptr, int dtype, int64_t D, int64_t BH, int64_t N, int rows);
// The same view of a contiguous FP32 [BH, N, D] tensor: boxes of 32 elements
// (128 bytes) by `rows` rows, 128-byte swizzle (tma_map.cu).
CUresult make_tensor_map_3d_f32(CUtensorMap* m, const void* ptr, int64_t D, int64_t BH, int64_t N, int rows);
// Message for a failed tensor-map encode: `what` and the driver status.
const char* tensor_map_error(const char* what, CUresult rc);

// Stream-ordered scratch from a per-device memory pool that keeps its memory
// between calls (no release back to the driver), so a steady stream of
// launches allocates only once.  Freed with cudaFreeAsync on the same stream.
cudaError_t scratch_alloc_async(void** p, size_t bytes, cudaStream_t stream);
// A value distinct for every call in the process: 56 bits, never 0.
unsigned long long next_launch_epoch();

// Devices the per-device caches of the launchers cover.
constexpr int kMaxDevices = 64;

// Properties of the current device, queried once per device (thread-safe).
struct DeviceProps {
  int device = -1;
  int sms = 0;
  int l2_bytes = 0;
};
bool device_props(DeviceProps* out, const char** msg);

// Raises `kern`'s dynamic shared-memory limit to `bytes` on the current
// device the first time it is launched there.  `done` is the kernel's own
// per-device flag array; concurrent first calls both set the same attribute.
template <typename Kern>
cudaError_t ensure_smem_limit(Kern kern, size_t bytes, int dev, std::atomic<bool> (&done)[kMaxDevices]) {
  if (done[dev].load(std::memory_order_relaxed)) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) done[dev].store(true, std::memory_order_relaxed);
  return e;
}

// Launches `kern` with programmatic stream serialisation: its CTAs may start
// (and run their set-up) while the previous kernel in the stream finishes;
// the kernel itself calls griddepcontrol.wait before reading global memory.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kern)(Params...), unsigned grid, unsigned block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Params>(args)...);
}

// Persistent two-chain kernel (attn_fwd_chain.cu): head dims 64 and 128, N up
// to kMaxSeqLen.  launch_attn_fwd dispatches to it when chain_supported().
bool chain_supported(const AttnParams& p);
int launch_attn_fwd_chain(const AttnParams& p, const char** msg);

// Launches one CTA that waits on an mbarrier nothing ever arrives on, using
// the same bounded-wait helper as the attention kernel; it must give up after
// `timeout_ns` and set bit 1 of *err_word.
int launch_wait_probe(uint32_t* err_word, uint64_t timeout_ns, cudaStream_t stream);

// Device error bits.
constexpr uint32_t kDevErrTimeout = 1u;
constexpr uint32_t kDevErrLayout = 2u;  // shared-memory window not 1024-byte aligned

}  // namespace sma
