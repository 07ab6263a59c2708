// Host-side helpers of the kernel launchers: TMA tensor maps and per-device
// properties.  The driver entry point is reached through the runtime
// (cudaGetDriverEntryPoint), so the library does not link libcuda.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdio>
#include <mutex>

#include "sma_internal.h"

namespace sma {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 lookup_encode_fn() {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  return nullptr;
}

// Looked up once per process (a function-local static is initialised once,
// even with several host threads).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static const PFN_cuTensorMapEncodeTiled_v12000 fn = lookup_encode_fn();
  return fn;
}

struct DeviceSlot {
  std::once_flag once;
  DeviceProps props;
  bool ok = false;
};
DeviceSlot g_devices[kMaxDevices];

}  // namespace

bool device_props(DeviceProps* out, const char** msg) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *msg = "no current CUDA device (or device index out of range)";
    return false;
  }
  DeviceSlot& s = g_devices[dev];
  std::call_once(s.once, [&]() {
    s.props.device = dev;
    s.ok = cudaDeviceGetAttribute(&s.props.sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
           cudaDeviceGetAttribute(&s.props.l2_bytes, cudaDevAttrL2CacheSize, dev) == cudaSuccess && s.props.sms > 0;
  });
  if (!s.ok) {
    *msg = "cannot query the SM count / L2 size of the current device";
    return false;
  }
  *out = s.props;
  return true;
}

CUresult make_tensor_map_3d(CUtensorMap* m, const void* ptr, int dtype, int64_t D, int64_t BH, int64_t N, int rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return CUDA_ERROR_NOT_FOUND;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(N * D * 2)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(m, dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
            const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// FP32 [BH][N][D] tensor, boxes of 32 elements (128 bytes, 128-byte swizzle)
// by `rows` rows.
CUresult make_tensor_map_3d_f32(CUtensorMap* m, const void* ptr, int64_t D, int64_t BH, int64_t N, int rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return CUDA_ERROR_NOT_FOUND;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 4), static_cast<cuuint64_t>(N * D * 4)};
  cuuint32_t box[3] = {32u, static_cast<cuuint32_t>(rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

namespace {
struct PoolSlot {
  std::once_flag once;
  cudaMemPool_t pool = nullptr;
  cudaError_t err = cudaSuccess;
};
PoolSlot g_pools[kMaxDevices];
std::atomic<unsigned long long> g_epoch{0};
}  // namespace

cudaError_t scratch_alloc_async(void** p, size_t bytes, cudaStream_t stream) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  PoolSlot& s = g_pools[dev];
  std::call_once(s.once, [&]() {
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    s.err = cudaMemPoolCreate(&s.pool, &props);
    if (s.err == cudaSuccess) {
      uint64_t keep = ~uint64_t{0};
      s.err = cudaMemPoolSetAttribute(s.pool, cudaMemPoolAttrReleaseThreshold, &keep);
    }
  });
  if (s.err != cudaSuccess) return s.err;
  return cudaMallocFromPoolAsync(p, bytes, s.pool, stream);
}

unsigned long long next_launch_epoch() {
  return ((g_epoch.fetch_add(1, std::memory_order_relaxed) + 1) & ((1ull << 55) - 1)) | (1ull << 55);
}

const char* tensor_map_error(const char* what, CUresult rc) {
  static thread_local char buf[160];
  snprintf(buf, sizeof(buf), "%s: cuTensorMapEncodeTiled failed (CUresult %d; pointer alignment, shape, or no driver entry point)",
           what, static_cast<int>(rc));
  return buf;
}

}  // namespace sma
