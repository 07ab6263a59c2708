// C-ABI layer of libsma.so: argument validation, dispatch to the kernel
// launchers, the thread-local error message, and the device error word the
// kernels raise when a bounded wait gives up.
//
// Mirrors the reference pybind layer (csrc/binding.cpp:9-71), whose checks
// (CUDA tensors, 4-D shapes, fp16/bf16 dtype) become SMA_* status codes here;
// the Python shim turns them into RuntimeError like TORCH_CHECK does.
#include <atomic>
#include <cstdio>
#include <string>

#include <nvtx3/nvToolsExt.h>

#include "sma_capi.h"
#include "sma_internal.h"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_timeout_ns{2000000000ull};

// NVTX range over one entry point (host side: argument checks and launches).
// nvtx3 is header-only and costs a branch when no profiler is attached.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

// Device word the kernels OR error bits into (one instance per device).
__device__ uint32_t g_device_error_word;

using sma::kMaxDevices;
// Per-device address caches.  Several host threads may fill an entry on their
// first call; they all store the same value, and the atomics make that
// well-defined.
std::atomic<uint32_t*> g_err_ptr[kMaxDevices] = {};

int fail(int code, const char* msg) {
  g_last_error = msg ? msg : "unknown error";
  return code;
}

int fail_cuda(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return sma::kErrCuda;
}

// Device address of the error word on the current device.  Every entry point
// that launches calls this first; it also makes the device's primary context
// current on the calling thread, which the runtime otherwise binds only at the
// thread's first runtime call that needs it, while the tensor-map encoding
// (a driver call) needs it bound already.  A host thread whose first CUDA
// work is a call into this library (an autograd worker, say) would otherwise
// fail there.
int error_word(uint32_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(sma::kErrCuda, "device index out of range");
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaSetDevice");
  uint32_t* ptr = g_err_ptr[dev].load(std::memory_order_relaxed);
  if (ptr == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_device_error_word);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress");
    ptr = static_cast<uint32_t*>(p);
    g_err_ptr[dev].store(ptr, std::memory_order_relaxed);
  }
  *out = ptr;
  return sma::kOk;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Fixed device scratch of sma_attn_bwd_noalloc: the FP32 dQ accumulator
// (B*H*N*D floats) followed by Delta (B*H*N floats).  One copy per device,
// part of the module image (so it is reserved on every device where the
// library's module is loaded, whether or not the entry point is called),
// so that entry point allocates nothing.
constexpr int64_t kNoAllocScratchFloats = int64_t{8} << 20;  // 32 MiB
static __device__ __align__(256) float g_bwd_noalloc_scratch[kNoAllocScratchFloats];
std::atomic<float*> g_noalloc_ptr[kMaxDevices] = {};

// Device address of the fixed scratch on the current device (looked up once per device).
int noalloc_scratch(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(sma::kErrCuda, "device index out of range");
  float* ptr = g_noalloc_ptr[dev].load(std::memory_order_relaxed);
  if (ptr == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bwd_noalloc_scratch);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress");
    ptr = static_cast<float*>(p);
    g_noalloc_ptr[dev].store(ptr, std::memory_order_relaxed);
  }
  *out = ptr;
  return sma::kOk;
}

}  // namespace

extern "C" {

int sma_pack_mask(const void* mask, void* packed, int64_t B, int64_t H, int64_t N, void* stream) {
  NvtxRange range("sma_pack_mask");
  if (B < 0 || H < 0 || N < 0) return fail(sma::kErrArg, "pack_mask: negative dimension");
  if (B == 0 || H == 0 || N == 0) return sma::kOk;
  if (mask == nullptr || packed == nullptr) return fail(sma::kErrArg, "pack_mask: null pointer");
  const char* msg = nullptr;
  int rc = sma::launch_pack_mask(static_cast<const uint8_t*>(mask), static_cast<uint32_t*>(packed), B * H * N,
                                 N, static_cast<cudaStream_t>(stream), &msg);
  return rc == sma::kOk ? rc : fail(rc, msg);
}

}  // extern "C"

namespace {

// bool_mask != nullptr: the forward reads the bool mask itself and writes the
// packed words to mask_packed (sma_attn_fwd_mask).
int attn_fwd_impl(int dtype, const void* q, const void* k, const void* v, const void* mask_packed,
                  const uint32_t* occupancy, const void* bool_mask, void* out, float* lse, int64_t B, int64_t H,
                  int64_t N, int64_t D, float scale, void* stream) {
  NvtxRange range(bool_mask != nullptr ? "sma_attn_fwd_mask" : "sma_attn_fwd");
  if (dtype != SMA_DTYPE_FP16 && dtype != SMA_DTYPE_BF16)
    return fail(sma::kErrDtype, "attention: unsupported dtype, need fp16 or bf16");
  if (B < 0 || H < 0 || N < 0 || D <= 0) return fail(sma::kErrArg, "attention: bad dimension");
  if (D != 64 && D != 128) return fail(sma::kErrUnsupportedD, "attention: head dim must be 64 or 128");
  if (N > SMA_MAX_SEQ_LEN)
    return fail(sma::kErrUnsupportedN, "attention: sequence length above the supported maximum (65536)");
  if (occupancy != nullptr && N > SMA_MAX_SEQ_LEN_OCCUPANCY)
    return fail(sma::kErrUnsupportedN, "attention: occupancy map given for a sequence length above 8192");
  if (!(scale > 0.f) || !(scale < INFINITY)) return fail(sma::kErrArg, "attention: scale must be finite and > 0");
  if (B == 0 || H == 0 || N == 0) return sma::kOk;
  if (!q || !k || !v || !mask_packed || !out) return fail(sma::kErrArg, "attention: null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(sma::kErrArg, "attention: q/k/v/out must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(mask_packed) & 3u) != 0 || (lse && (reinterpret_cast<uintptr_t>(lse) & 3u)))
    return fail(sma::kErrArg, "attention: mask_packed/lse must be 4-byte aligned");
  if (bool_mask != nullptr && (N % 32 != 0 || !aligned16(bool_mask) || !aligned16(mask_packed)))
    return fail(sma::kErrArg, "attention: the bool-mask forward needs N % 32 == 0 and 16-byte aligned mask / mask_packed");
  uint32_t* err = nullptr;
  int rc = error_word(&err);
  if (rc != sma::kOk) return rc;
  sma::AttnParams p{};
  p.dtype = dtype;
  p.q = q;
  p.k = k;
  p.v = v;
  p.mask = static_cast<const uint32_t*>(mask_packed);
  p.occ = occupancy;
  p.bmask = static_cast<const uint8_t*>(bool_mask);
  p.packed_out = bool_mask != nullptr ? static_cast<uint32_t*>(const_cast<void*>(mask_packed)) : nullptr;
  p.out = out;
  p.lse = lse;
  p.B = B;
  p.H = H;
  p.N = N;
  p.D = D;
  p.scale = scale;
  p.err_word = err;
  p.timeout_ns = g_timeout_ns.load(std::memory_order_relaxed);
  p.stream = static_cast<cudaStream_t>(stream);
  const char* msg = nullptr;
  rc = sma::launch_attn_fwd(p, &msg);
  return rc == sma::kOk ? rc : fail(rc, msg);
}

}  // namespace

extern "C" {

int sma_attn_fwd(int dtype, const void* q, const void* k, const void* v, const void* mask_packed, void* out,
                 float* lse, int64_t B, int64_t H, int64_t N, int64_t D, float scale, void* stream) {
  return attn_fwd_impl(dtype, q, k, v, mask_packed, nullptr, nullptr, out, lse, B, H, N, D, scale, stream);
}

int sma_attn_fwd_mask(int dtype, const void* q, const void* k, const void* v, const void* mask, void* mask_packed,
                      void* out, float* lse, int64_t B, int64_t H, int64_t N, int64_t D, float scale, void* stream) {
  if (mask == nullptr && B > 0 && H > 0 && N > 0) return fail(sma::kErrArg, "attention: null mask");
  return attn_fwd_impl(dtype, q, k, v, mask_packed, nullptr, mask, out, lse, B, H, N, D, scale, stream);
}

int sma_pack_mask_occupancy(const void* mask, void* packed, void* occupancy, int64_t B, int64_t H, int64_t N,
                            void* stream) {
  NvtxRange range("sma_pack_mask_occupancy");
  if (B < 0 || H < 0 || N < 0) return fail(sma::kErrArg, "pack_mask_occupancy: negative dimension");
  if (N > SMA_MAX_SEQ_LEN_OCCUPANCY)
    return fail(sma::kErrUnsupportedN, "pack_mask_occupancy: sequence length above the occupancy map's maximum (8192)");
  if (B == 0 || H == 0 || N == 0) return sma::kOk;
  const char* msg = nullptr;
  int rc = sma::launch_pack_mask_occ(static_cast<const uint8_t*>(mask), static_cast<uint32_t*>(packed),
                                     static_cast<uint32_t*>(occupancy), B * H, N,
                                     static_cast<cudaStream_t>(stream), &msg);
  return rc == sma::kOk ? rc : fail(rc, msg);
}

int sma_attn_fwd_occupancy(int dtype, const void* q, const void* k, const void* v, const void* mask_packed,
                           const void* occupancy, void* out, float* lse, int64_t B, int64_t H, int64_t N,
                           int64_t D, float scale, void* stream) {
  if (occupancy == nullptr) return fail(sma::kErrArg, "attention: null occupancy map");
  if ((reinterpret_cast<uintptr_t>(occupancy) & 3u) != 0)
    return fail(sma::kErrArg, "attention: occupancy map must be 4-byte aligned");
  return attn_fwd_impl(dtype, q, k, v, mask_packed, static_cast<const uint32_t*>(occupancy), nullptr, out, lse, B, H,
                       N, D, scale, stream);
}

int sma_attn_bwd(int dtype, const void* q, const void* k, const void* v, const void* out, const void* dout,
                 const float* lse, const void* mask_packed, void* dq, void* dk, void* dv, float* dq_accum, float* delta,
                 int64_t B, int64_t H, int64_t N, int64_t D, float scale, void* stream) {
  NvtxRange range("sma_attn_bwd");
  if (dtype != SMA_DTYPE_FP16 && dtype != SMA_DTYPE_BF16)
    return fail(sma::kErrDtype, "backward: unsupported dtype, need fp16 or bf16");
  if (B < 0 || H < 0 || N < 0 || D <= 0) return fail(sma::kErrArg, "backward: bad dimension");
  if (D != 64 && D != 128) return fail(sma::kErrUnsupportedD, "backward: head dim must be 64 or 128");
  if (N > SMA_MAX_SEQ_LEN) return fail(sma::kErrUnsupportedN, "backward: sequence length above the supported maximum (65536)");
  if (!(scale > 0.f) || !(scale < INFINITY)) return fail(sma::kErrArg, "backward: scale must be finite and > 0");
  if (B == 0 || H == 0 || N == 0) return sma::kOk;
  if (!q || !k || !v || !out || !dout || !lse || !mask_packed || !dq || !dk || !dv || !dq_accum || !delta)
    return fail(sma::kErrArg, "backward: null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(dout) || !aligned16(dq) ||
      !aligned16(dk) || !aligned16(dv) || !aligned16(dq_accum))
    return fail(sma::kErrArg, "backward: q/k/v/out/dout/dq/dk/dv/dq_accum must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(lse) & 3u) || (reinterpret_cast<uintptr_t>(delta) & 3u) ||
      (reinterpret_cast<uintptr_t>(mask_packed) & 3u))
    return fail(sma::kErrArg, "backward: lse/delta/mask_packed must be 4-byte aligned");
  uint32_t* err = nullptr;
  int rc = error_word(&err);
  if (rc != sma::kOk) return rc;
  sma::BwdParams p{};
  p.dtype = dtype;
  p.q = q;
  p.k = k;
  p.v = v;
  p.out = out;
  p.dout = dout;
  p.lse = lse;
  p.mask = static_cast<const uint32_t*>(mask_packed);
  p.dq = dq;
  p.dk = dk;
  p.dv = dv;
  p.dq_accum = dq_accum;
  p.delta = delta;
  p.B = B;
  p.H = H;
  p.N = N;
  p.D = D;
  p.scale = scale;
  p.err_word = err;
  p.timeout_ns = g_timeout_ns.load(std::memory_order_relaxed);
  p.stream = static_cast<cudaStream_t>(stream);
  const char* msg = nullptr;
  rc = sma::launch_attn_bwd(p, &msg);
  return rc == sma::kOk ? rc : fail(rc, msg);
}

int sma_attn_bwd_noalloc(int dtype, const void* q, const void* k, const void* v, const void* out, const void* dout,
                         const float* lse, const void* mask_packed, void* dq, void* dk, void* dv, int64_t B,
                         int64_t H, int64_t N, int64_t D, float scale, void* stream) {
  // The checks of sma_attn_bwd, with its codes, come first; then the size
  // of the fixed scratch.
  if (dtype != SMA_DTYPE_FP16 && dtype != SMA_DTYPE_BF16)
    return fail(sma::kErrDtype, "backward: unsupported dtype, need fp16 or bf16");
  if (B < 0 || H < 0 || N < 0 || D <= 0) return fail(sma::kErrArg, "backward: bad dimension");
  if (D != 64 && D != 128) return fail(sma::kErrUnsupportedD, "backward: head dim must be 64 or 128");
  if (N > SMA_MAX_SEQ_LEN) return fail(sma::kErrUnsupportedN, "backward: sequence length above the supported maximum (65536)");
  if (B == 0 || H == 0 || N == 0) return sma::kOk;
  // dQ accumulator + Delta must fit the fixed scratch (checked without overflow).
  const int64_t per_bh = N * (D + 1);
  if (B > kNoAllocScratchFloats || H > kNoAllocScratchFloats || B * H > kNoAllocScratchFloats / per_bh)
    return fail(sma::kErrArg, "backward (no-alloc): B*H*N*(D+1) floats exceed the fixed 32 MiB scratch");
  float* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != sma::kOk) return rc;
  return sma_attn_bwd(dtype, q, k, v, out, dout, lse, mask_packed, dq, dk, dv, scratch, scratch + B * H * N * D, B,
                      H, N, D, scale, stream);
}

int sma_device_status(void* stream, int clear) {
  uint32_t* err = nullptr;
  int rc = error_word(&err);
  if (rc != sma::kOk) return rc;
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda(e, "cudaStreamSynchronize");
  uint32_t v = 0;
  e = cudaMemcpyAsync(&v, err, sizeof(v), cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda(e, "read device error word");
  if (clear) {
    // Ordered on the caller's stream, so other streams of the device keep running.
    e = cudaMemsetAsync(err, 0, sizeof(uint32_t), static_cast<cudaStream_t>(stream));
    if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail_cuda(e, "clear device error word");
  }
  if (v & sma::kDevErrTimeout) return fail(sma::kErrTimeout, "a device-side wait timed out");
  if (v & sma::kDevErrLayout) return fail(sma::kErrCuda, "attention kernel: shared memory not 1024-byte aligned");
  return sma::kOk;
}

int sma_set_wait_timeout_ns(uint64_t ns) {
  if (ns == 0) return fail(sma::kErrArg, "timeout must be positive");
  g_timeout_ns.store(ns, std::memory_order_relaxed);
  return sma::kOk;
}

int sma_debug_wait_probe(uint64_t timeout_ns, void* stream) {
  uint32_t* err = nullptr;
  int rc = error_word(&err);
  if (rc != sma::kOk) return rc;
  rc = sma::launch_wait_probe(err, timeout_ns, static_cast<cudaStream_t>(stream));
  return rc == sma::kOk ? rc : fail(rc, "wait probe launch failed");
}

const char* sma_last_error(void) { return g_last_error.c_str(); }

int sma_abi_version(void) { return SMA_ABI_VERSION; }

}  // extern "C"
