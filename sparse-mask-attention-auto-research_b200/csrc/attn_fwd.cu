// Attention forward dispatch and the bounded-wait probe.
//
// Computes, per (batch*head, query row r):
//   s_j  = scale * <q_r, k_j>                     for every key j with mask bit set
//   O_r  = sum_j softmax(s)_j * v_j               (0 if the row has no set bit)
//   lse_r = log(sum_j exp(s_j))                   (-FLT_MAX if the row has no set bit)
// which is the reference forward (csrc/sparse_attention.cu:64-143; FP32 oracle
// python/sparse_attention.py:26-44).  Both head dims run the persistent
// two-chain kernel of attn_fwd_chain.cu (128-key tiles for D = 64, 64-key
// tiles for D = 128); this file checks the sequence-length limits and holds
// the probe kernel the tests use to show that a device-side wait gives up
// and reports instead of hanging.
#include "sma_internal.h"
#include "sma_ptx.cuh"

namespace sma {
namespace {

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
  if (p.D != 64 && p.D != 128) {
    *msg = "attention: head dim must be 64 or 128";
    return kErrUnsupportedD;
  }
  if (p.N > kMaxSeqLen) {
    *msg = "attention: sequence length above the supported maximum (65536)";
    return kErrUnsupportedN;
  }
  if (p.occ != nullptr && p.N > kMaxSeqLenOcc) {
    *msg = "attention: occupancy map given for a sequence length above 8192";
    return kErrUnsupportedN;
  }
  if (p.bmask != nullptr && (p.N % 32 != 0 || p.packed_out == nullptr ||
                            (reinterpret_cast<uintptr_t>(p.bmask) & 15u) != 0 ||
                            (reinterpret_cast<uintptr_t>(p.packed_out) & 15u) != 0)) {
    *msg = "attention: the bool-mask forward needs N % 32 == 0 and 16-byte aligned mask / packed output";
    return kErrArg;
  }
  if (!chain_supported(p)) {
    *msg = "attention: shape not supported by the attention kernel";
    return kErrUnsupportedN;
  }
  return launch_attn_fwd_chain(p, msg);
}

int launch_wait_probe(uint32_t* err_word, uint64_t timeout_ns, cudaStream_t stream) {
  wait_probe_kernel<<<1, 32, 0, stream>>>(err_word, timeout_ns);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace sma
