// ORACLE — test infrastructure only.
//
// extern "C" entry points around the reference's own CUDA kernels
// (csrc/sparse_attention.cu of yulangz/sparse-mask-attention-auto-research),
// compiled from the reference sources where they lie by oracle/build_ref.py
// into oracle/_ref/libref_sma.so.  GPU tests use it as a second checker at
// full workload sizes; nothing in the product links or loads it.
#include <cuda_runtime.h>
#include <stdint.h>

#include "sparse_attention.h"  // reference header: SparseAttentionParams + launchers

extern "C" {

// pack_mask_bits(), csrc/sparse_attention.cu:44-54
int ref_pack_mask(const void* mask, void* packed, int B, int H, int N, void* stream) {
  pack_mask_bits(static_cast<const bool*>(mask), static_cast<uint32_t*>(packed), B, H, N,
                 static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}

// sparse_attention_fwd_fp16/_bf16(), csrc/sparse_attention.cu:149-185, with
// the parameter block filled the way csrc/binding.cpp:24-36 fills it.
int ref_attn_fwd(int bf16, const void* q, const void* k, const void* v, const void* mask_packed, void* out,
                 float* lse, int B, int H, int N, int D, float scale, int is_training, void* stream) {
  SparseAttentionParams p{};
  p.q = q;
  p.k = k;
  p.v = v;
  p.mask_packed = static_cast<const uint32_t*>(mask_packed);
  p.out = out;
  p.lse = is_training ? lse : nullptr;
  p.batch_size = B;
  p.num_heads = H;
  p.seq_len = N;
  p.head_dim = D;
  p.scale = scale;
  p.is_training = is_training != 0;
  if (bf16)
    sparse_attention_fwd_bf16(p, static_cast<cudaStream_t>(stream));
  else
    sparse_attention_fwd_fp16(p, static_cast<cudaStream_t>(stream));
  return static_cast<int>(cudaGetLastError());
}

}  // extern "C"
