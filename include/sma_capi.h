/*
 * sma_capi.h - C ABI of the B200 sparse-mask attention library (libsma.so).
 *
 * Plain pointers and sizes only: every tensor argument is a device pointer to
 * a contiguous row-major buffer, every stream argument is a cudaStream_t passed
 * as void* (NULL = legacy default stream).  Work is enqueued asynchronously on
 * that stream; nothing synchronises except sma_device_status().
 *
 * Every function returns an SMA_* status.  On a non-zero status,
 * sma_last_error() returns a message describing the failure (thread-local,
 * valid until the next call on the same thread).
 *
 * Each entry point names the reference interface it replaces
 * (yulangz/sparse-mask-attention-auto-research, paths relative to its root).
 */
#ifndef SMA_CAPI_H_
#define SMA_CAPI_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define SMA_OK 0
#define SMA_ERR_ARG 1             /* bad pointer / size / layout argument          */
#define SMA_ERR_DTYPE 2           /* dtype is neither fp16 nor bf16                 */
#define SMA_ERR_UNSUPPORTED_D 3   /* head dim other than 64 or 128                  */
#define SMA_ERR_LAUNCH 4          /* kernel launch failed                           */
#define SMA_ERR_TIMEOUT 5         /* a device-side wait gave up (see sma_device_status) */
#define SMA_ERR_UNSUPPORTED_N 6   /* sequence length above the path's maximum       */
#define SMA_ERR_CUDA 7            /* CUDA runtime / driver error                    */

/* Element types of q, k, v and out. */
#define SMA_DTYPE_FP16 0
#define SMA_DTYPE_BF16 1

/* Longest supported sequence (both head dims); the occupancy map
 * (sma_pack_mask_occupancy) covers N <= 8192. */
#define SMA_MAX_SEQ_LEN 65536
#define SMA_MAX_SEQ_LEN_OCCUPANCY 8192

#if defined(__GNUC__)
#define SMA_API __attribute__((visibility("default")))
#else
#define SMA_API
#endif
#define SMA_ABI_VERSION 1

/*
 * Pack a bool mask [B, H, N, N] (one byte per element, non-zero = attend)
 * into 32-bit words [B, H, N, ceil(N/32)]: bit b of word w of a row is the
 * mask at column 32*w + b; bits at columns >= N are zero.  The output has the
 * bit pattern of the reference's int32 packed tensor.
 *
 * Replaces: pack_mask()            csrc/binding.cpp:49-66
 *           pack_mask_bits()       csrc/sparse_attention.cu:44-54
 *           (CPU fallback          python/sparse_attention.py:189-206)
 * Unlike the reference binding, the caller allocates `packed`.
 */
SMA_API int sma_pack_mask(const void* mask, void* packed, int64_t B, int64_t H, int64_t N, void* stream);

/*
 * Masked-softmax attention forward:
 *   out[b,h,i,:] = sum_j softmax_j(scale * q_i . k_j  over j with bit(i,j) set) * v[b,h,j,:]
 * q, k, v, out: [B, H, N, D] of `dtype`; mask_packed: [B, H, N, ceil(N/32)]
 * words as produced by sma_pack_mask; lse: [B, H, N] float32 log-sum-exp of
 * the scaled scores, or NULL to skip it (the reference's is_training=false).
 * Rows with no set bit get out = 0 and lse = -FLT_MAX (the reference CUDA
 * convention, csrc/sparse_attention.cu:133,141).
 * Supported: D in {64, 128}, 1 <= N <= SMA_MAX_SEQ_LEN, 16-byte aligned
 * q/k/v/out, scale finite and > 0 (the kernels fold the scale into the
 * exponent after the masked row max; the reference always passes 1/sqrt(D)).
 * When the (batch*head, 128-row query tile) items are fewer than twice the
 * SM count and at least 64 key tiles long, each item is split along keys
 * over several SMs and merged; that path takes scratch (about
 * items * pieces * 128 * (D + 4) floats) from a per-device stream-ordered
 * pool the library keeps, released on `stream` after the launch.
 *
 * Replaces: forward()                          csrc/binding.cpp:9-47
 *           sparse_attention_fwd_fp16/_bf16()  csrc/sparse_attention.cu:149-185
 *           SparseAttentionParams              csrc/sparse_attention.h:12-38
 */
SMA_API int sma_attn_fwd(int dtype, const void* q, const void* k, const void* v, const void* mask_packed,
                 void* out, float* lse, int64_t B, int64_t H, int64_t N, int64_t D, float scale,
                 void* stream);

/*
 * The pack + forward pair in one launch: the attention kernel reads the bool
 * mask [B, H, N, N] (one byte per element, non-zero = attend) itself, packs
 * each query tile's rows as it scans them for live key tiles, and writes the
 * packed words to mask_packed ([B, H, N, N/32], bit for bit what
 * sma_pack_mask writes, kept for the backward).  out and lse are those of
 * sma_attn_fwd on the packed mask, bit for bit.
 * Needs N % 32 == 0 and 16-byte aligned mask and mask_packed (SMA_ERR_ARG
 * otherwise: callers then use sma_pack_mask + sma_attn_fwd); the rest as for
 * sma_attn_fwd.  On B200 the pair of launches is faster (the packer streams
 * the mask at HBM speed, while here each query tile's rows are read and
 * packed by the softmax warps between tiles, on the kernel's critical path),
 * so sparse_attention() uses the pair; this entry saves a launch only.
 *
 * Replaces: the pack_mask() + SparseAttentionFunction forward pair that
 *           sparse_attention() runs   python/sparse_attention.py:122-156
 *           (pack_mask_bits()         csrc/sparse_attention.cu:44-54,
 *            forward()                csrc/binding.cpp:9-47)
 */
SMA_API int sma_attn_fwd_mask(int dtype, const void* q, const void* k, const void* v, const void* mask,
                              void* mask_packed, void* out, float* lse, int64_t B, int64_t H, int64_t N, int64_t D,
                              float scale, void* stream);

/*
 * Fused bool -> bit packing plus occupancy map.  Writes `packed` exactly as
 * sma_pack_mask does and `occupancy`: uint32 [B*H, ceil(N/128), 2], where bit t
 * of the pair for (batch*head, query tile qt) is set iff key tile t (keys
 * 128t .. 128t+127) has a set mask bit in query rows 128qt .. 128qt+127.
 * Needs N % 32 == 0, N <= SMA_MAX_SEQ_LEN_OCCUPANCY, a 16-byte aligned mask and 4-byte
 * aligned outputs (SMA_ERR_ARG / SMA_ERR_UNSUPPORTED_N otherwise; callers
 * then use sma_pack_mask).  The packer reads every mask byte anyway, so the
 * map costs no extra HBM pass.
 * No reference counterpart: the reference's attention re-tests every mask bit.
 */
SMA_API int sma_pack_mask_occupancy(const void* mask, void* packed, void* occupancy, int64_t B, int64_t H,
                                    int64_t N, void* stream);

/*
 * sma_attn_fwd with the occupancy map written by sma_pack_mask_occupancy for
 * the same mask: the head-dim-64 kernel takes its live key tiles from the
 * map instead of scanning the packed rows; results are identical to
 * sma_attn_fwd.  (The map describes 128-key tiles; head dim 128 works on
 * 64-key tiles, scans the packed rows and ignores it.)
 * No reference counterpart.
 */
SMA_API int sma_attn_fwd_occupancy(int dtype, const void* q, const void* k, const void* v, const void* mask_packed,
                                   const void* occupancy, void* out, float* lse, int64_t B, int64_t H, int64_t N,
                                   int64_t D, float scale, void* stream);

/*
 * Masked-softmax attention backward (head dims 64 and 128): given the forward's
 * inputs, its out and lse (as written by sma_attn_fwd with a non-NULL lse)
 * and the upstream gradient dout, writes dq, dk, dv ([B, H, N, D] of `dtype`):
 *   P = exp(scale * q k^T - lse) where the mask bit is set, else 0
 *   dv = P^T dout;  dS = P * (dout v^T - rowsum(dout * out));
 *   dq = scale * dS k;  dk = scale * dS^T q
 * dq_accum (FP32 [B, H, N, D]) and delta (FP32 [B, H, N]) are caller-provided
 * scratch.  Rows with no set bit get dq = 0; keys no row attends get dk = dv = 0.
 * Needs D in {64, 128}, 16-byte aligned q/k/v/out/dout/dq/dk/dv/dq_accum.
 *
 * Replaces: sparse_attn_cuda.backward(dout, q, k, v, out, lse, mask_packed,
 *           dq, dk, dv, scale), called by python/sparse_attention.py:93-96 but
 *           never bound by csrc/binding.cpp; the result follows the
 *           reference's CPU formulas (python/sparse_attention.py:97-111).
 */
SMA_API int sma_attn_bwd(int dtype, const void* q, const void* k, const void* v, const void* out, const void* dout,
                         const float* lse, const void* mask_packed, void* dq, void* dk, void* dv, float* dq_accum,
                         float* delta, int64_t B, int64_t H, int64_t N, int64_t D, float scale, void* stream);

/*
 * sma_attn_bwd with the FP32 scratch taken from a fixed 32 MiB device array
 * inside the library (one per device, found once per device with
 * cudaGetSymbolAddress): no memory is allocated and no allocating routine is
 * called.  Inputs whose B*H*N*(D+1) floats exceed the array return
 * SMA_ERR_ARG (dtype, head dim and sequence length are checked first, with
 * the codes of sma_attn_bwd).  Calls sharing a device share the array: order
 * them on one stream.  The 32 MiB are part of the library's module image, so
 * they are reserved on every device where the module is loaded, whether or
 * not this entry point is ever called.  No reference counterpart.
 */
SMA_API int sma_attn_bwd_noalloc(int dtype, const void* q, const void* k, const void* v, const void* out,
                                 const void* dout, const float* lse, const void* mask_packed, void* dq, void* dk,
                                 void* dv, int64_t B, int64_t H, int64_t N, int64_t D, float scale, void* stream);

/*
 * Synchronise `stream`, then report whether any kernel of this library on the
 * current device gave up a bounded device-side wait since the last clear
 * (SMA_ERR_TIMEOUT), or whether the stream holds a CUDA error (SMA_ERR_CUDA).
 * clear != 0 resets the device error word.
 * No reference counterpart (the reference never checks its launches).
 */
SMA_API int sma_device_status(void* stream, int clear);

/*
 * Upper bound, in nanoseconds, of every device-side wait in later launches
 * (default 2e9).  No reference counterpart.
 */
SMA_API int sma_set_wait_timeout_ns(uint64_t ns);

/*
 * Launch a one-CTA kernel that waits, through the library's bounded-wait
 * helper, on a barrier nothing ever signals; it gives up after timeout_ns and
 * raises the device error word.  Used to test failure reporting without
 * faulting or hanging a GPU.  No reference counterpart.
 */
SMA_API int sma_debug_wait_probe(uint64_t timeout_ns, void* stream);

/* Thread-local message for the last non-zero status. */
SMA_API const char* sma_last_error(void);

/* SMA_ABI_VERSION of the loaded library. */
SMA_API int sma_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* SMA_CAPI_H_ */
