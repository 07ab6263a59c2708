// Bool-mask bytes -> packed bits, shared by the mask packer (pack_mask.cu)
// and the attention kernel that reads the bool mask itself (attn_fwd_chain.cu).
//
// Bit b of an output word is the byte at column b of its 32 columns; any
// non-zero byte counts as set (the reference packer's `mask[...] ? 1 : 0`,
// csrc/sparse_attention.cu:20-42).
#pragma once

#include <cstdint>

namespace sma {

// 4 mask bytes -> 4 bits (byte k -> bit k), any non-zero byte set.
__device__ __forceinline__ uint32_t pack4_any(uint32_t x) {
  // High bit of each byte := byte != 0 (no carries cross byte lanes).
  const uint32_t hi = (((x & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | x) & 0x80808080u;
  // Gather the four high bits into bits 28..31 with one multiply.
  return (hi * 0x00204081u) >> 28;
}

// 16 mask bytes -> 16 bits, any non-zero byte set.
__device__ __forceinline__ uint32_t pack16_any(uint4 v) {
  return pack4_any(v.x) | (pack4_any(v.y) << 4) | (pack4_any(v.z) << 8) | (pack4_any(v.w) << 12);
}

// 16 mask bytes that are all 0 or 1 -> 16 bits (low half of the result).
// x * 0x01020408 moves byte k's bit 8k to bit 24 + k; no two partial products
// share a bit position, so nothing carries and bits 24..27 are exactly the
// four bytes.  Byte 3 of the four products is then gathered two at a time.
__device__ __forceinline__ uint32_t pack16_01(uint4 v) {
  constexpr uint32_t kM = 0x01020408u;
  const uint32_t a = v.x * kM, b = v.y * kM, c = v.z * kM, d = v.w * kM;
  const uint32_t ac = __byte_perm(a, c, 0x7373u);  // byte 0: bits of v.x, byte 1: bits of v.z
  const uint32_t bd = __byte_perm(b, d, 0x7373u);  // byte 0: bits of v.y, byte 1: bits of v.w
  return ac + (bd << 4);                           // nibbles never overlap: + is |
}

// True when every byte of the 32 is 0 or 1 (the bytes torch writes for bool).
__device__ __forceinline__ bool bytes_are_01(const uint4& lo, const uint4& hi) {
  return ((lo.x | lo.y | lo.z | lo.w | hi.x | hi.y | hi.z | hi.w) & 0xFEFEFEFEu) == 0u;
}

// 32 mask bytes (two 16-byte halves) -> one packed word.
__device__ __forceinline__ uint32_t pack32_01(const uint4& lo, const uint4& hi) {
  return __byte_perm(pack16_01(lo), pack16_01(hi), 0x5410u);
}
__device__ __forceinline__ uint32_t pack32_any(const uint4& lo, const uint4& hi) {
  return pack16_any(lo) | (pack16_any(hi) << 16);
}

}  // namespace sma
