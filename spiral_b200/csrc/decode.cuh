// decode.cuh — exact per-format decoders shared by the dequant kernels.
//
// Each helper produces 8 consecutive weights of one canonical block as four
// packed bf16x2 words (a uint4), value = bf16_rne(scale * integer) computed
// in fp32.  This is the B200 counterpart of the reference's per-tile
// dequantizers (src/quants/q4_0/unpack.aie.h:31-46,
// q8_0/unpack.aie.h:18-52, q6_k/unpack.aie.h:81-138), which build the same
// exact product from multi-term bf16 scale splits; fp32 is native here, so a
// single exact multiply replaces the split.
#pragma once

#include "common.cuh"

namespace spiral {

// ---- Q4_0 ----------------------------------------------------------------
// qs8 = the 8 qs bytes [8*(part&1), +8) as two little-endian words; `high`
// selects the high nibbles (weights 16..31 of the block).  h: the fp16 scale
// bits (after any flush).  Each nibble becomes u = 1024 + q in an fp16 half
// (one LOP3 per two), t = u - 1032 = q - 8 exactly, and t * d is one exact
// product (zero signs as the reference's (q - 8) * d).
__device__ __forceinline__ uint4 q4_0_decode8(uint32_t w0, uint32_t w1, bool high, unsigned short h) {
  if (high) {
    w0 >>= 4;
    w1 >>= 4;
  }
  constexpr uint32_t kB = 0x64086408u;  // 1032, 1032
  const uint32_t a02 = hsub2(lop_and_or(w0, 0x000F000Fu, 0x64006400u), kB);
  const uint32_t a13 = hsub2(lop_and_or(w0 >> 8, 0x000F000Fu, 0x64006400u), kB);
  const uint32_t b02 = hsub2(lop_and_or(w1, 0x000F000Fu, 0x64006400u), kB);
  const uint32_t b13 = hsub2(lop_and_or(w1 >> 8, 0x000F000Fu, 0x64006400u), kB);
  return make_uint4(h2mul_lo(a02, a13, h), h2mul_hi(a02, a13, h), h2mul_lo(b02, b13, h), h2mul_hi(b02, b13, h));
}

// ---- Q8_0 ----------------------------------------------------------------
// 8 int8 quants as two words; each byte with its sign bit flipped becomes
// u = 1024 + (q + 128), t = u - 1152 = q exactly, then t * d.
__device__ __forceinline__ uint4 q8_0_decode8(uint32_t w0, uint32_t w1, unsigned short h) {
  constexpr uint32_t kB = 0x64806480u;  // 1152, 1152
  const uint32_t a02 = hsub2(lop_and_xor(w0, 0x00FF00FFu, 0x64806480u), kB);
  const uint32_t a13 = hsub2(lop_and_xor(w0 >> 8, 0x00FF00FFu, 0x64806480u), kB);
  const uint32_t b02 = hsub2(lop_and_xor(w1, 0x00FF00FFu, 0x64806480u), kB);
  const uint32_t b13 = hsub2(lop_and_xor(w1 >> 8, 0x00FF00FFu, 0x64806480u), kB);
  return make_uint4(h2mul_lo(a02, a13, h), h2mul_hi(a02, a13, h), h2mul_lo(b02, b13, h), h2mul_hi(b02, b13, h));
}

// ---- Q6_K ----------------------------------------------------------------
// Assemble four 6-bit quants (as bytes 0..63) for sub-group s from the ql
// word of that s (low nibbles for s<2, high for s>=2) and the qh word.
__device__ __forceinline__ uint32_t q6_k_assemble4(uint32_t ql, uint32_t qh, int s) {
  const uint32_t lo = (ql >> (4 * (s >> 1))) & 0x0F0F0F0Fu;
  const uint32_t hi = ((qh >> (2 * s)) & 0x03030303u) << 4;
  return lo | hi;
}
// Four assembled quants times ds = d*sc (exact fp32), as two bf16x2 words.
__device__ __forceinline__ uint2 q6_k_scale4(uint32_t q4, float ds) {
  constexpr float kBias = 8388640.0f;  // 2^23 + 32
  uint2 r;
  r.x = pack_bf16x2((byte_as_f32_magic<0>(q4) - kBias) * ds, (byte_as_f32_magic<1>(q4) - kBias) * ds);
  r.y = pack_bf16x2((byte_as_f32_magic<2>(q4) - kBias) * ds, (byte_as_f32_magic<3>(q4) - kBias) * ds);
  return r;
}

// Generic 8-weight decoder reading a block with 2-byte granularity from any
// address space (used by the scalar-load fallback and the tile-order kernel).
// `blk` points at the block start; `k8` is the 8-weight chunk index within
// the block (0..3 for Q4_0/Q8_0, 0..31 for Q6_K).
__device__ __forceinline__ uint32_t ld_u16_any(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}
__device__ __forceinline__ uint32_t ld_u32_2aligned(const uint8_t* p) {
  return ld_u16_any(p) | (ld_u16_any(p + 2) << 16);
}

template <int FMT>
__device__ __forceinline__ uint4 decode8_generic(const uint8_t* blk, int k8, bool ftz);

template <>
__device__ __forceinline__ uint4 decode8_generic<kQ4_0>(const uint8_t* blk, int k8, bool ftz) {
  const unsigned short h = fp16_scale_bits(ld_u16_any(blk), ftz);
  const uint8_t* qs = blk + 2 + 8 * (k8 & 1);
  return q4_0_decode8(ld_u32_2aligned(qs), ld_u32_2aligned(qs + 4), k8 >= 2, h);
}
template <>
__device__ __forceinline__ uint4 decode8_generic<kQ8_0>(const uint8_t* blk, int k8, bool ftz) {
  const unsigned short h = fp16_scale_bits(ld_u16_any(blk), ftz);
  const uint8_t* qs = blk + 2 + 8 * k8;
  return q8_0_decode8(ld_u32_2aligned(qs), ld_u32_2aligned(qs + 4), h);
}
template <>
__device__ __forceinline__ uint4 decode8_generic<kQ6_K>(const uint8_t* blk, int k8, bool ftz) {
  // weights y = 8*k8 .. +7: y = 128h + 32s + l, l0 = y % 32 (multiple of 8).
  const int y0 = 8 * k8;
  const int h = y0 >> 7, s = (y0 >> 5) & 3, l0 = y0 & 31;
  const float d = fp16_bits_to_f32(ld_u16_any(blk + 208), ftz);
  const float ds = d * static_cast<float>(static_cast<int8_t>(blk[192 + 8 * h + 2 * s + (l0 >> 4)]));
  const uint8_t* ql = blk + 64 * h + 32 * (s & 1) + l0;
  const uint8_t* qh = blk + 128 + 32 * h + l0;
  const uint2 a = q6_k_scale4(q6_k_assemble4(ld_u32_2aligned(ql), ld_u32_2aligned(qh), s), ds);
  const uint2 b = q6_k_scale4(q6_k_assemble4(ld_u32_2aligned(ql + 4), ld_u32_2aligned(qh + 4), s), ds);
  return make_uint4(a.x, a.y, b.x, b.y);
}

}  // namespace spiral
