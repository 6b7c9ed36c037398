// decode_ext.cuh — exact 8-weight decoders for the extended GGUF formats
// (Q4_K, Q5_K, IQ4_NL, IQ4_XS, F16, BF16), as decode8_generic
// specializations: weights [8*k8, 8*k8 + 8) of one block as four packed
// bf16x2 words.
//
// The reference names these formats as its next step (src/quants/TODO.md:
// 16-22) without code; the block layouts and the arithmetic follow ggml's
// published definitions (block_q4_K / block_q5_K / block_iq4_nl /
// block_iq4_xs, dequantize_row_*): one IEEE float32 rounding per operation in
// ggml's order, then one bf16 RNE rounding.  The float32 operations are the
// non-contracting intrinsics (__fmul_rn, __fsub_rn), so the compiler cannot
// fuse d1*q - m1 into one FMA and change the rounding.
#pragma once

#include "decode.cuh"

namespace spiral {

// (scale, min) of sub-block j (0..7) from the 12 packed bytes of a K-quant
// super-block: 6 bits each, the high two bits of sub-blocks 4..7 stored in
// the top bits of bytes 0..7 (ggml get_scale_min_k4).
__device__ __forceinline__ void kquant_scale_min(const uint8_t* sc12, int j, int& sc, int& m) {
  if (j < 4) {
    sc = sc12[j] & 63;
    m = sc12[j + 4] & 63;
  } else {
    sc = (sc12[j + 4] & 0xF) | ((sc12[j - 4] >> 6) << 4);
    m = (sc12[j + 4] >> 4) | ((sc12[j] >> 6) << 4);
  }
}

// K-quant: weights y0..y0+7 (y0 = 8*k8) lie in 64-weight chunk i = y0/64,
// half h = (y0/32)&1 (low / high nibbles of the chunk's 32 bytes), sub-block
// j = 2i + h; y = (d*sc_j) * q - (dmin*m_j), both products exact.
template <bool Q5>
__device__ __forceinline__ uint4 kquant_decode8(const uint8_t* blk, int k8, bool ftz) {
  const int y0 = 8 * k8, i = y0 >> 6, h = (y0 >> 5) & 1, l0 = y0 & 31, j = 2 * i + h;
  const float d = fp16_bits_to_f32(ld_u16_any(blk), ftz);
  const float dmin = fp16_bits_to_f32(ld_u16_any(blk + 2), ftz);
  int sc, m;
  kquant_scale_min(blk + 4, j, sc, m);
  const float d1 = __fmul_rn(d, static_cast<float>(sc));
  const float m1 = __fmul_rn(dmin, static_cast<float>(m));
  const uint8_t* qs = blk + (Q5 ? 48 : 16) + 32 * i + l0;
  float v[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    int q = (qs[t] >> (4 * h)) & 0xF;
    if constexpr (Q5) q += ((blk[16 + l0 + t] >> j) & 1) << 4;
    v[t] = __fsub_rn(__fmul_rn(d1, static_cast<float>(q)), m1);
  }
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

template <>
__device__ __forceinline__ uint4 decode8_generic<kQ4_K>(const uint8_t* blk, int k8, bool ftz) {
  return kquant_decode8<false>(blk, k8, ftz);
}
template <>
__device__ __forceinline__ uint4 decode8_generic<kQ5_K>(const uint8_t* blk, int k8, bool ftz) {
  return kquant_decode8<true>(blk, k8, ftz);
}

// The IQ4 codebook entry of nibble q (ggml kvalues_iq4nl), by two byte
// permutes over the table held in four immediates: no memory access.
__device__ __forceinline__ float iq4_value(uint32_t q) {
  // entries 0..7 and 8..15 as little-endian int8 bytes
  const uint32_t lo = __byte_perm(0xBFAD9881u, 0xF6EADDCFu, q & 7u);
  const uint32_t hi = __byte_perm(0x26190D01u, 0x71594535u, q & 7u);
  const uint32_t b = (q & 8u) ? hi : lo;
  return static_cast<float>(static_cast<int8_t>(b & 0xFFu));
}

template <>
__device__ __forceinline__ uint4 decode8_generic<kIQ4_NL>(const uint8_t* blk, int k8, bool ftz) {
  // weights 0..15: low nibbles of qs[0..16); 16..31: high nibbles
  const int y0 = 8 * k8, h = y0 >> 4, l0 = y0 & 15;
  const float d = fp16_bits_to_f32(ld_u16_any(blk), ftz);
  const uint8_t* qs = blk + 2 + l0;
  float v[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) v[t] = __fmul_rn(d, iq4_value((qs[t] >> (4 * h)) & 0xFu));
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

template <>
__device__ __forceinline__ uint4 decode8_generic<kIQ4_XS>(const uint8_t* blk, int k8, bool ftz) {
  // sub-block ib of 32 weights: 6-bit scale ls from scales_l (4 bits) and
  // scales_h (2 bits); weights 0..15 low nibbles of qs[16 ib ..], 16..31 high
  const int y0 = 8 * k8, ib = y0 >> 5, h = (y0 >> 4) & 1, l0 = y0 & 15;
  const float d = fp16_bits_to_f32(ld_u16_any(blk), ftz);
  const uint32_t scales_h = ld_u16_any(blk + 2);
  const int ls = ((blk[4 + (ib >> 1)] >> (4 * (ib & 1))) & 0xF) | (((scales_h >> (2 * ib)) & 3) << 4);
  const float dl = __fmul_rn(d, static_cast<float>(ls - 32));
  const uint8_t* qs = blk + 8 + 16 * ib + l0;
  float v[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) v[t] = __fmul_rn(dl, iq4_value((qs[t] >> (4 * h)) & 0xFu));
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

// F16: 8 halves (exact in fp32) rounded once to bf16.
template <>
__device__ __forceinline__ uint4 decode8_generic<kF16>(const uint8_t* blk, int, bool) {
  float v[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) v[t] = fp16_bits_to_f32(ld_u16_any(blk + 2 * t), false);
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

// BF16: the values themselves.
template <>
__device__ __forceinline__ uint4 decode8_generic<kBF16>(const uint8_t* blk, int, bool) {
  return make_uint4(ld_u32_2aligned(blk), ld_u32_2aligned(blk + 4), ld_u32_2aligned(blk + 8),
                    ld_u32_2aligned(blk + 12));
}

}  // namespace spiral
