// chunk_decode.cuh — exact register-level block decoders that feed tensor
// memory (tcgen05 A operands) in natural k order.
//
// Input: a register image R of 16-byte shared-memory loads; a block starts at
// byte O of that image (O even, compile-time).  Output: the block's 32
// weights as 16 bf16x2 words, word i = weights (2i, 2i+1), exactly
// bf16_rne(d * (q - bias)) — the reference oracle's value
// (src/quants/tests/formats/q4_0.py:47-60, q8_0.py:43-60) up to the sign of a
// zero weight, which no dot product can see.
//
// A quant byte goes into an fp32 mantissa with one byte permute
// (f = 1 + byte * 2^-15, or 1 + 16q * 2^-15 = 1 + q * 2^-11 for a high
// nibble kept in place) and one exact fma.rn.f32x2 computes
// f * (2^s d) - (2^s + bias) d = (q - bias) d for a pair; both constants are
// exact in fp32, so only the final cvt.rn.bf16x2.f32 rounds.
#pragma once

#include "common.cuh"

namespace spiral {

__device__ __forceinline__ uint32_t fma2_pack_bf16(uint32_t fa, uint32_t fb, uint64_t D2, uint64_t C2) {
  const uint64_t in = (static_cast<uint64_t>(fb) << 32) | fa;
  uint64_t out;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(out) : "l"(in), "l"(D2), "l"(C2));
  return pack_bf16x2(__uint_as_float(static_cast<uint32_t>(out)), __uint_as_float(static_cast<uint32_t>(out >> 32)));
}
__device__ __forceinline__ uint64_t dup2f(float v) {
  const uint64_t b = __float_as_uint(v);
  return (b << 32) | b;
}
template <int I>
__device__ __forceinline__ uint32_t b2f1(uint32_t w) {
  return __byte_perm(w, 0x3F800000u, 0x7604u | (I << 4));
}
// Bytes [o, o+4) of a register image of 16-byte loads, o even.
template <int O>
__device__ __forceinline__ uint32_t word_at(const uint32_t* R) {
  if constexpr ((O & 3) == 0) {
    return R[O >> 2];
  } else {
    return __funnelshift_r(R[O >> 2], R[(O >> 2) + 1], 16);
  }
}
template <int O>
__device__ __forceinline__ uint32_t half_at(const uint32_t* R) {
  return (R[O >> 2] >> ((O & 3) * 8)) & 0xFFFFu;
}

template <int FMT>
struct BlockDecoder;

// Q4_0 block at O: fp16 d, then qs[16]; weight j < 16 = qs[j] & 15,
// j >= 16 = qs[j-16] >> 4; value (q - 8) d.
template <>
struct BlockDecoder<kQ4_0> {
  template <int O>
  __device__ __forceinline__ static void block(const uint32_t* R, bool ftz, uint32_t (&out)[16]) {
    const float d = fp16_bits_to_f32(half_at<O>(R), ftz);
    const uint64_t DL = dup2f(d * 32768.0f), CL = dup2f(d * -32776.0f);  // 2^15 + 8 = 8 * 4097
    const uint64_t DH = dup2f(d * 2048.0f), CH = dup2f(d * -2056.0f);    // 2^11 + 8 = 8 * 257
    const uint32_t q[4] = {word_at<O + 2>(R), word_at<O + 6>(R), word_at<O + 10>(R), word_at<O + 14>(R)};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t L = q[i] & 0x0F0F0F0Fu, Hn = q[i] & 0xF0F0F0F0u;
      out[2 * i] = fma2_pack_bf16(b2f1<0>(L), b2f1<1>(L), DL, CL);        // weights 4i, 4i+1
      out[2 * i + 1] = fma2_pack_bf16(b2f1<2>(L), b2f1<3>(L), DL, CL);    // 4i+2, 4i+3
      out[8 + 2 * i] = fma2_pack_bf16(b2f1<0>(Hn), b2f1<1>(Hn), DH, CH);  // 16+4i, 16+4i+1
      out[9 + 2 * i] = fma2_pack_bf16(b2f1<2>(Hn), b2f1<3>(Hn), DH, CH);
    }
  }
};

// Q8_0 block at O: fp16 d, then 32 int8; value q d.  Bytes are biased to
// unsigned (x ^ 0x80) and 2^15 + 128 = 128 * 257 removes the bias exactly.
template <>
struct BlockDecoder<kQ8_0> {
  template <int O>
  __device__ __forceinline__ static void block(const uint32_t* R, bool ftz, uint32_t (&out)[16]) {
    const float d = fp16_bits_to_f32(half_at<O>(R), ftz);
    const uint64_t D = dup2f(d * 32768.0f), C = dup2f(d * -32896.0f);
    const uint32_t q[8] = {word_at<O + 2>(R),  word_at<O + 6>(R),  word_at<O + 10>(R), word_at<O + 14>(R),
                           word_at<O + 18>(R), word_at<O + 22>(R), word_at<O + 26>(R), word_at<O + 30>(R)};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t u = q[i] ^ 0x80808080u;
      out[2 * i] = fma2_pack_bf16(b2f1<0>(u), b2f1<1>(u), D, C);
      out[2 * i + 1] = fma2_pack_bf16(b2f1<2>(u), b2f1<3>(u), D, C);
    }
  }
};

}  // namespace spiral
