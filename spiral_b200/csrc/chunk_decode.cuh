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

// Q6_K super-block half H (weights 128H .. 128H+127) for one feature row,
// read straight from global memory.  The super-block starts P bytes past a
// 16-byte boundary (P even; 210-byte blocks in 16-byte aligned rows), so the
// loads are 16-byte aligned windows and every field offset is compile-time:
//   ql[64H .. 64H+64)  -> window bytes [64H, 64H+80),  5 loads
//   qh[32H .. 32H+32)  -> [128+32H, 176+32H),           3 loads
//   sc[8H .. 8H+8), d  -> [192, 224),                   2 loads
// (relative to the super-block start minus P).  The windows may run up to 14
// bytes past the super-block; with rows a multiple of 8 super-blocks the last
// super-block of a row has P = 14 and every window ends inside the row.
// Output: 4 sub-blocks s (weights 128H + 32s + l, l < 32) as 16 bf16x2 words
// each, weight (q6 - 32) * (d * sc[8H + 2s + l/16]) with
// q6 = (ql[64H + 32(s&1) + l] >> 4(s>>1)) & 15 | ((qh[32H + l] >> 2s) & 3) << 4
// (src/quants/tests/formats/q6_k.py:55-97).  With bit 7 set the byte lands in
// an fp32 mantissa as f = 1 + q6 * 2^-7, and f * (128 ds) - 160 ds =
// (q6 - 32) ds exactly (ds = d * sc has at most 18 significant bits).
template <int P, int H>
struct Q6KHalf {
  template <int O>
  __device__ __forceinline__ static uint32_t byte_at(const uint32_t* R) {
    return (R[O >> 2] >> ((O & 3) * 8)) & 0xFFu;
  }
  template <int I>
  __device__ __forceinline__ static uint32_t b2f2(uint32_t w) {
    return __byte_perm(w, 0x3F000000u, 0x7054u | (I << 8));
  }
  // Emits the half's 4 sub-blocks through store(j, out[16]).
  template <typename Store>
  __device__ __forceinline__ static void run(const uint8_t* sb, bool ftz, Store&& store) {
    const uint8_t* win = sb - P;
    uint32_t Rl[20], Rh[12], Rs[8];
    const uint4* pl = reinterpret_cast<const uint4*>(win + 64 * H);
    const uint4* ph = reinterpret_cast<const uint4*>(win + 128 + 32 * H);
    const uint4* ps = reinterpret_cast<const uint4*>(win + 192);
#pragma unroll
    for (int i = 0; i < 5; ++i) {
      const uint4 v = __ldg(pl + i);
      Rl[4 * i] = v.x; Rl[4 * i + 1] = v.y; Rl[4 * i + 2] = v.z; Rl[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const uint4 v = __ldg(ph + i);
      Rh[4 * i] = v.x; Rh[4 * i + 1] = v.y; Rh[4 * i + 2] = v.z; Rh[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 v = __ldg(ps + i);
      Rs[4 * i] = v.x; Rs[4 * i + 1] = v.y; Rs[4 * i + 2] = v.z; Rs[4 * i + 3] = v.w;
    }
    const float d = fp16_bits_to_f32(half_at<P + 16>(Rs), ftz);
    sub<0>(Rl, Rh, Rs, d, store);
    sub<1>(Rl, Rh, Rs, d, store);
    sub<2>(Rl, Rh, Rs, d, store);
    sub<3>(Rl, Rh, Rs, d, store);
  }
  template <int S, typename Store>
  __device__ __forceinline__ static void sub(const uint32_t* Rl, const uint32_t* Rh, const uint32_t* Rs, float d,
                                             Store& store) {
    const float ds0 = d * static_cast<float>(static_cast<int8_t>(byte_at<P + 8 * H + 2 * S>(Rs)));
    const float ds1 = d * static_cast<float>(static_cast<int8_t>(byte_at<P + 8 * H + 2 * S + 1>(Rs)));
    const uint64_t D0 = dup2f(ds0 * 128.0f), C0 = dup2f(ds0 * -160.0f);
    const uint64_t D1 = dup2f(ds1 * 128.0f), C1 = dup2f(ds1 * -160.0f);
    uint32_t out[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t ql, qh;
      switch (i) {  // compile-time offsets
        case 0: ql = word_at<P + 32 * (S & 1) + 0>(Rl); qh = word_at<P + 0>(Rh); break;
        case 1: ql = word_at<P + 32 * (S & 1) + 4>(Rl); qh = word_at<P + 4>(Rh); break;
        case 2: ql = word_at<P + 32 * (S & 1) + 8>(Rl); qh = word_at<P + 8>(Rh); break;
        case 3: ql = word_at<P + 32 * (S & 1) + 12>(Rl); qh = word_at<P + 12>(Rh); break;
        case 4: ql = word_at<P + 32 * (S & 1) + 16>(Rl); qh = word_at<P + 16>(Rh); break;
        case 5: ql = word_at<P + 32 * (S & 1) + 20>(Rl); qh = word_at<P + 20>(Rh); break;
        case 6: ql = word_at<P + 32 * (S & 1) + 24>(Rl); qh = word_at<P + 24>(Rh); break;
        default: ql = word_at<P + 32 * (S & 1) + 28>(Rl); qh = word_at<P + 28>(Rh); break;
      }
      const uint32_t q = ((ql >> (4 * (S >> 1))) & 0x0F0F0F0Fu) | (((qh >> (2 * S)) & 0x03030303u) << 4) | 0x80808080u;
      const uint64_t D = i < 4 ? D0 : D1, C = i < 4 ? C0 : C1;
      out[2 * i] = fma2_pack_bf16(b2f2<0>(q), b2f2<1>(q), D, C);
      out[2 * i + 1] = fma2_pack_bf16(b2f2<2>(q), b2f2<3>(q), D, C);
    }
    store(S, out);
  }
};

}  // namespace spiral
