// gemv_decode.cuh — register-level decoders that feed mma.sync.m16n8k16 A
// fragments straight from canonical GGUF blocks in shared memory, shared by
// the decode GEMV (gemv.cu, gemv_xs.cu) and the MoE expert GEMVs (moe.cu).
//
// Dequantization is exact, by one of two routes.
//  * Q4_0 / Q8_0 (fp16 route): one LOP3 puts two quants into the mantissas of
//    an fp16 pair, u = 2^e + q (q a nibble at bits 0-3 with 0x6400 = 1024, a
//    nibble at bits 4-7 with 0x5400 = 64 (mantissa unit 2^-4), or a byte with
//    its sign bit flipped at bits 0-7 with 0x6400); one mixed-precision
//    fma.rn.f32.f16 per weight computes u*d - (2^e + bias)*d with the fp16
//    scale d itself as the other operand.  The product u*d is exact inside
//    the FMA, the bias product (2^e + bias)*d has at most 19 significant bits
//    and the result (q - bias)*d at most 19, so the FMA does not round.
//  * Q6_K (fp32 route): a 6-bit quant with bit 7 set goes into an fp32
//    mantissa with one byte permute, f = 1 + q*2^-7, and one fma.rn.f32x2
//    per pair computes f*(128 ds) - 160 ds with ds = d*sc (at most 19 bits):
//    exact again.  (ds does not fit an fp16 operand.)
// cvt.rn.bf16x2.f32 then rounds once to nearest even, so the A fragments hold
// exactly the bf16 weights of the standalone dequant (bf16_rne(d*int), up to
// the sign of a zero weight, which cannot change a dot product).  The fp16
// route costs 10 integer-pipe instructions per MMA against 15 for a byte
// permute per weight, which matters because the decode, not HBM, bounds
// these kernels.
#pragma once

#include "common.cuh"

namespace spiral {

template <int FMT> struct GemvFmt;
// kGroupK weights per group (the unit a consumer warp decodes); kSteps MMA
// k-steps per group; a chunk must be a multiple of kChunkAlign groups to stay
// 16-byte aligned.
template <> struct GemvFmt<kQ4_0> {
  static constexpr int kGroupK = 128, kGroupBytes = 72, kSteps = 8, kChunkAlign = 2, kMaxStages = 8;
};
template <> struct GemvFmt<kQ8_0> {
  static constexpr int kGroupK = 128, kGroupBytes = 136, kSteps = 8, kChunkAlign = 2, kMaxStages = 8;
};
template <> struct GemvFmt<kQ6_K> {
  static constexpr int kGroupK = 256, kGroupBytes = 210, kSteps = 16, kChunkAlign = 8, kMaxStages = 8;
};

// ------------------------------------------------------------- helpers ---


__device__ __forceinline__ void mma_bf16_16816(float (&acc)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// Two fp32 bit patterns through one exact fma.rn.f32x2 with (D, C), then one
// RNE pack to bf16x2 (fa in the low half).
__device__ __forceinline__ uint32_t fma2_pack(uint32_t fa, uint32_t fb, uint64_t D2, uint64_t C2) {
  const uint64_t in = (static_cast<uint64_t>(fb) << 32) | fa;
  uint64_t out;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(out) : "l"(in), "l"(D2), "l"(C2));
  return pack_bf16x2(__uint_as_float(static_cast<uint32_t>(out)), __uint_as_float(static_cast<uint32_t>(out >> 32)));
}
__device__ __forceinline__ uint64_t dup2(float v) {
  const uint64_t b = __float_as_uint(v);
  return (b << 32) | b;
}

// Byte i of w (its bit 7 set) into bits 16..23 of 0x3F_00_00_00:
// f = 1 + (byte & 0x7f) * 2^-7.
template <int I>
__device__ __forceinline__ uint32_t byte_to_f2(uint32_t w) {
  return __byte_perm(w, 0x3F000000u, 0x7054u | (I << 8));
}

// --------------------------------------------- per-format group decoders --
// ra / rb: this lane's two feature rows (r and r + 8) at the group start in
// the stage (4-byte aligned for Q4_0/Q8_0, 2-byte for Q6_K); c = lane % 4;
// xg = this lane's B-fragment column at step 0 of the group in the permuted
// activations (stride 32 bytes per step).  xk(s, c) gives the k offset
// (within the group) of the 4 consecutive weights lane column c contracts at
// step s; the activation staging uses it to build the permuted copy.

template <int FMT>
struct GroupDecoder;

// Q4_0: lane c owns block c of the 4-block group (18 bytes at 18c).  Step
// 2j covers the low nibbles of qs word j (weights 4j..4j+3), step 2j+1 the
// high nibbles (weights 16+4j..16+4j+3).
template <>
struct GroupDecoder<kQ4_0> {
  __device__ __forceinline__ static void run(const uint8_t* ra, const uint8_t* rb, int c, const uint8_t* xg, bool ftz,
                                             float (&acc)[4]) {
    run_b(ra, rb, c, [xg](int s) { return *reinterpret_cast<const uint2*>(xg + 32 * s); }, ftz, acc);
  }
  // bx(s): this lane's B fragment of step s (the activations of xk(s, c)).
  template <class BX>
  __device__ __forceinline__ static void run_b(const uint8_t* ra, const uint8_t* rb, int c, BX&& bx, bool ftz,
                                               float (&acc)[4]) {
    // qs starts at 18c + 2: 4-byte aligned for odd c, 2 mod 4 for even c.
    const int woff = 18 * c + 2 * (c & 1);
    const uint32_t sh = (c & 1) ? 0u : 16u;
    uint32_t qa[4], qb[4];
    {
      uint32_t wa[5], wb[5];
#pragma unroll
      for (int i = 0; i < 5; ++i) {
        wa[i] = lds32(ra + woff + 4 * i);
        wb[i] = lds32(rb + woff + 4 * i);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        qa[j] = __funnelshift_r(wa[j], wa[j + 1], sh);
        qb[j] = __funnelshift_r(wb[j], wb[j + 1], sh);
      }
    }
    const unsigned short ha = fp16_scale_bits(lds_u16(ra + 18 * c), ftz);
    const unsigned short hb = fp16_scale_bits(lds_u16(rb + 18 * c), ftz);
    const float da = fp16_bits_to_f32(ha, false), db = fp16_bits_to_f32(hb, false);
    // low nibble: u = 1024 + q, bias 1032 = 8 * 129; high nibble (bits 4-7
    // under 0x5400): u = 64 + q, bias 72
    const float CLa = da * -1032.0f, CHa = da * -72.0f, CLb = db * -1032.0f, CHb = db * -72.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // bytes 0 and 2 of the word in u02, bytes 1 and 3 in u13
      const uint32_t a8 = qa[j] >> 8, b8 = qb[j] >> 8;
      const uint32_t la02 = lop_and_or(qa[j], 0x000F000Fu, 0x64006400u), la13 = lop_and_or(a8, 0x000F000Fu, 0x64006400u);
      const uint32_t lb02 = lop_and_or(qb[j], 0x000F000Fu, 0x64006400u), lb13 = lop_and_or(b8, 0x000F000Fu, 0x64006400u);
      const uint2 b0 = bx(2 * j);
      mma_bf16_16816(acc, h2pack_lo(la02, la13, ha, CLa), h2pack_lo(lb02, lb13, hb, CLb), h2pack_hi(la02, la13, ha, CLa),
                     h2pack_hi(lb02, lb13, hb, CLb), b0.x, b0.y);
      const uint32_t ua02 = lop_and_or(qa[j], 0x00F000F0u, 0x54005400u), ua13 = lop_and_or(a8, 0x00F000F0u, 0x54005400u);
      const uint32_t ub02 = lop_and_or(qb[j], 0x00F000F0u, 0x54005400u), ub13 = lop_and_or(b8, 0x00F000F0u, 0x54005400u);
      const uint2 b1 = bx(2 * j + 1);
      mma_bf16_16816(acc, h2pack_lo(ua02, ua13, ha, CHa), h2pack_lo(ub02, ub13, hb, CHb), h2pack_hi(ua02, ua13, ha, CHa),
                     h2pack_hi(ub02, ub13, hb, CHb), b1.x, b1.y);
    }
  }
  __host__ __device__ __forceinline__ static int xk(int s, int c) { return 32 * c + 16 * (s & 1) + 4 * (s >> 1); }
};

// Q8_0: lane c owns block c (34 bytes at 34c); step s = weights 4s..4s+3.
template <>
struct GroupDecoder<kQ8_0> {
  __device__ __forceinline__ static void run(const uint8_t* ra, const uint8_t* rb, int c, const uint8_t* xg, bool ftz,
                                             float (&acc)[4]) {
    run_b(ra, rb, c, [xg](int s) { return *reinterpret_cast<const uint2*>(xg + 32 * s); }, ftz, acc);
  }
  template <class BX>
  __device__ __forceinline__ static void run_b(const uint8_t* ra, const uint8_t* rb, int c, BX&& bx, bool ftz,
                                               float (&acc)[4]) {
    const int woff = 34 * c + 2 * (c & 1);
    const uint32_t sh = (c & 1) ? 0u : 16u;
    // u = 1024 + (q + 128) (the byte with its sign bit flipped), bias 1152 = 128 * 9
    const unsigned short ha = fp16_scale_bits(lds_u16(ra + 34 * c), ftz);
    const unsigned short hb = fp16_scale_bits(lds_u16(rb + 34 * c), ftz);
    const float Ca = fp16_bits_to_f32(ha, false) * -1152.0f, Cb = fp16_bits_to_f32(hb, false) * -1152.0f;
    uint32_t pa = lds32(ra + woff), pb = lds32(rb + woff);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const uint32_t na = lds32(ra + woff + 4 * (s + 1)), nb = lds32(rb + woff + 4 * (s + 1));
      const uint32_t qa = __funnelshift_r(pa, na, sh), qb = __funnelshift_r(pb, nb, sh);
      pa = na;
      pb = nb;
      const uint32_t a02 = lop_and_xor(qa, 0x00FF00FFu, 0x64806480u), a13 = lop_and_xor(qa >> 8, 0x00FF00FFu, 0x64806480u);
      const uint32_t b02 = lop_and_xor(qb, 0x00FF00FFu, 0x64806480u), b13 = lop_and_xor(qb >> 8, 0x00FF00FFu, 0x64806480u);
      const uint2 b = bx(s);
      mma_bf16_16816(acc, h2pack_lo(a02, a13, ha, Ca), h2pack_lo(b02, b13, hb, Cb), h2pack_hi(a02, a13, ha, Ca),
                     h2pack_hi(b02, b13, hb, Cb), b.x, b.y);
    }
  }
  __host__ __device__ __forceinline__ static int xk(int s, int c) { return 32 * c + 4 * s; }
};

// Q6_K: one super-block per group; lane c owns l in [8c, 8c+8) of both
// halves.  Step t = 8h + 4*half + s covers y = 128h + 32s + 8c + 4*half + 0..3.
// The 6-bit quant with bit 7 set gives f = 1 + q6 2^-7;
// f*(128 ds) - 160 ds = (q6 - 32) ds with ds = d*sc (exact, <= 18 bits).
template <>
struct GroupDecoder<kQ6_K> {
  // 8 bytes at p (p % 4 == sh/8 for a 2-byte aligned super-block start).
  __device__ __forceinline__ static void load8(const uint8_t* p, uint32_t sh, uint32_t& lo, uint32_t& hi) {
    const uint8_t* a = p - (sh >> 3);
    const uint32_t w0 = lds32(a), w1 = lds32(a + 4), w2 = lds32(a + 8);
    lo = __funnelshift_r(w0, w1, sh);
    hi = __funnelshift_r(w1, w2, sh);
  }
  __device__ __forceinline__ static uint32_t assemble(uint32_t ql, uint32_t qh, int s) {
    const uint32_t lo = (s >= 2 ? (ql >> 4) : ql) & 0x0F0F0F0Fu;
    const uint32_t hb = (s == 0 ? (qh << 4) : s == 1 ? (qh << 2) : s == 2 ? qh : (qh >> 2)) & 0x30303030u;
    return lo | hb | 0x80808080u;
  }
  __device__ __forceinline__ static void run(const uint8_t* ra, const uint8_t* rb, int c, const uint8_t* xg, bool ftz,
                                             float (&acc)[4], uint32_t sh) {
    run_b(ra, rb, c, [xg](int t) { return *reinterpret_cast<const uint2*>(xg + 32 * t); }, ftz, acc, sh);
  }
  template <class BX>
  __device__ __forceinline__ static void run_b(const uint8_t* ra, const uint8_t* rb, int c, BX&& bx, bool ftz,
                                               float (&acc)[4], uint32_t sh) {
    const float da = fp16_bits_to_f32(lds_u16(ra + 208), ftz);
    const float db = fp16_bits_to_f32(lds_u16(rb + 208), ftz);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint64_t Da[4], Ca[4], Db[4], Cb[4];
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int si = 192 + 8 * h + 2 * s + (c >> 1);
        const float dsa = da * static_cast<float>(static_cast<int8_t>(ra[si]));
        const float dsb = db * static_cast<float>(static_cast<int8_t>(rb[si]));
        Da[s] = dup2(dsa * 128.0f);
        Ca[s] = dup2(dsa * -160.0f);
        Db[s] = dup2(dsb * 128.0f);
        Cb[s] = dup2(dsb * -160.0f);
      }
      uint32_t qla[2], qlb[2], qha[2], qla_b[2], qlb_b[2], qh_b[2];
      load8(ra + 64 * h + 8 * c, sh, qla[0], qla[1]);
      load8(ra + 64 * h + 32 + 8 * c, sh, qlb[0], qlb[1]);
      load8(ra + 128 + 32 * h + 8 * c, sh, qha[0], qha[1]);
      load8(rb + 64 * h + 8 * c, sh, qla_b[0], qla_b[1]);
      load8(rb + 64 * h + 32 + 8 * c, sh, qlb_b[0], qlb_b[1]);
      load8(rb + 128 + 32 * h + 8 * c, sh, qh_b[0], qh_b[1]);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint32_t qa = assemble((s & 1) ? qlb[half] : qla[half], qha[half], s);
          const uint32_t qb = assemble((s & 1) ? qlb_b[half] : qla_b[half], qh_b[half], s);
          const uint2 b = bx(8 * h + 4 * half + s);
          mma_bf16_16816(acc, fma2_pack(byte_to_f2<0>(qa), byte_to_f2<1>(qa), Da[s], Ca[s]),
                         fma2_pack(byte_to_f2<0>(qb), byte_to_f2<1>(qb), Db[s], Cb[s]),
                         fma2_pack(byte_to_f2<2>(qa), byte_to_f2<3>(qa), Da[s], Ca[s]),
                         fma2_pack(byte_to_f2<2>(qb), byte_to_f2<3>(qb), Db[s], Cb[s]), b.x, b.y);
        }
      }
    }
  }
  __host__ __device__ __forceinline__ static int xk(int t, int c) {
    const int h = t >> 3, half = (t >> 2) & 1, s = t & 3;
    return 128 * h + 32 * s + 8 * c + 4 * half;
  }
};

}  // namespace spiral
