// common.cuh — shared device helpers for the sm_100a quantized-weight kernels.
//
// Canonical GGUF block layouts (little-endian), as the reference pins them:
//   Q4_0: [fp16 d][16 B qs]; weight j<16 = qs[j]&15, j>=16 = qs[j-16]>>4,
//         value (q-8)*d                  (src/quants/q4_0/layout.h:10-16,
//                                          tests/formats/q4_0.py:47-60)
//   Q8_0: [fp16 d][32 x int8]; value q*d (q8_0/layout.h:10-13,
//                                          tests/formats/q8_0.py:43-60)
//   Q6_K: [ql 128][qh 64][int8 sc 16][fp16 d], 256 weights; for half h and
//         l < 32: y[128h+32s+l] = d*sc[8h+2s+l/16]*(q6-32) with q6 from
//         ql[64h+32(s&1)+l] (low nibble for s<2, high for s>=2) and two bits
//         (qh[32h+l] >> 2s) & 3 on top (q6_k/layout.h:10-15,
//                                          tests/formats/q6_k.py:55-97)
// Every product d*int (and d*sc*int) is exact in fp32 (at most 24 significant
// bits), so "fp32 multiply, one bf16 RNE rounding" reproduces the reference
// oracle's float32 product .astype(bfloat16) bit for bit.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace spiral {

enum : int { kQ4_0 = 2, kQ8_0 = 8, kQ6_K = 14 };
// Extended formats (ggml type ids): the K-quants Q4_K / Q5_K, the codebook
// formats IQ4_NL / IQ4_XS and the 2-byte pass-through types.
enum : int { kF16 = 1, kQ4_K = 12, kQ5_K = 13, kIQ4_NL = 20, kIQ4_XS = 23, kBF16 = 30 };

template <int FMT> struct Fmt;
template <> struct Fmt<kQ4_0> { static constexpr int kBlockK = 32;  static constexpr int kBlockBytes = 18; };
template <> struct Fmt<kQ8_0> { static constexpr int kBlockK = 32;  static constexpr int kBlockBytes = 34; };
template <> struct Fmt<kQ6_K> { static constexpr int kBlockK = 256; static constexpr int kBlockBytes = 210; };
template <> struct Fmt<kQ4_K> { static constexpr int kBlockK = 256; static constexpr int kBlockBytes = 144; };
template <> struct Fmt<kQ5_K> { static constexpr int kBlockK = 256; static constexpr int kBlockBytes = 176; };
template <> struct Fmt<kIQ4_NL> { static constexpr int kBlockK = 32; static constexpr int kBlockBytes = 18; };
template <> struct Fmt<kIQ4_XS> { static constexpr int kBlockK = 256; static constexpr int kBlockBytes = 136; };
// The 2-byte types are handled in chunks of 8 values (16 bytes).
template <> struct Fmt<kF16> { static constexpr int kBlockK = 8; static constexpr int kBlockBytes = 16; };
template <> struct Fmt<kBF16> { static constexpr int kBlockK = 8; static constexpr int kBlockBytes = 16; };

// Device-wide sticky error word.  Bounded waits that give up OR a code in here
// instead of trapping; the host reads and clears it (spiral_device_status).
enum : uint32_t {
  kDevErrMbarTimeout = 1u << 0,
  kDevErrTmemAlloc = 1u << 1,
  kDevErrBadLaunch = 1u << 2,
  kDevErrPeerTimeout = 1u << 3,  // a rank's gathered-GEMV pieces never arrived
};
extern __device__ uint32_t g_device_error;

__device__ __forceinline__ void raise_device_error(uint32_t code) {
  atomicOr(&g_device_error, code);
}

__host__ __device__ __forceinline__ int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }

// ----------------------------------------------------------- numerics -----

// fp16 bits -> fp32, exact (subnormals kept).  With ftz, subnormal inputs
// (exponent 0, mantissa != 0) become +0, as the reference repack stores them
// for its device path (src/quants/common/repack.h:29-34); zeros keep their
// sign.
__device__ __forceinline__ float fp16_bits_to_f32(uint32_t h, bool ftz) {
  if (ftz && (h & 0x7c00u) == 0u && (h & 0x03ffu) != 0u) return 0.0f;
  float f;
  asm("{ .reg .f16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"((unsigned short)h));
  return f;
}

// Two fp32 -> packed bf16x2 (lo in bits 0-15), round-to-nearest-even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Unsigned byte i of w placed in an fp32 whose value is 2^23 + byte.
template <int I>
__device__ __forceinline__ float byte_as_f32_magic(uint32_t w) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | I));
}

// ------------------------------------------------ exact fp16-route decode --
// Two quants placed in the mantissas of an fp16 pair by one LOP3
// (u = 2^e + q), then u * d + c per weight by a mixed-precision FMA with the
// fp16 scale d itself: u * d is exact inside the FMA and c = -(2^e + bias) d
// and the result (q - bias) d have at most 19 significant bits, so nothing
// rounds before the final bf16 conversion.
// (a & m) | o and (a & m) ^ o in one LOP3 each.
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t o) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(m), "r"(o));
  return r;
}
__device__ __forceinline__ uint32_t lop_and_xor(uint32_t a, uint32_t m, uint32_t o) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(m), "r"(o));
  return r;
}
// u.lo * d + c and u.hi * d + c for the fp16 pair u and the fp16 scale d,
// in fp32 with one rounding.
__device__ __forceinline__ float fmah_lo(uint32_t u, unsigned short d, float c) {
  float r;
  asm("{ .reg .b16 l, h; mov.b32 {l, h}, %1; fma.rn.f32.f16 %0, l, %2, %3; }" : "=f"(r) : "r"(u), "h"(d), "f"(c));
  return r;
}
__device__ __forceinline__ float fmah_hi(uint32_t u, unsigned short d, float c) {
  float r;
  asm("{ .reg .b16 l, h; mov.b32 {l, h}, %1; fma.rn.f32.f16 %0, h, %2, %3; }" : "=f"(r) : "r"(u), "h"(d), "f"(c));
  return r;
}
// The fp16 scale operand: a subnormal scale becomes +0 under ftz, zeros keep
// their sign, as fp16_bits_to_f32 does.
__device__ __forceinline__ unsigned short fp16_scale_bits(uint32_t h, bool ftz) {
  return (ftz && (h & 0x7c00u) == 0u && (h & 0x03ffu) != 0u) ? static_cast<unsigned short>(0)
                                                             : static_cast<unsigned short>(h);
}
// Two weights of the fp16 route, rounded to one bf16 pair (x in the low half).
__device__ __forceinline__ uint32_t h2pack_lo(uint32_t ux, uint32_t uy, unsigned short d, float c) {
  return pack_bf16x2(fmah_lo(ux, d, c), fmah_lo(uy, d, c));
}
__device__ __forceinline__ uint32_t h2pack_hi(uint32_t ux, uint32_t uy, unsigned short d, float c) {
  return pack_bf16x2(fmah_hi(ux, d, c), fmah_hi(uy, d, c));
}

// The product form for outputs that must match bit for bit, zero signs
// included (the standalone dequant): t = u - (2^e + bias) per fp16 half
// (exact: |q - bias| <= 128), then fma(t, d, -0), which is t * d rounded once
// with the IEEE sign of a zero product (+0 + -0 would lose it; -0 + -0
// keeps it).
__device__ __forceinline__ uint32_t hsub2(uint32_t u, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(u), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t h2mul_lo(uint32_t tx, uint32_t ty, unsigned short d) {
  return pack_bf16x2(fmah_lo(tx, d, -0.0f), fmah_lo(ty, d, -0.0f));
}
__device__ __forceinline__ uint32_t h2mul_hi(uint32_t tx, uint32_t ty, unsigned short d) {
  return pack_bf16x2(fmah_hi(tx, d, -0.0f), fmah_hi(ty, d, -0.0f));
}

// ----------------------------------------- programmatic dependent launch --
// A kernel launched with programmatic stream serialization lets its
// successor be scheduled once every CTA has called launch_dependents, and
// must call griddep_wait before it reads anything its predecessor wrote (the
// wait returns when the predecessor has completed and its writes are visible).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// --------------------------------------------------------- shared memory --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 4 bytes at a 2-byte aligned shared address.
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
  return __funnelshift_r(w[0], w[1], sh);
}
__device__ __forceinline__ uint32_t lds_u16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

// --------------------------------------------------- mbarrier + bulk copy --

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// The same test, but the thread may be suspended by the hardware until the
// phase completes or about `hint_ns` have passed: a waiting warp then issues
// nothing, leaving the issue slots to the warps that are decoding.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase: gives up after kWaitLimitNs of device
// time, records kDevErrMbarTimeout in the device error word and returns
// false, so callers drain and exit instead of hanging the GPU.  Each test
// may sleep up to kWaitSleepNs, so a waiting warp costs almost no issue slots.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint32_t kWaitSleepNs = 100000u;         // 100 us per suspended test
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      if (mbar_try_wait_sleep(bar, parity, kWaitSleepNs)) return true;
    }
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(kDevErrMbarTimeout);
      return false;
    }
  }
}

// L2 policy for data read exactly once (weights streamed by a GEMV).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 1-D bulk (TMA) copy global -> shared, completion counted on `bar` in bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace spiral
