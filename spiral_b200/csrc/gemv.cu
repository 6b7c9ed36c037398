// gemv.cu — fused dequant-GEMV (decode, M <= 8 activation vectors) for sm_100a.
//
// B200 counterpart of the reference's fused unpack_mmul
// (src/quants/q4_0/mmul.aie.h:16-90, q8_0/mmul.aie.h:16-117,
// q6_k/mmul.aie.h:18-84): out[m][n] = sum_k in[m][k] * bf16(W[n][k]) with
// fp32 accumulation.  The weights are streamed from HBM exactly once.
//
// Structure (one persistent CTA per SM, 8 consumer warps + 1 producer warp):
//  * A "tile" is 16 output features (one m16 MMA row block) over all of K.
//    Tiles are dealt to CTAs round-robin.
//  * The producer lane streams each tile's rows chunk by chunk (up to 8
//    "groups" of K per chunk) with 1-D bulk (TMA) copies into a ring of shared
//    stages, one copy per row, completion counted in bytes on an mbarrier.
//    Weights use an L2 evict-first policy: they are read once.
//  * Consumer warp w takes group w of every chunk (a K-split inside the CTA),
//    dequantizes it in registers straight into the bf16 A fragments of
//    mma.sync.m16n8k16 (rows = features, k = 16 weights, n = 8 activation
//    vectors, padded), and accumulates in fp32.  At the end of a tile the 8
//    warps' partial 16x8 tiles are summed in a fixed order (deterministic)
//    and stored.
//  * Activations x are staged once per CTA into shared memory in a k order
//    permuted to match how each lane's A fragment is decoded, so every B
//    fragment is one conflict-free 8-byte shared load.  The MMA contracts
//    over k, so permuting k identically in A and B leaves the sum unchanged.
//
// Exactness: the A fragments are the same bf16 weights the standalone
// dequant produces (bf16_rne(d*int)), so results differ from the reference's
// dequant-then-fp32-matmul only by fp32 summation order.  Q4_0 uses a packed
// bf16 form of the exact product: d = hi + lo with hi = bf16(d) and lo =
// bf16(d - hi) exact (fp16 d has 11 significant bits), t = q - 8 exact, and
// fma.rn.bf16x2(t, hi, t*lo) = bf16_rne(t*hi + t*lo) = bf16_rne(t*d) since
// t*lo is exact in bf16.  (The only difference from the fp32 route is the
// sign of a zero weight, which cannot change a dot product.)
#include <atomic>

#include "api_internal.h"
#include "decode.cuh"

namespace spiral {

template <int FMT> struct GemvFmt;
// kGroupK weights per group; one group is what a consumer warp decodes per
// chunk.  kSteps = kGroupK / 16 MMA k-steps.  A chunk holds up to 8 groups of
// every tile row and is always a 16-byte multiple (2 groups for Q4_0/Q8_0, 8
// super-blocks for Q6_K).
template <> struct GemvFmt<kQ4_0> {
  static constexpr int kGroupK = 128, kGroupBytes = 72, kSteps = 8, kStages = 8, kGroupAlign = 2;
};
template <> struct GemvFmt<kQ8_0> {
  static constexpr int kGroupK = 128, kGroupBytes = 136, kSteps = 8, kStages = 5, kGroupAlign = 2;
};
template <> struct GemvFmt<kQ6_K> {
  static constexpr int kGroupK = 256, kGroupBytes = 210, kSteps = 16, kStages = 4, kGroupAlign = 8;
};

constexpr int kConsumerWarps = 8;
constexpr int kChunkGroups = kConsumerWarps;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kTileRows = 16;
constexpr int kBarrierBytes = 256;  // room for up to 16 mbarriers
constexpr int kRedBytes = kConsumerWarps * 32 * 16;

struct GemvParams {
  const uint8_t* w;
  int64_t w_stride;
  const uint16_t* x;
  int64_t x_s8, x_sm;
  void* y;
  int64_t y_s8, y_sm;
  int64_t N, K;
  int64_t groups_per_row;
  int M;
  int chunks_per_row;
  int stages;
  int row_pitch;  // bytes per row slot in a stage
  int x_pitch;    // bytes per activation vector in the permuted copy
  int y_bf16, accumulate, ftz, x_vec16;
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

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// Exact split of an fp32 value with <= 16 significant bits into bf16 hi + lo,
// each broadcast into both halves of a bf16x2 word.
__device__ __forceinline__ void split_scale_bf16x2(float d, uint32_t& hi2, uint32_t& lo2) {
  const uint32_t hi = pack_bf16x2(d, d);
  const float hf = __uint_as_float(hi << 16);
  const float lf = d - hf;  // exact
  lo2 = pack_bf16x2(lf, lf);
  hi2 = hi;
}

// Two Q4_0 weights from nibbles at bits [0,4) and [16,20) of w.
__device__ __forceinline__ uint32_t q4_0_pair(uint32_t w, uint32_t hi2, uint32_t lo2) {
  const uint32_t v = (w & 0x000F000Fu) | 0x43004300u;  // bf16 128 + q
  const uint32_t t = bf16x2_sub(v, 0x43084308u);       // q - 8, exact
  return bf16x2_fma(t, hi2, bf16x2_mul(t, lo2));
}

// --------------------------------------------- per-format group decoders --
// ra / rb: this lane's two feature rows (r and r + 8) at the group start in
// the stage; c = lane % 4; xg = this lane's B-fragment column at step 0 of
// the group in the permuted activations (stride 32 bytes per step).

template <int FMT>
__device__ __forceinline__ void group_mma(const uint8_t* ra, const uint8_t* rb, int c, const uint8_t* xg, bool ftz,
                                          float (&acc)[4]);

// Q4_0: lane c owns block c of the 4-block group.  Step s uses qs word
// j = s/2: pairs (weights 4j+o, 4j+o+2) and (16+4j+o, 16+4j+o+2), o = s%2.
template <>
__device__ __forceinline__ void group_mma<kQ4_0>(const uint8_t* ra, const uint8_t* rb, int c, const uint8_t* xg,
                                                 bool ftz, float (&acc)[4]) {
  const uint8_t* ba = ra + 18 * c;
  const uint8_t* bb = rb + 18 * c;
  uint32_t hia, loa, hib, lob;
  split_scale_bf16x2(fp16_bits_to_f32(lds_u16(ba), ftz), hia, loa);
  split_scale_bf16x2(fp16_bits_to_f32(lds_u16(bb), ftz), hib, lob);
  uint32_t qa[4], qb[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    qa[j] = lds_u32_a2(ba + 2 + 4 * j);
    qb[j] = lds_u32_a2(bb + 2 + 4 * j);
  }
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const int j = s >> 1;
    const uint32_t wa = (s & 1) ? (qa[j] >> 8) : qa[j];
    const uint32_t wb = (s & 1) ? (qb[j] >> 8) : qb[j];
    const uint2 b = *reinterpret_cast<const uint2*>(xg + 32 * s);
    mma_bf16_16816(acc, q4_0_pair(wa, hia, loa), q4_0_pair(wb, hib, lob), q4_0_pair(wa >> 4, hia, loa),
                   q4_0_pair(wb >> 4, hib, lob), b.x, b.y);
  }
}

// Q8_0: lane c owns block c of the group; step s = weights 4s..4s+3.
__device__ __forceinline__ uint32_t q8_0_pair(uint32_t w, int i, float d) {
  constexpr float kBias = 8388736.0f;  // 2^23 + 128
  const float f0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | i)) - kBias;
  const float f1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | (i + 1))) - kBias;
  return pack_bf16x2(f0 * d, f1 * d);
}
template <>
__device__ __forceinline__ void group_mma<kQ8_0>(const uint8_t* ra, const uint8_t* rb, int c, const uint8_t* xg,
                                                 bool ftz, float (&acc)[4]) {
  const uint8_t* ba = ra + 34 * c;
  const uint8_t* bb = rb + 34 * c;
  const float da = fp16_bits_to_f32(lds_u16(ba), ftz);
  const float db = fp16_bits_to_f32(lds_u16(bb), ftz);
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const uint32_t wa = lds_u32_a2(ba + 2 + 4 * s) ^ 0x80808080u;
    const uint32_t wb = lds_u32_a2(bb + 2 + 4 * s) ^ 0x80808080u;
    const uint2 b = *reinterpret_cast<const uint2*>(xg + 32 * s);
    mma_bf16_16816(acc, q8_0_pair(wa, 0, da), q8_0_pair(wb, 0, db), q8_0_pair(wa, 2, da), q8_0_pair(wb, 2, db), b.x,
                   b.y);
  }
}

// Q6_K: one super-block per group; lane c owns l in [8c, 8c+8) of both
// halves.  Step t = 8h + 4*half + s covers y = 128h + 32s + 8c + 4*half + 0..3.
template <>
__device__ __forceinline__ void group_mma<kQ6_K>(const uint8_t* ra, const uint8_t* rb, int c, const uint8_t* xg,
                                                 bool ftz, float (&acc)[4]) {
  const float da = fp16_bits_to_f32(lds_u16(ra + 208), ftz);
  const float db = fp16_bits_to_f32(lds_u16(rb + 208), ftz);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float dsa[4], dsb[4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int si = 192 + 8 * h + 2 * s + (c >> 1);
      dsa[s] = da * static_cast<float>(static_cast<int8_t>(ra[si]));
      dsb[s] = db * static_cast<float>(static_cast<int8_t>(rb[si]));
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int o = 8 * c + 4 * half;
      const uint32_t qla_a = lds_u32_a2(ra + 64 * h + o), qlb_a = lds_u32_a2(ra + 64 * h + 32 + o);
      const uint32_t qh_a = lds_u32_a2(ra + 128 + 32 * h + o);
      const uint32_t qla_b = lds_u32_a2(rb + 64 * h + o), qlb_b = lds_u32_a2(rb + 64 * h + 32 + o);
      const uint32_t qh_b = lds_u32_a2(rb + 128 + 32 * h + o);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint2 wa = q6_k_scale4(q6_k_assemble4((s & 1) ? qlb_a : qla_a, qh_a, s), dsa[s]);
        const uint2 wb = q6_k_scale4(q6_k_assemble4((s & 1) ? qlb_b : qla_b, qh_b, s), dsb[s]);
        const uint2 b = *reinterpret_cast<const uint2*>(xg + 32 * (8 * h + 4 * half + s));
        mma_bf16_16816(acc, wa.x, wb.x, wa.y, wb.y, b.x, b.y);
      }
    }
  }
}

// ------------------------------------------------- activation staging ----

__device__ __forceinline__ uint4 load_x8(const GemvParams& p, int m, int64_t k) {
  const uint16_t* base = p.x + (k >> 3) * p.x_s8 + static_cast<int64_t>(m) * p.x_sm;
  if (p.x_vec16) return __ldg(reinterpret_cast<const uint4*>(base));
  uint32_t e[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = base[i];
  return make_uint4(e[0] | (e[1] << 16), e[2] | (e[3] << 16), e[4] | (e[5] << 16), e[6] | (e[7] << 16));
}

// Writes the permuted activations: entry (m, group, step, c) = the 4 bf16
// that lane column c contracts at that step, at
//   xs + m*x_pitch + (group*kSteps + step)*32 + c*8.
template <int FMT>
__device__ void stage_x(const GemvParams& p, uint8_t* xs, int tid, int nthreads) {
  using F = GemvFmt<FMT>;
  const int64_t groups = p.K / F::kGroupK;
  const int64_t units = static_cast<int64_t>(p.M) * groups * 4;
  for (int64_t u = tid; u < units; u += nthreads) {
    const int m = static_cast<int>(u / (groups * 4));
    const int64_t rem = u - static_cast<int64_t>(m) * groups * 4;
    const int64_t g = rem >> 2;
    const int c = static_cast<int>(rem & 3);
    uint8_t* out = xs + static_cast<int64_t>(m) * p.x_pitch + g * F::kSteps * 32 + c * 8;
    if constexpr (FMT == kQ4_0 || FMT == kQ8_0) {
      const int64_t k0 = g * 128 + 32 * c;  // this lane column's block
      uint32_t X[16];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = load_x8(p, m, k0 + 8 * i);
        X[4 * i] = v.x;
        X[4 * i + 1] = v.y;
        X[4 * i + 2] = v.z;
        X[4 * i + 3] = v.w;
      }
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        uint2 e;
        if constexpr (FMT == kQ4_0) {
          const int j = s >> 1;
          const uint32_t sel = (s & 1) ? 0x7632u : 0x5410u;
          e.x = __byte_perm(X[2 * j], X[2 * j + 1], sel);
          e.y = __byte_perm(X[8 + 2 * j], X[9 + 2 * j], sel);
        } else {
          e.x = X[2 * s];
          e.y = X[2 * s + 1];
        }
        *reinterpret_cast<uint2*>(out + 32 * s) = e;
      }
    } else {
      const int64_t k0 = g * 256 + 8 * c;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const uint4 v = load_x8(p, m, k0 + 128 * h + 32 * s);
          *reinterpret_cast<uint2*>(out + 32 * (8 * h + s)) = make_uint2(v.x, v.y);
          *reinterpret_cast<uint2*>(out + 32 * (8 * h + 4 + s)) = make_uint2(v.z, v.w);
        }
      }
    }
  }
}

// --------------------------------------------------------------- kernel ---

template <int FMT>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvParams p) {
  using F = GemvFmt<FMT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + p.stages;
  float4* red = reinterpret_cast<float4*>(smem + kBarrierBytes);
  uint8_t* xs = smem + kBarrierBytes + kRedBytes;
  uint8_t* stages = xs + static_cast<int64_t>(p.M) * p.x_pitch;
  const int stage_bytes = kTileRows * p.row_pitch;
  // Set when a bounded wait gave up: later waits are skipped (not retried) so
  // every warp still reaches every named barrier and the kernel ends.
  int& abort_flag = *reinterpret_cast<int*>(smem + kBarrierBytes - 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tiles = (p.N + kTileRows - 1) / kTileRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------- producer ----
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t it = 0;
      for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
        const int64_t n0 = tile * kTileRows;
        const int rows = static_cast<int>(::spiral::min64(kTileRows, p.N - n0));
        const uint8_t* src_tile = p.w + n0 * p.w_stride;
        for (int ch = 0; ch < p.chunks_per_row; ++ch, ++it) {
          const int s = static_cast<int>(it % p.stages);
          const uint32_t ph = (it / p.stages) & 1u;
          if (!mbar_wait(&empty[s], ph ^ 1u) || *(volatile int*)&abort_flag) {
            abort_flag = 1;
            goto drain;
          }
          const int64_t g0 = static_cast<int64_t>(ch) * kChunkGroups;
          const int ng = static_cast<int>(::spiral::min64(kChunkGroups, p.groups_per_row - g0));
          const uint32_t bytes = static_cast<uint32_t>(ng * F::kGroupBytes);
          mbar_arrive_expect_tx(&full[s], bytes * rows);
          uint8_t* dst = stages + s * stage_bytes;
          const uint8_t* src = src_tile + g0 * F::kGroupBytes;
          for (int r = 0; r < rows; ++r) bulk_g2s(dst + r * p.row_pitch, src + r * p.w_stride, bytes, &full[s], pol);
        }
      }
    drain:
      // Every issued stage must land before the CTA may exit.
      const uint32_t first = it > static_cast<uint32_t>(p.stages) ? it - p.stages : 0u;
      for (uint32_t i = first; i < it; ++i) mbar_wait(&full[i % p.stages], (i / p.stages) & 1u);
    }
    return;
  }

  // --------------------------------------------------------- consumers -----
  stage_x<FMT>(p, xs, threadIdx.x, kConsumerWarps * 32);
  named_bar_sync(1, kConsumerWarps * 32);

  const int r = lane >> 2, c = lane & 3;
  const int mx = r < p.M ? r : 0;  // vectors >= M read vector 0; their columns are discarded
  const uint8_t* xcol = xs + static_cast<int64_t>(mx) * p.x_pitch + c * 8;
  uint32_t it = 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int ch = 0; ch < p.chunks_per_row; ++ch, ++it) {
      const int s = static_cast<int>(it % p.stages);
      const uint32_t ph = (it / p.stages) & 1u;
      bool ready = false;
      if (!*(volatile int*)&abort_flag) {
        ready = mbar_wait(&full[s], ph);
        if (!ready) abort_flag = 1;
      }
      const int64_t g0 = static_cast<int64_t>(ch) * kChunkGroups;
      const int ng = static_cast<int>(::spiral::min64(kChunkGroups, p.groups_per_row - g0));
      if (ready && warp < ng) {
        const uint8_t* st = stages + s * stage_bytes + warp * F::kGroupBytes;
        group_mma<FMT>(st + r * p.row_pitch, st + (r + 8) * p.row_pitch, c,
                       xcol + (g0 + warp) * F::kSteps * 32, p.ftz != 0, acc);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    red[warp * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    named_bar_sync(1, kConsumerWarps * 32);
    if (threadIdx.x < 128) {
      const int l = threadIdx.x >> 2, j = threadIdx.x & 3;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) sum += reinterpret_cast<const float*>(&red[w * 32 + l])[j];
      const int row = (l >> 2) + 8 * (j >> 1);
      const int m = 2 * (l & 3) + (j & 1);
      const int64_t n = tile * kTileRows + row;
      if (m < p.M && n < p.N) {
        const int64_t off = (n >> 3) * p.y_s8 + static_cast<int64_t>(m) * p.y_sm + (n & 7);
        if (p.y_bf16) {
          static_cast<uint16_t*>(p.y)[off] = static_cast<uint16_t>(pack_bf16x2(sum, 0.f) & 0xFFFFu);
        } else if (p.accumulate) {
          static_cast<float*>(p.y)[off] += sum;
        } else {
          static_cast<float*>(p.y)[off] = sum;
        }
      }
    }
    named_bar_sync(1, kConsumerWarps * 32);
  }
}

// Fallback for shapes the pipelined kernel does not take (unaligned rows,
// K not a multiple of the chunk granularity, very large K).  One warp per
// feature row, generic 2-byte loads, fp32 FMAs, warp-shuffle reduction.
template <int FMT>
__global__ void __launch_bounds__(256) gemv_generic(const MatArgs a) {
  constexpr int kBK = Fmt<FMT>::kBlockK, kBB = Fmt<FMT>::kBlockBytes;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t n = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); n < a.N; n += warps) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const uint8_t* row = a.w + n * a.w_stride;
    for (int64_t kc = lane; kc < a.K / 8; kc += 32) {
      const int64_t k = kc * 8, blk = k / kBK;
      const uint4 q = decode8_generic<FMT>(row + blk * kBB, static_cast<int>((k - blk * kBK) / 8), a.ftz);
      const uint32_t wq[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        if (m >= a.M) break;
        const uint16_t* xp = a.x + (k >> 3) * a.x_s8 + m * a.x_sm;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float wv = __uint_as_float((i & 1) ? (wq[i >> 1] & 0xFFFF0000u) : (wq[i >> 1] << 16));
          s = fmaf(wv, __uint_as_float(static_cast<uint32_t>(xp[i]) << 16), s);
        }
        acc[m] += s;
      }
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      if (m >= a.M) break;
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) {
        const int64_t off = (n >> 3) * a.y_s8 + m * a.y_sm + (n & 7);
        if (a.y_bf16) {
          static_cast<uint16_t*>(a.y)[off] = static_cast<uint16_t>(pack_bf16x2(v, 0.f) & 0xFFFFu);
        } else if (a.accumulate) {
          static_cast<float*>(a.y)[off] += v;
        } else {
          static_cast<float*>(a.y)[off] = v;
        }
      }
    }
  }
}

// ------------------------------------------------------------- launch ----

template <int FMT>
static size_t gemv_smem_bytes(const MatArgs& a, int stages, int* row_pitch, int* x_pitch, int* chunks) {
  using F = GemvFmt<FMT>;
  const int64_t gpr = a.K / F::kGroupK;
  const int chunk_groups = static_cast<int>(std::min<int64_t>(kChunkGroups, gpr));
  *chunks = static_cast<int>((gpr + kChunkGroups - 1) / kChunkGroups);
  *row_pitch = ((chunk_groups * F::kGroupBytes + 15) / 16) * 16 + 16;  // +16: spreads banks, covers over-read
  *x_pitch = static_cast<int>(a.K * 2 + 32);
  return kBarrierBytes + kRedBytes + static_cast<size_t>(a.M) * (*x_pitch) +
         static_cast<size_t>(stages) * kTileRows * (*row_pitch);
}

template <int FMT>
static bool gemv_fast_ok_t(const MatArgs& a) {
  using F = GemvFmt<FMT>;
  const int64_t align_k = static_cast<int64_t>(F::kGroupK) * F::kGroupAlign;
  if (a.M < 1 || a.M > 8) return false;
  if (a.K % align_k != 0) return false;
  if (reinterpret_cast<uintptr_t>(a.w) % 16 != 0 || a.w_stride % 16 != 0) return false;
  int rp, xp, ch;
  return gemv_smem_bytes<FMT>(a, 2, &rp, &xp, &ch) <= device_max_smem_optin();
}

bool gemv_fast_ok(const MatArgs& a) {
  switch (a.fmt) {
    case kQ4_0: return gemv_fast_ok_t<kQ4_0>(a);
    case kQ8_0: return gemv_fast_ok_t<kQ8_0>(a);
    case kQ6_K: return gemv_fast_ok_t<kQ6_K>(a);
  }
  return false;
}

template <int FMT>
static cudaError_t gemv_t(const MatArgs& a, cudaStream_t stream) {
  using F = GemvFmt<FMT>;
  if (!gemv_fast_ok_t<FMT>(a)) {
    const int64_t blocks = std::min<int64_t>((a.N + 7) / 8, int64_t(device_sm_count()) * 16);
    gemv_generic<FMT><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
    return cudaGetLastError();
  }
  GemvParams p{};
  p.w = a.w;
  p.w_stride = a.w_stride;
  p.x = a.x;
  p.x_s8 = a.x_s8;
  p.x_sm = a.x_sm;
  p.y = a.y;
  p.y_s8 = a.y_s8;
  p.y_sm = a.y_sm;
  p.N = a.N;
  p.K = a.K;
  p.M = static_cast<int>(a.M);
  p.groups_per_row = a.K / F::kGroupK;
  p.y_bf16 = a.y_bf16;
  p.accumulate = a.accumulate;
  p.ftz = a.ftz;
  p.x_vec16 = (reinterpret_cast<uintptr_t>(a.x) % 16 == 0) && (a.x_s8 * 2) % 16 == 0 && (a.x_sm * 2) % 16 == 0;
  int stages = F::kStages;
  size_t smem = 0;
  for (; stages >= 2; --stages) {
    smem = gemv_smem_bytes<FMT>(a, stages, &p.row_pitch, &p.x_pitch, &p.chunks_per_row);
    if (smem <= device_max_smem_optin()) break;
  }
  p.stages = stages;
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = FMT == kQ4_0 ? 0 : (FMT == kQ8_0 ? 1 : 2);
  static std::atomic<bool> configured[64][3];
  if (!configured[dev & 63][slot].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(gemv_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(device_max_smem_optin()));
    if (e != cudaSuccess) return e;
    configured[dev & 63][slot].store(true, std::memory_order_release);
  }
  // Occupancy depends only on (device, format, dynamic smem); cache it so
  // launches made under CUDA-graph capture issue no extra runtime calls.
  static std::atomic<int64_t> occ_cache[64][3][8];
  const int bucket = static_cast<int>(std::min<int64_t>(7, a.M - 1));
  const int64_t key = (static_cast<int64_t>(smem) << 8);
  int occ = 0;
  const int64_t cached = occ_cache[dev & 63][slot][bucket].load(std::memory_order_relaxed);
  if (cached != 0 && (cached & ~int64_t(0xff)) == key) {
    occ = static_cast<int>(cached & 0xff);
  } else {
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, gemv_kernel<FMT>, kGemvThreads, smem);
    if (e != cudaSuccess) return e;
    occ = std::max(occ, 1);
    occ_cache[dev & 63][slot][bucket].store(key | occ, std::memory_order_relaxed);
  }
  const int64_t tiles = (a.N + kTileRows - 1) / kTileRows;
  const int64_t grid = std::min<int64_t>(tiles, int64_t(device_sm_count()) * occ);
  gemv_kernel<FMT><<<static_cast<unsigned>(grid), kGemvThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t gemv(const MatArgs& a, cudaStream_t stream) {
  switch (a.fmt) {
    case kQ4_0: return gemv_t<kQ4_0>(a, stream);
    case kQ8_0: return gemv_t<kQ8_0>(a, stream);
    case kQ6_K: return gemv_t<kQ6_K>(a, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace spiral
