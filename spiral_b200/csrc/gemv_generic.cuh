// gemv_generic.cuh — the fallback MUL_MAT kernel for any format with a
// decode8_generic decoder: shapes the pipelined kernels do not take
// (unaligned rows, K not a multiple of their chunk granularity) and the
// extended formats.
#pragma once

#include "api_internal.h"
#include "decode.cuh"

namespace spiral {

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

}  // namespace spiral
