// gemv_xs6.cu — activation-stationary decode GEMV (M <= 8) for Q6_K rows of
// six super-blocks: K = 1536, 1260-byte rows, the shape of the Gemma-style
// output head (N = 262,144).  MUL_MAT of the reference's q6_k unpack_mmul
// (src/quants/q6_k/mmul.aie.h:18-84) at a model shape the reference lists as
// its next step (src/quants/TODO.md:186-212).
//
// The rows are not 16-byte multiples, but four of them are (5,040 bytes), and
// at a 1,260-byte pitch the eight rows one fragment load touches fall on
// different banks, so an item of 32 rows is streamed as eight bulk copies of
// four contiguous rows and read in place.  One CTA per SM, 14 warps:
//   warps 0-11  decode: warp w owns super-block g = w % 6 of K and row block
//               w / 6 (16 rows) of every item; its activation fragments (the
//               16 k-steps of super-block g) are loaded once, into registers.
//   warp 12     producer: the items' bulk copies into a ring of stages.
//   warp 13     reducer: sums the six super-block partials of each output in
//               order and stores y.
// The summation order depends on K alone, so the result is bitwise
// repeatable.  All waits are bounded.
#include <atomic>

#include "api_internal.h"
#include "common.cuh"
#include "gemv_decode.cuh"

namespace spiral {
namespace {

constexpr int kX6Groups = 6;             // super-blocks per row
constexpr int kX6RowBytes = 6 * 210;     // 1260
constexpr int kX6Rows = 32;              // rows per item (2 MMA row blocks)
constexpr int kX6Warps = 12;
constexpr int kX6WarpProducer = 12, kX6WarpReducer = 13;
constexpr int kX6Threads = 14 * 32;
constexpr int kX6MaxStages = 8;
constexpr int kX6Header = 1024;
constexpr int kX6RedBytes = 2 * kX6Warps * 32 * 16;       // 2 buffers x 12 warps x 32 lanes x float4
constexpr int kX6CopyBytes = 4 * kX6RowBytes;             // 5,040: four rows, a multiple of 16
constexpr int kX6StageBytes = kX6Rows * kX6RowBytes;      // 40,320

struct X6Params {
  const uint8_t* w;
  const uint16_t* x;
  int64_t x_s8, x_sm;
  void* y;
  int64_t y_s8, y_sm;
  int64_t N;
  int M;
  int y_bf16, accumulate, static_weights, stages;
};

// 14 warps spread 4 + 4 + 3 + 3 over the sub-partitions: 128 registers per
// thread is the most that launches.
template <bool FTZ>
__global__ void __maxnreg__(128) gemv_xs6_kernel(const X6Params p) {
  using D = GroupDecoder<kQ6_K>;
  constexpr int kSteps = GemvFmt<kQ6_K>::kSteps;  // 16 k-steps per super-block
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kX6MaxStages;
  uint64_t* red_full = empty + kX6MaxStages;
  uint64_t* red_empty = red_full + 2;
  int& abort_flag = *reinterpret_cast<int*>(smem + 512);
  float4* red = reinterpret_cast<float4*>(smem + kX6Header);
  uint8_t* stg = smem + kX6Header + kX6RedBytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t items = p.N / kX6Rows;
  const int S = p.stages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kX6Warps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&red_full[b], kX6Warps * 32);
      mbar_init(&red_empty[b], 32);
    }
    abort_flag = 0;
    fence_mbar_init();
    griddep_launch_dependents();
  }
  __syncthreads();

  if (warp == kX6WarpProducer) {
    // ---------------------------------------------------------- producer --
    if (!p.static_weights) griddep_wait();
    const uint64_t pol = l2_evict_first_policy();
    uint32_t it = 0;
    int stage = 0;
    uint32_t phase = 0u;
    for (int64_t i = blockIdx.x; i < items; i += gridDim.x, ++it) {
      int go = 0;
      if (lane == 0) {
        go = !*(volatile int*)&abort_flag && mbar_wait(&empty[stage], phase ^ 1u);
        if (go) {
          mbar_arrive_expect_tx(&full[stage], kX6StageBytes);
        } else {
          abort_flag = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      if (lane < kX6Rows / 4)
        bulk_g2s(stg + stage * kX6StageBytes + lane * kX6CopyBytes,
                 p.w + (i * kX6Rows + 4 * lane) * kX6RowBytes, kX6CopyBytes, &full[stage], pol);
      if (++stage == S) {
        stage = 0;
        phase ^= 1u;
      }
    }
    // every issued copy must land before the CTA may exit
    if (lane == 0) {
      const uint32_t first = it > static_cast<uint32_t>(S) ? it - S : 0u;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % S], (j / S) & 1u);
    }
    return;
  }

  griddep_wait();  // x may come from the preceding kernel, which may also read y

  if (warp == kX6WarpReducer) {
    // ---------------------------------------------------------- reducer --
    // Lane l: for each row block b, the six partials (warps 6b + g) of
    // fragment lane l summed in super-block order; outputs rows l / 4 and
    // l / 4 + 8 of the block, vectors 2 (l % 4) and + 1.
    int local = 0;
    for (int64_t i = blockIdx.x; i < items; i += gridDim.x, ++local) {
      const int rbuf = local & 1;
      if (!mbar_try_wait(&red_full[rbuf], static_cast<uint32_t>(local >> 1) & 1u) && !*(volatile int*)&abort_flag) {
        if (!mbar_wait(&red_full[rbuf], static_cast<uint32_t>(local >> 1) & 1u)) abort_flag = 1;
      }
      float4 v[2];
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const float4* rp = red + (rbuf * kX6Warps + b * kX6Groups) * 32 + lane;
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int g = 0; g < kX6Groups; ++g) {
          const float4 q = rp[g * 32];
          sum.x += q.x;
          sum.y += q.y;
          sum.z += q.z;
          sum.w += q.w;
        }
        v[b] = sum;
      }
      mbar_arrive(&red_empty[rbuf]);
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        const float sums[4] = {v[b].x, v[b].y, v[b].z, v[b].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int m = 2 * (lane & 3) + (j & 1);
          const int64_t n = i * kX6Rows + 16 * b + (lane >> 2) + 8 * (j >> 1);
          if (m < p.M) {
            const int64_t off = (n >> 3) * p.y_s8 + static_cast<int64_t>(m) * p.y_sm + (n & 7);
            if (p.y_bf16) {
              static_cast<uint16_t*>(p.y)[off] = static_cast<uint16_t>(pack_bf16x2(sums[j], 0.f) & 0xFFFFu);
            } else if (p.accumulate) {
              static_cast<float*>(p.y)[off] += sums[j];
            } else {
              static_cast<float*>(p.y)[off] = sums[j];
            }
          }
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers --
  const int r = lane >> 2, c = lane & 3;
  const int g = warp % kX6Groups, rbk = warp / kX6Groups;
  // This warp's activation fragments for super-block g: two steps (t and
  // t + 4) share one aligned 16-byte load of 8 consecutive k.
  uint2 Bx[kSteps];
  {
    const bool vec = (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0 && (p.x_s8 & 7) == 0 && (p.x_sm & 7) == 0;
#pragma unroll
    for (int t = 0; t < kSteps; ++t) {
      if ((t >> 2) & 1) continue;  // filled with its lower half
      const int k = g * 256 + D::xk(t, c);  // k % 8 == 0
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < p.M) {
        const uint16_t* src = p.x + (k >> 3) * p.x_s8 + r * p.x_sm;
        if (vec) {
          v = __ldg(reinterpret_cast<const uint4*>(src));
        } else {
          v.x = static_cast<uint32_t>(src[0]) | (static_cast<uint32_t>(src[1]) << 16);
          v.y = static_cast<uint32_t>(src[2]) | (static_cast<uint32_t>(src[3]) << 16);
          v.z = static_cast<uint32_t>(src[4]) | (static_cast<uint32_t>(src[5]) << 16);
          v.w = static_cast<uint32_t>(src[6]) | (static_cast<uint32_t>(src[7]) << 16);
        }
      }
      Bx[t] = make_uint2(v.x, v.y);
      Bx[t + 4] = make_uint2(v.z, v.w);
    }
  }
  // MMA row r of the warp's row block = item row 16 rbk + r (+ 8); rows start
  // 4-byte aligned, super-block g at 210 g, 2 mod 4 for odd g
  const uint8_t* ra0 = stg + (16 * rbk + r) * kX6RowBytes + g * 210;
  const uint32_t sh = (g & 1) ? 16u : 0u;
  int stage = 0, local = 0;
  uint32_t phase = 0u;
  for (int64_t i = blockIdx.x; i < items; i += gridDim.x, ++local) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    bool ready = mbar_try_wait(&full[stage], phase);
    if (!ready && !*(volatile int*)&abort_flag) {
      ready = mbar_wait(&full[stage], phase);
      if (!ready) abort_flag = 1;
    }
    if (ready) {
      const uint8_t* ra = ra0 + stage * kX6StageBytes;
      D::run_b(ra, ra + 8 * kX6RowBytes, c, [&](int t) { return Bx[t]; }, FTZ, acc, sh);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == S) {
      stage = 0;
      phase ^= 1u;
    }
    const int rbuf = local & 1;
    if (local >= 2 && !mbar_try_wait(&red_empty[rbuf], static_cast<uint32_t>((local >> 1) - 1) & 1u) &&
        !*(volatile int*)&abort_flag) {
      if (!mbar_wait(&red_empty[rbuf], static_cast<uint32_t>((local >> 1) - 1) & 1u)) abort_flag = 1;
    }
    red[(rbuf * kX6Warps + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    mbar_arrive(&red_full[rbuf]);
  }
}

}  // namespace

bool gemv_xs6_ok(const MatArgs& a) {
  if (a.fmt != kQ6_K || a.K != kX6Groups * 256 || a.M < 1 || a.M > 8) return false;
  if (a.w_stride != kX6RowBytes || reinterpret_cast<uintptr_t>(a.w) % 16 != 0) return false;
  if (a.N < kX6Rows || a.N % kX6Rows != 0) return false;
  const size_t fixed = kX6Header + kX6RedBytes;
  return fixed + 2 * size_t(kX6StageBytes) <= device_max_smem_optin();
}

cudaError_t gemv_xs6(const MatArgs& a, cudaStream_t stream) {
  if (!gemv_xs6_ok(a)) return cudaErrorNotSupported;
  X6Params p{};
  p.w = a.w;
  p.x = a.x;
  p.x_s8 = a.x_s8;
  p.x_sm = a.x_sm;
  p.y = a.y;
  p.y_s8 = a.y_s8;
  p.y_sm = a.y_sm;
  p.N = a.N;
  p.M = static_cast<int>(a.M);
  p.y_bf16 = a.y_bf16;
  p.accumulate = a.accumulate;
  p.static_weights = a.static_weights;
  const size_t fixed = kX6Header + kX6RedBytes;
  const size_t avail = device_max_smem_optin();
  p.stages = static_cast<int>(std::min<size_t>(kX6MaxStages, (avail - fixed) / kX6StageBytes));
  const size_t smem = fixed + size_t(p.stages) * kX6StageBytes;
  auto* kernel = a.ftz ? gemv_xs6_kernel<true> : gemv_xs6_kernel<false>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<bool> configured[64][2];
  if (!configured[dev & 63][a.ftz ? 1 : 0].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(avail));
    if (e != cudaSuccess) return e;
    configured[dev & 63][a.ftz ? 1 : 0].store(true, std::memory_order_release);
  }
  const int64_t items = a.N / kX6Rows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(items, int64_t(device_sm_count()))));
  cfg.blockDim = dim3(kX6Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace spiral
