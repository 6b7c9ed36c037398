// gemm.cu — fused dequant-GEMM (prefill, many activation vectors) on the
// sm_100a tensor cores (tcgen05 + tensor memory).
//
// B200 counterpart of the reference's fused unpack_mmul
// (src/quants/q4_0/mmul.aie.h:16-90, q8_0/mmul.aie.h:16-117,
// q6_k/mmul.aie.h:18-84) for large M: y[m][n] = sum_k bf16(W[n][k]) x[m][k].
//
// One persistent CTA per SM computes 128-feature x BN-token output tiles:
//   warp 0      TMA producer: activation tiles x[BN tokens][64 k] land in a
//               4-deep shared ring with the 128-byte swizzle (B operand).
//   warp 1      MMA issuer (one thread): tcgen05.mma.kind::f16, A = the
//               dequantized weight tile read from tensor memory, B = the
//               swizzled activations, D = fp32 accumulator in tensor memory.
//   warps 2-9   dequant: one thread per weight row (= TMEM lane); each
//               quadrant of 32 rows is served by two warps that split every
//               256-weight K chunk in halves.  They read canonical GGUF
//               blocks straight from global memory, expand them exactly
//               (fp16 scale x integer in fp32, one RNE rounding to bf16) and
//               store the bf16 pairs into a TMEM A stage (two stages).
//   warps 10-13 epilogue: read D back (tcgen05.ld), round, store y.
// Tensor memory: columns [0, BN) accumulator, [256, 384) and [384, 512) the
// two A stages (a 256-wide K chunk is 128 columns of bf16 pairs).
// All pipeline waits are bounded; a wait that gives up marks the device
// error word and the CTA drains and exits.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>

#include "api_internal.h"
#include "chunk_decode.cuh"
#include "decode.cuh"
#include "tcgen05.cuh"
#include "tma_host.h"

namespace spiral {

constexpr int kGemmRows = 128;      // features per tile (MMA M, TMEM lanes)
constexpr int kChunkK = 256;        // K per A stage
constexpr int kXSliceK = 64;        // K per activation ring slot (128 bytes)
constexpr int kXStages = 4;
constexpr int kAStages = 2;
constexpr int kAColBase = 256;      // first TMEM column of the A stages
constexpr int kAStageCols = kChunkK / 2;
constexpr int kGemmThreads = 14 * 32;
constexpr int kWarpProducer = 0, kWarpMma = 1, kWarpDequant0 = 2, kWarpEpilogue0 = 10;

struct GemmParams {
  const uint8_t* w;
  int64_t w_stride;
  void* y;
  int64_t y_stride;  // elements
  int M, N, K;
  int y_bf16, accumulate, ftz;
  int token_blocks, feature_blocks;
  int tma_store;  // bf16 output written through the staging tile + TMA store
};

// ------------------------------------------------------ weight dequant ----

template <int FMT>
struct ChunkDecoder;

// Q4_0: a 256-weight chunk of one row is 8 blocks (144 bytes).  Half h takes
// blocks 4h..4h+3; its bytes [72h, 72h+72) lie in the 16-byte aligned window
// [64h, 64h+80).
template <>
struct ChunkDecoder<kQ4_0> {
  static constexpr int kChunkBytes = 144;
  static constexpr int kLoads = 5;
  __device__ __forceinline__ static int64_t window(int h) { return 64 * h; }
  template <int H, int J>
  __device__ __forceinline__ static void block(const uint32_t* R, bool ftz, uint32_t (&out)[16]) {
    BlockDecoder<kQ4_0>::block<8 * H + 18 * J>(R, ftz, out);
  }
};

// Q8_0: 8 blocks of 34 bytes (272); half h's bytes [136h, 136h+136) lie in
// [128h, 128h+144).
template <>
struct ChunkDecoder<kQ8_0> {
  static constexpr int kChunkBytes = 272;
  static constexpr int kLoads = 9;
  __device__ __forceinline__ static int64_t window(int h) { return 128 * h; }
  template <int H, int J>
  __device__ __forceinline__ static void block(const uint32_t* R, bool ftz, uint32_t (&out)[16]) {
    BlockDecoder<kQ8_0>::block<8 * H + 34 * J>(R, ftz, out);
  }
};

// Q6_K: a 256-weight chunk of one row is one 210-byte super-block; half h
// takes weights [128h, 128h + 128) (Q6KHalf, compile-time offsets for each
// of the 8 possible 16-byte phases of the super-block start).
template <>
struct ChunkDecoder<kQ6_K> {
  static constexpr int kChunkBytes = 210;
  static constexpr int kLoads = 1;  // unused: Q6KHalf loads its own windows
  __device__ __forceinline__ static int64_t window(int) { return 0; }
};

template <int H, typename Store>
__device__ __forceinline__ void q6k_half_any_phase(const uint8_t* sb, int phase, bool ftz, Store&& store) {
  switch (phase) {
    case 0: Q6KHalf<0, H>::run(sb, ftz, store); break;
    case 2: Q6KHalf<2, H>::run(sb, ftz, store); break;
    case 4: Q6KHalf<4, H>::run(sb, ftz, store); break;
    case 6: Q6KHalf<6, H>::run(sb, ftz, store); break;
    case 8: Q6KHalf<8, H>::run(sb, ftz, store); break;
    case 10: Q6KHalf<10, H>::run(sb, ftz, store); break;
    case 12: Q6KHalf<12, H>::run(sb, ftz, store); break;
    default: Q6KHalf<14, H>::run(sb, ftz, store); break;
  }
}

// ------------------------------------------------------------- kernel -----

template <int FMT, int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                const GemmParams p) {
  using CD = ChunkDecoder<FMT>;
  constexpr uint32_t kXStageBytes = BN * 128;
  constexpr uint32_t kIdesc = tc::idesc_bf16_f32(kGemmRows, BN);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzled activation ring
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xring = smem;
  uint16_t* ystage = reinterpret_cast<uint16_t*>(smem + kXStages * kXStageBytes);  // [BN][128] bf16
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kXStages * kXStageBytes + BN * kGemmRows * 2);
  uint64_t* x_full = bars;
  uint64_t* x_empty = bars + kXStages;
  uint64_t* a_full = bars + 2 * kXStages;
  uint64_t* a_empty = a_full + kAStages;
  uint64_t* d_full = a_empty + kAStages;
  uint64_t* d_empty = d_full + 1;
  uint64_t* done = d_empty + 1;
  uint32_t* tmem_base_smem = reinterpret_cast<uint32_t*>(done + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_base_smem + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = p.token_blocks * p.feature_blocks;
  const int kchunks = p.K / kChunkK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kXStages; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
    }
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(&a_full[i], 8);
      mbar_init(&a_empty[i], 1);
    }
    mbar_init(d_full, 1);
    mbar_init(d_empty, 4);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kWarpProducer) {
    tc::tmem_alloc(tmem_base_smem, 512);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_base_smem;
  volatile int* abortv = abort_flag;
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (*abortv) return false;
    if (!mbar_wait(bar, parity)) {
      *abortv = 1;
      return false;
    }
    return true;
  };

  if (warp == kWarpProducer) {
    // ------------------------------------------------ activation producer --
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        const int tb = t % p.token_blocks;
        for (int kx = 0; kx < p.K / kXSliceK; ++kx, ++it) {
          const int s = it % kXStages;
          if (!wait(&x_empty[s], ((it / kXStages) & 1u) ^ 1u)) break;
          mbar_arrive_expect_tx(&x_full[s], kXStageBytes);
          tc::tma_load_2d(xring + s * kXStageBytes, &xmap, kx * kXSliceK, tb * BN, &x_full[s]);
        }
        if (*abortv) break;
      }
    }
  } else if (warp == kWarpMma) {
    // ------------------------------------------------------- MMA issuer ----
    if (lane == 0) {
      uint32_t xit = 0, ait = 0, tcount = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tcount) {
        if (!wait(d_empty, (tcount & 1u) ^ 1u)) break;
        tc::fence_after_sync();
        for (int kc = 0; kc < kchunks; ++kc, ++ait) {
          const int s = ait % kAStages;
          if (!wait(&a_full[s], (ait / kAStages) & 1u)) break;
          tc::fence_after_sync();
          for (int sub = 0; sub < kChunkK / kXSliceK; ++sub, ++xit) {
            const int xs = xit % kXStages;
            if (!wait(&x_full[xs], (xit / kXStages) & 1u)) break;
            tc::fence_after_sync();
            const uint32_t xaddr = smem_u32(xring + xs * kXStageBytes);
#pragma unroll
            for (int j = 0; j < kXSliceK / 16; ++j) {
              const uint32_t a_taddr = tmem + kAColBase + s * kAStageCols + (sub * (kXSliceK / 16) + j) * 8;
              tc::mma_ts(tmem, a_taddr, tc::sdesc_sw128_kmajor(xaddr + j * 32), kIdesc, kc | sub | j);
            }
            tc::commit(&x_empty[xs]);
          }
          tc::commit(&a_empty[s]);
        }
        tc::commit(d_full);
        if (*abortv) break;
      }
      // all MMAs issued by this thread must finish before TMEM is released
      tc::commit(done);
      mbar_wait(done, 0);
    }
  } else if (warp < kWarpEpilogue0) {
    // ---------------------------------------------------------- dequant ----
    const int q = warp & 3;                      // TMEM lane quadrant
    const int h = (warp - kWarpDequant0) >> 2;   // half of each K chunk
    const int row = 32 * q + lane;
    uint32_t ait = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int fb = t / p.token_blocks;
      const int n = fb * kGemmRows + row;
      const bool valid = n < p.N;
      const uint8_t* wrow = p.w + static_cast<int64_t>(valid ? n : 0) * p.w_stride;
      if constexpr (FMT == kQ6_K) {
        for (int kc = 0; kc < kchunks; ++kc, ++ait) {
          const int s = ait % kAStages;
          if (!wait(&a_empty[s], ((ait / kAStages) & 1u) ^ 1u)) break;
          tc::fence_after_sync();
          const uint32_t tbase = tmem + (static_cast<uint32_t>(32 * q) << 16) + kAColBase + s * kAStageCols + 64 * h;
          auto store = [&](int j, const uint32_t (&out)[16]) { tc::st_32x32b_x16(tbase + 16 * j, out); };
          // Every lane runs the same path (tcgen05.st is warp-collective): rows
          // past N decode row 0 and their outputs are never stored.  The
          // phase is warp-uniform (16-byte aligned base and row stride).
          const uint8_t* sb = wrow + static_cast<int64_t>(kc) * CD::kChunkBytes;
          const int phase = static_cast<int>(reinterpret_cast<uintptr_t>(sb) & 15u);
          if (h == 0)
            q6k_half_any_phase<0>(sb, phase, p.ftz, store);
          else
            q6k_half_any_phase<1>(sb, phase, p.ftz, store);
          tc::wait_st();
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[s]);
        }
      } else {
      // The next chunk's packed bytes are loaded one chunk ahead (into Rn)
      // while this chunk is decoded, so the global-load latency leaves the
      // path between a free A stage and a full one.
      uint32_t R[CD::kLoads * 4], Rn[CD::kLoads * 4];
      auto load_chunk = [&](int kcl, uint32_t (&dst)[CD::kLoads * 4]) {
        if (valid) {
          const uint4* src =
              reinterpret_cast<const uint4*>(wrow + static_cast<int64_t>(kcl) * CD::kChunkBytes + CD::window(h));
#pragma unroll
          for (int i = 0; i < CD::kLoads; ++i) {
            const uint4 v = __ldg(src + i);
            dst[4 * i] = v.x;
            dst[4 * i + 1] = v.y;
            dst[4 * i + 2] = v.z;
            dst[4 * i + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < CD::kLoads * 4; ++i) dst[i] = 0u;
        }
      };
      load_chunk(0, R);
      for (int kc = 0; kc < kchunks; ++kc, ++ait) {
        const int s = ait % kAStages;
        if (kc + 1 < kchunks) load_chunk(kc + 1, Rn);
        if (!wait(&a_empty[s], ((ait / kAStages) & 1u) ^ 1u)) break;
        tc::fence_after_sync();
        const uint32_t tbase = tmem + (static_cast<uint32_t>(32 * q) << 16) + kAColBase + s * kAStageCols + 64 * h;
        uint32_t out[16];
        if (h == 0) {
          CD::template block<0, 0>(R, p.ftz, out); tc::st_32x32b_x16(tbase + 0, out);
          CD::template block<0, 1>(R, p.ftz, out); tc::st_32x32b_x16(tbase + 16, out);
          CD::template block<0, 2>(R, p.ftz, out); tc::st_32x32b_x16(tbase + 32, out);
          CD::template block<0, 3>(R, p.ftz, out); tc::st_32x32b_x16(tbase + 48, out);
        } else {
          CD::template block<1, 0>(R, p.ftz, out); tc::st_32x32b_x16(tbase + 0, out);
          CD::template block<1, 1>(R, p.ftz, out); tc::st_32x32b_x16(tbase + 16, out);
          CD::template block<1, 2>(R, p.ftz, out); tc::st_32x32b_x16(tbase + 32, out);
          CD::template block<1, 3>(R, p.ftz, out); tc::st_32x32b_x16(tbase + 48, out);
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&a_full[s]);
#pragma unroll
        for (int i = 0; i < CD::kLoads * 4; ++i) R[i] = Rn[i];
      }
      }
      if (*abortv) break;
    }
  } else {
    // --------------------------------------------------------- epilogue ----
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const int et = threadIdx.x - kWarpEpilogue0 * 32;  // 0..127
    const uint32_t trow = tmem + (static_cast<uint32_t>(32 * q) << 16);
    uint32_t tcount = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++tcount) {
      const int tb = t % p.token_blocks, fb = t / p.token_blocks;
      if (!wait(d_full, tcount & 1u)) break;
      tc::fence_after_sync();
      const int n = fb * kGemmRows + row;
      const int m0 = tb * BN;
      if (p.tma_store) {
        // The previous tile's store must have finished reading the staging tile.
        if (et == 0) tc::bulk_wait_read_all();
        named_bar_sync(1, 128);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t v[32];
          tc::ld_32x32b_x32(trow + c, v);
          tc::wait_ld();
          if (c + 32 >= BN) {  // accumulator fully read: the next tile's MMAs may start
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i)
            ystage[(c + i) * kGemmRows + row] =
                static_cast<uint16_t>(pack_bf16x2(__uint_as_float(v[i]), 0.f) & 0xFFFFu);
        }
        tc::fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (et == 0) {
          tc::tma_store_2d(&ymap, ystage, fb * kGemmRows, m0);
          tc::bulk_commit_group();
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 16) {
          uint32_t v[16];
          tc::ld_32x32b_x16(trow + c, v);
          tc::wait_ld();
          if (n < p.N) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int m = m0 + c + i;
              if (m < p.M) {
                const float f = __uint_as_float(v[i]);
                const int64_t off = static_cast<int64_t>(m) * p.y_stride + n;
                if (p.y_bf16) {
                  static_cast<uint16_t*>(p.y)[off] = static_cast<uint16_t>(pack_bf16x2(f, 0.f) & 0xFFFFu);
                } else if (p.accumulate) {
                  static_cast<float*>(p.y)[off] += f;
                } else {
                  static_cast<float*>(p.y)[off] = f;
                }
              }
            }
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_empty);
      }
    }
    if (et == 0) tc::bulk_wait_all();
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kWarpProducer) tc::tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------ host side ---

namespace {

template <int BN>
constexpr size_t gemm_smem() {
  return 1024 /*alignment slack*/ + kXStages * BN * 128 + BN * kGemmRows * 2 /*y staging*/ + 256 /*barriers*/;
}

}  // namespace

bool gemm_supported(const MatArgs& a) {
  if (a.fmt != kQ4_0 && a.fmt != kQ8_0 && a.fmt != kQ6_K) return false;
  // Q6_K: rows of whole 8-super-block runs keep its 16-byte windows in bounds
  if (a.fmt == kQ6_K && a.K % 2048 != 0) return false;
  if (a.x_s8 != 8 || a.y_s8 != 8) return false;  // row-major operands only
  if (a.K % kChunkK != 0 || a.K > (int64_t(1) << 30)) return false;
  if (a.M > (int64_t(1) << 30) || a.N > (int64_t(1) << 30)) return false;
  if (reinterpret_cast<uintptr_t>(a.x) % 16 != 0 || (a.x_sm * 2) % 16 != 0) return false;
  if (reinterpret_cast<uintptr_t>(a.w) % 16 != 0 || a.w_stride % 16 != 0) return false;
  return tensor_map_encoder() != nullptr;
}

template <int FMT, int BN>
static cudaError_t gemm_launch(const MatArgs& a, cudaStream_t stream) {
  CUtensorMap map;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(a.K), static_cast<cuuint64_t>(a.M)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(a.x_sm * 2)};
  const cuuint32_t box[2] = {kXSliceK, BN};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = tensor_map_encoder()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a.x), dims, strides,
                                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  // bf16 output: a TMA tensor store of each [BN][128] tile (clipped at M, N)
  CUtensorMap ymap;
  memset(&ymap, 0, sizeof(ymap));
  const bool tma_store = a.y_bf16 && !a.accumulate && reinterpret_cast<uintptr_t>(a.y) % 16 == 0 &&
                         (a.y_sm * 2) % 16 == 0;
  if (tma_store) {
    const cuuint64_t ydims[2] = {static_cast<cuuint64_t>(a.N), static_cast<cuuint64_t>(a.M)};
    const cuuint64_t ystrides[1] = {static_cast<cuuint64_t>(a.y_sm * 2)};
    const cuuint32_t ybox[2] = {kGemmRows, BN};
    const CUresult ry = tensor_map_encoder()(&ymap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.y, ydims, ystrides, ybox, estr,
                                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (ry != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  GemmParams p{};
  p.tma_store = tma_store ? 1 : 0;
  p.w = a.w;
  p.w_stride = a.w_stride;
  p.y = a.y;
  p.y_stride = a.y_sm;
  p.M = static_cast<int>(a.M);
  p.N = static_cast<int>(a.N);
  p.K = static_cast<int>(a.K);
  p.y_bf16 = a.y_bf16;
  p.accumulate = a.accumulate;
  p.ftz = a.ftz;
  p.token_blocks = static_cast<int>((a.M + BN - 1) / BN);
  p.feature_blocks = static_cast<int>((a.N + kGemmRows - 1) / kGemmRows);
  constexpr size_t smem = gemm_smem<BN>();
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<bool> configured[64];
  if (!configured[dev & 63].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<FMT, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    configured[dev & 63].store(true, std::memory_order_release);
  }
  const int tiles = p.token_blocks * p.feature_blocks;
  const int grid = std::min(tiles, device_sm_count());
  gemm_kernel<FMT, BN><<<grid, kGemmThreads, smem, stream>>>(map, ymap, p);
  return cudaGetLastError();
}

// Tiles of 128 features x 256 tokens, or x 128 tokens when the 256-token
// tiling leaves SMs idle (e.g. M = 512, N = 4096: 64 tiles on 148 SMs); the
// narrower tile dequantizes each weight tile twice as often per token but
// keeps every SM busy.
cudaError_t gemm(const MatArgs& a, cudaStream_t stream) {
  const int64_t tiles256 = ((a.M + 255) / 256) * ((a.N + kGemmRows - 1) / kGemmRows);
  const bool narrow = tiles256 < device_sm_count();
  switch (a.fmt) {
    case kQ4_0: return narrow ? gemm_launch<kQ4_0, 128>(a, stream) : gemm_launch<kQ4_0, 256>(a, stream);
    case kQ8_0: return narrow ? gemm_launch<kQ8_0, 128>(a, stream) : gemm_launch<kQ8_0, 256>(a, stream);
    case kQ6_K: return narrow ? gemm_launch<kQ6_K, 128>(a, stream) : gemm_launch<kQ6_K, 256>(a, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace spiral
