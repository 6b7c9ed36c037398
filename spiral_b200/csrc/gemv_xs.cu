// gemv_xs.cu — activation-stationary dequant-GEMV (decode, M <= 8) on
// sm_100a: the fast path of the quantized MUL_MAT (reference unpack_mmul,
// src/quants/q4_0/mmul.aie.h:16-90, q8_0/mmul.aie.h:16-117,
// q6_k/mmul.aie.h:18-84) for Q4_0 / Q8_0 at K in {1536, 2048, 3072, 4096}
// and Q6_K at K = 4096 (K = NW warps x GPW decode groups, NW = 16 or 12):
//
//   y[m][n] = sum_k bf16(W[n][k]) * x[m][k]      (fp32 accumulate)
//
// Structure (one persistent CTA per SM: NW consumer warps, a producer and a
// reducer warp):
//  * A tile is 16 output features; tiles are dealt to CTAs round-robin.
//    The producer warp streams the weights: 8 of its lanes each issue one
//    1-D bulk copy of a pair of consecutive rows (rows are contiguous in the
//    dense GGUF tensor; one copy per row when the row stride is padded) into
//    a ring of stages.  It is a warp of its own because issuing bulk copies
//    stalls the issuing warp while many are in flight (a consumer that
//    issued them held every reduction back by microseconds).  Pairs sit at a pitch
//    of 2 rows + 16 bytes, and MMA row g (g + 8) is weight row 2g (2g + 1),
//    so the 8 rows a fragment load touches lie in different banks.
//  * Warp w owns the fixed K slice [w*K/NW, (w+1)*K/NW) of every tile.  Its
//    activation fragments (the B operands of all its mma.sync.m16n8k16 steps)
//    are loaded once, at kernel start, straight from global x into registers
//    (bf16, the exact inputs: nothing is converted).  Per tile the warp
//    decodes its slice with the exact decoders of gemv_decode.cuh (A
//    fragments hold bf16_rne(d * q), bit for bit the standalone dequant) and
//    the NW warps' partial 16x8 tiles are summed in warp order by a reducer
//    warp of its own through a double-buffered shared array, handed over with
//    mbarriers, so decoding warps never wait for a reduction (reductions done
//    by rotating sets of the decoding warps cost about 0.3 us per tile: the
//    tile's last partial waited for the previous tile's reducers).
// The summation order depends on K alone, so every row gets the same bits
// whatever its position, shard or tile count (the row-sharded call with the
// all-gather fused in equals the single-GPU call bit for bit).
#include <atomic>

#include "api_internal.h"
#include "common.cuh"
#include "gemv_decode.cuh"

namespace spiral {
namespace {

// NW consumer warps (16, or 12 for K of 12 decode groups: 1536 / 3072): warp
// w owns K slice w; then the producer and the reducer warp.
template <int NW>
struct XsWarps {
  static constexpr int kProducer = NW, kReducer = NW + 1;
  static constexpr int kThreads = (NW + 2) * 32;
  static constexpr int kRedBytes = 2 * NW * 32 * 16;
  // 18 warps spread 5 + 5 + 4 + 4 over the sub-partitions: 96 registers per
  // thread is the most that launches; 14 warps (4 + 4 + 3 + 3) allow 128
  static constexpr int kMaxRegs = NW > 14 ? 96 : 128;
};
constexpr int kXsRows = 16;  // tile height (MMA M)
constexpr int kXsMaxStages = 8;
constexpr int kXsHeader = 2048;  // barriers and abort word; gathered-tile staging at 1024
constexpr int kXsRedBytes = 2 * 16 * 32 * 16;  // the largest (NW = 16)
constexpr int kXsBarConsumers = 1;  // named barrier of the consumer warps

struct XsParams {
  const uint8_t* w;
  int64_t w_stride;
  const uint16_t* x;
  int64_t x_s8, x_sm;
  void* y;
  int64_t y_s8, y_sm;
  int64_t N;
  int M, K;
  int row_bytes, pair_pitch, stages, pair_copies;
  int y_bf16, accumulate, static_weights;
  // gathered output (the exchange protocol of gemv.cu, api_internal.h)
  uint8_t* const* xchg_peers;
  int64_t n_offset, n_total;
  int rank, world;
};

__device__ __forceinline__ uint32_t xchg_flag_xs(uint32_t calls) { return calls | 0x80000000u; }

// The step whose 4 activations follow step s's in k (its B fragment is the
// upper half of the same 16-byte load), or -1 when s is itself an upper half.
template <int FMT>
__host__ __device__ constexpr int xs_pair_step(int s) {
  return FMT == kQ4_0 ? (((s >> 1) & 1) == 0 ? s + 2 : -1)
                      : FMT == kQ8_0 ? ((s & 1) == 0 ? s + 1 : -1) : (((s >> 2) & 1) == 0 ? s + 4 : -1);
}

// Bounded wait that gives up at once when another warp already gave up (the
// abort word is read only when the phase is not complete yet).
__device__ __forceinline__ bool xs_wait(uint64_t* bar, uint32_t parity, int& abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  if (*(volatile int*)&abort_flag) return false;
  if (mbar_wait(bar, parity)) return true;
  abort_flag = 1;
  return false;
}

// Weight row of MMA row R of a tile.
__device__ __forceinline__ int xs_weight_row(int R) { return R < 8 ? 2 * R : 2 * (R - 8) + 1; }

template <int FMT, int GPW, bool GATHER, bool FTZ, int NW>
__global__ void __maxnreg__(XsWarps<NW>::kMaxRegs) gemv_xs_kernel(const XsParams p) {
  constexpr int kXsWarps = NW;
  constexpr int kXsWarpProducer = XsWarps<NW>::kProducer, kXsWarpReducer = XsWarps<NW>::kReducer;
  using F = GemvFmt<FMT>;
  constexpr int kSteps = F::kSteps;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kXsMaxStages;
  uint64_t* red_full = empty + kXsMaxStages;
  uint64_t* red_empty = red_full + 2;
  uint64_t* xready = red_empty + 2;  // every consumer warp holds its activation fragments
  // Set when a bounded wait gave up: later waits are skipped (not retried)
  // so every warp still reaches every named barrier and the kernel ends.
  int& abort_flag = *reinterpret_cast<int*>(smem + 248);
  float4* red = reinterpret_cast<float4*>(smem + kXsHeader);
  uint8_t* stages = smem + kXsHeader + kXsRedBytes;
  const int stage_bytes = 8 * p.pair_pitch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tiles = (p.N + kXsRows - 1) / kXsRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kXsWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&red_full[b], kXsWarps * 32);
      mbar_init(&red_empty[b], 32);
    }
    mbar_init(xready, kXsWarps);
    abort_flag = 0;
    fence_mbar_init();
    griddep_launch_dependents();
  }
  __syncthreads();

  if (warp == kXsWarpProducer) {
    // ---------------------------------------------------------- producer --
    // tile `it` of this CTA into stage it % stages, once every consumer warp
    // has finished the tile that used that stage before
    // Only the first two tiles are requested before the consumers have
    // loaded their activations: behind a full ring of weight copies those
    // small loads would wait for microseconds.
    if (!p.static_weights) griddep_wait();
    const uint64_t pol = l2_evict_first_policy();
    constexpr uint32_t kEarly = 2;
    uint32_t it = 0;
    for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
      const int s = static_cast<int>(it % p.stages);
      if (it == kEarly && lane == 0 && !*(volatile int*)&abort_flag && !mbar_wait(xready, 0)) abort_flag = 1;
      const int64_t n0 = tile * kXsRows;
      const int rows = static_cast<int>(::spiral::min64(kXsRows, p.N - n0));
      int go = 0;
      if (lane == 0) {
        go = !*(volatile int*)&abort_flag && mbar_wait(&empty[s], ((it / p.stages) & 1u) ^ 1u);
        if (go) {
          mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(p.row_bytes) * rows);
        } else {
          abort_flag = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      uint8_t* dst = stages + s * stage_bytes;
      const uint8_t* src = p.w + n0 * p.w_stride;
      if (p.pair_copies) {
        // lane q < 8: rows 2q and 2q + 1 (contiguous), or 2q alone at the end
        const int rq = rows - 2 * lane;
        if (lane < 8 && rq > 0)
          bulk_g2s(dst + lane * p.pair_pitch, src + 2 * lane * p.w_stride,
                   static_cast<uint32_t>(p.row_bytes) * (rq >= 2 ? 2u : 1u), &full[s], pol);
      } else if (lane < rows) {
        bulk_g2s(dst + (lane >> 1) * p.pair_pitch + (lane & 1) * p.row_bytes, src + lane * p.w_stride,
                 static_cast<uint32_t>(p.row_bytes), &full[s], pol);
      }
    }
    // Every issued copy must land before the CTA may exit (after an abort
    // the consumers stop waiting for them).
    if (lane == 0) {
      const uint32_t first = it > static_cast<uint32_t>(p.stages) ? it - p.stages : 0u;
      for (uint32_t i = first; i < it; ++i) mbar_wait(&full[i % p.stages], (i / p.stages) & 1u);
    }
    return;
  }

  // ------------------------------------------------------------ consumers --
  griddep_wait();  // activations may come from the preceding kernel
  uint32_t calls = 0u;
  if constexpr (GATHER) calls = *reinterpret_cast<volatile const uint32_t*>(p.xchg_peers[p.rank]);
  const int r = lane >> 2, c = lane & 3;

  const int ntiles = static_cast<int>(tiles);
  if (warp == kXsWarpReducer) {
    // ---------------------------------------------------------- reducer --
    // Lane l sums the 16 warps' float4 partials of fragment lane l in warp
    // order: outputs (rows r, r + 8 of MMA row r = l / 4) x (vectors
    // 2 (l % 4), + 1).
    uint16_t* tile_out = reinterpret_cast<uint16_t*>(smem + 1024);  // [8][16] bf16
    for (int tile = blockIdx.x, local = 0; tile < ntiles; tile += gridDim.x, ++local) {
      const int rbuf = local & 1;
      xs_wait(&red_full[rbuf], static_cast<uint32_t>(local >> 1) & 1u, abort_flag);
      const float4* rp = red + rbuf * kXsWarps * 32 + lane;
      float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kXsWarps; ++w) {
        const float4 v = rp[w * 32];
        sum.x += v.x;
        sum.y += v.y;
        sum.z += v.z;
        sum.w += v.w;
      }
      mbar_arrive(&red_empty[rbuf]);
      const float sums[4] = {sum.x, sum.y, sum.z, sum.w};
      if constexpr (GATHER) {
        // the tile's bf16 outputs, [m][16 rows], then 16-byte pieces to the
        // local output and flagged unit pairs to every other rank's slot
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int row = xs_weight_row((lane >> 2) + 8 * (j >> 1));
          const int m = 2 * (lane & 3) + (j & 1);
          tile_out[m * kXsRows + row] = static_cast<uint16_t>(pack_bf16x2(sums[j], 0.f) & 0xFFFFu);
        }
        __syncwarp();
        const int64_t r0 = static_cast<int64_t>(tile) * kXsRows;
        const int local_items = p.M * 2;
        const int items = *(volatile int*)&abort_flag ? local_items : local_items + p.M * 4 * (p.world - 1);
        for (int q = lane; q < items; q += 32) {
          if (q < local_items) {
            const int half = q & 1, mm = q >> 1;
            if (r0 + half * 8 + 8 > p.N) continue;
            *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.y) + static_cast<int64_t>(mm) * p.y_sm + p.n_offset +
                                      r0 + half * 8) = *reinterpret_cast<const uint4*>(tile_out + mm * kXsRows + half * 8);
          } else {
            const int qq = q - local_items;
            const int piece = qq & 3, mm = (qq >> 2) % p.M, k = (qq >> 2) / p.M;
            if (r0 + piece * 4 + 4 > p.N) continue;
            const int rr = k < p.rank ? k : k + 1;
            const uint2 d = *reinterpret_cast<const uint2*>(tile_out + mm * kXsRows + piece * 4);
            const uint64_t hi = static_cast<uint64_t>(xchg_flag_xs(calls)) << 32;
            const int64_t col = p.n_offset + r0 + piece * 4;
            uint8_t* dst = p.xchg_peers[rr] + kGemvXchgCtrlBytes + (calls & 1) * gemv_xchg_slot_bytes(p.n_total) +
                           mm * 4 * p.n_total + col * 4;
            asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(hi | d.x), "l"(hi | d.y)
                         : "memory");
          }
        }
        __syncwarp();
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int row = xs_weight_row((lane >> 2) + 8 * (j >> 1));
          const int m = 2 * (lane & 3) + (j & 1);
          const int64_t n = static_cast<int64_t>(tile) * kXsRows + row;
          if (m < p.M && n < p.N) {
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


  // This warp's activation fragments: for its groups g (global index
  // warp * GPW + g) and steps s, lane (r, c) holds x[r][4 consecutive k at
  // group start + xk(s, c)] (bf16x4) for vector r < M, zero otherwise.  Two
  // steps' fragments are one aligned 16-byte load; all loads are issued
  // before any is used (one round trip), then the producer is told.
  uint2 Bx[GPW][kSteps];
  {
    const bool vec = (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0 && (p.x_s8 & 7) == 0 && (p.x_sm & 7) == 0;
#pragma unroll
    for (int g = 0; g < GPW; ++g) {
#pragma unroll
      for (int s = 0; s < kSteps; ++s) {
        const int s2 = xs_pair_step<FMT>(s);
        if (s2 < 0) continue;  // filled with its lower half
        const int k = (warp * GPW + g) * F::kGroupK + GroupDecoder<FMT>::xk(s, c);  // k % 8 == 0
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
        Bx[g][s] = make_uint2(v.x, v.y);
        Bx[g][s2] = make_uint2(v.z, v.w);
      }
    }
    // arrive only once every load has returned (the values feed `dep`)
    uint32_t dep = 0u;
#pragma unroll
    for (int g = 0; g < GPW; ++g)
#pragma unroll
      for (int s = 0; s < kSteps; ++s) dep ^= Bx[g][s].x ^ Bx[g][s].y;
    asm volatile("" ::"r"(dep) : "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(xready);
  }

  // MMA row r = weight row 2r (pair r, first row); row r + 8 = 2r + 1
  const uint8_t* ra0 = stages + r * p.pair_pitch + warp * GPW * F::kGroupBytes;
  int stage = 0;
  uint32_t phase = 0u;
  for (int tile = blockIdx.x, local = 0; tile < ntiles; tile += gridDim.x, ++local) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const int s = stage;
    if (xs_wait(&full[s], phase, abort_flag)) {
      const uint8_t* ra = ra0 + s * stage_bytes;
      const uint8_t* rb = ra + p.row_bytes;
#pragma unroll
      for (int g = 0; g < GPW; ++g) {
        const uint8_t* ga = ra + g * F::kGroupBytes;
        const uint8_t* gb = rb + g * F::kGroupBytes;
        auto bx = [&](int st) { return Bx[g][st]; };
        if constexpr (FMT == kQ6_K) {
          // a 210-byte super-block starts 2 mod 4 when its index is odd
          GroupDecoder<FMT>::run_b(ga, gb, c, bx, FTZ, acc, ((warp * GPW + g) & 1) ? 16u : 0u);
        } else {
          GroupDecoder<FMT>::run_b(ga, gb, c, bx, FTZ, acc);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++stage == p.stages) {
      stage = 0;
      phase ^= 1u;
    }

    // hand the partial to the reducer warp
    const int rbuf = local & 1;
    if (local >= 2) xs_wait(&red_empty[rbuf], static_cast<uint32_t>((local >> 1) - 1) & 1u, abort_flag);
    red[(rbuf * kXsWarps + warp) * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    mbar_arrive(&red_full[rbuf]);
  }

  if constexpr (GATHER) {
    // Receive, exactly as the pipelined GEMV does (gemv.cu): poll the other
    // ranks' pieces in this rank's slot (bounded) and copy them to y; the
    // last CTA advances the call count.
    const int64_t pieces_per_row = p.n_total / 4;
    const int64_t total = static_cast<int64_t>(p.M) * pieces_per_row;
    const uint8_t* slot = p.xchg_peers[p.rank] + kGemvXchgCtrlBytes + (calls & 1) * gemv_xchg_slot_bytes(p.n_total);
    const uint32_t flag = xchg_flag_xs(calls);
    bool ok = !*(volatile int*)&abort_flag && !(*(volatile uint32_t*)&g_device_error & kDevErrPeerTimeout);
    constexpr int kCons = kXsWarps * 32;
    for (int64_t q = static_cast<int64_t>(blockIdx.x) * kCons + threadIdx.x; ok && q < total;
         q += static_cast<int64_t>(gridDim.x) * kCons) {
      const int64_t mm = q / pieces_per_row, col = (q - mm * pieces_per_row) * 4;
      if (col >= p.n_offset && col < p.n_offset + p.N) continue;
      const uint8_t* src = slot + mm * 4 * p.n_total + col * 4;
      uint64_t a, b;
      const uint64_t t0 = globaltimer_ns();
      for (;;) {
        asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
        if (static_cast<uint32_t>(a >> 32) == flag && static_cast<uint32_t>(b >> 32) == flag) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          raise_device_error(kDevErrPeerTimeout);
          ok = false;
          break;
        }
      }
      if (ok) {
        *reinterpret_cast<uint2*>(static_cast<uint16_t*>(p.y) + mm * p.y_sm + col) =
            make_uint2(static_cast<uint32_t>(a), static_cast<uint32_t>(b));
      }
    }
    named_bar_sync(kXsBarConsumers, kCons);
    if (threadIdx.x == 0) {
      uint32_t* ctrl = reinterpret_cast<uint32_t*>(p.xchg_peers[p.rank]);
      uint32_t before;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(before) : "l"(ctrl + 1) : "memory");
      if (before == gridDim.x - 1) {
        ctrl[1] = 0u;
        ctrl[0] = calls + 1u;
      }
    }
  }
}

// Consumer warps and groups per warp (K = NW warps x GPW groups of kGroupK);
// false = not served here.
bool xs_shape(const MatArgs& a, int* nw, int* gpw) {
  const int gk = a.fmt == kQ6_K ? 256 : 128;
  if (a.fmt != kQ4_0 && a.fmt != kQ8_0 && a.fmt != kQ6_K) return false;
  if (a.K % gk != 0) return false;
  const int64_t groups = a.K / gk;
  const int max_gpw = a.fmt == kQ6_K ? 1 : 2;
  for (int w : {16, 12}) {
    if (groups % w == 0 && groups / w <= max_gpw) {
      *nw = w;
      *gpw = static_cast<int>(groups / w);
      return true;
    }
  }
  return false;
}

struct XsPlan {
  int nw = 0, gpw = 0, row_bytes = 0, pair_pitch = 0, stages = 0;
  size_t smem = 0;
};

bool xs_plan(const MatArgs& a, XsPlan* out) {
  if (a.M < 1 || a.M > 8) return false;
  int nw = 0, gpw = 0;
  if (!xs_shape(a, &nw, &gpw)) return false;
  if (reinterpret_cast<uintptr_t>(a.w) % 16 != 0 || a.w_stride % 16 != 0) return false;
  const int bk = a.fmt == kQ6_K ? 256 : 32, bb = a.fmt == kQ4_0 ? 18 : (a.fmt == kQ8_0 ? 34 : 210);
  const int row_bytes = static_cast<int>(a.K / bk) * bb;  // a multiple of 16 for the K served
  const int pair_pitch = 2 * row_bytes + 16;              // +16: pairs on different banks
  const size_t fixed = kXsHeader + kXsRedBytes;
  const size_t avail = device_max_smem_optin();
  const size_t stage = size_t(8) * pair_pitch;
  if (fixed + 2 * stage > avail) return false;
  out->nw = nw;
  out->gpw = gpw;
  out->row_bytes = row_bytes;
  out->pair_pitch = pair_pitch;
  out->stages = static_cast<int>(std::min<size_t>(kXsMaxStages, (avail - fixed) / stage));
  out->smem = fixed + static_cast<size_t>(out->stages) * stage;
  return true;
}

template <int FMT, int GPW, int NW>
cudaError_t xs_launch_t(const XsParams& p, bool gather, bool ftz, size_t smem, cudaStream_t stream) {
  auto* kernel = gather ? (ftz ? gemv_xs_kernel<FMT, GPW, true, true, NW> : gemv_xs_kernel<FMT, GPW, true, false, NW>)
                        : (ftz ? gemv_xs_kernel<FMT, GPW, false, true, NW> : gemv_xs_kernel<FMT, GPW, false, false, NW>);
  int dev = 0;
  cudaGetDevice(&dev);
  const int fslot = FMT == kQ4_0 ? 0 : (FMT == kQ8_0 ? 1 : 2);
  const int slot = (((fslot * 2 + (GPW - 1)) * 2 + gather) * 2 + ftz) * 2 + (NW == 16 ? 0 : 1);
  static std::atomic<bool> configured[64][48];
  if (!configured[dev & 63][slot].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(device_max_smem_optin()));
    if (e != cudaSuccess) return e;
    configured[dev & 63][slot].store(true, std::memory_order_release);
  }
  const int64_t tiles = (p.N + kXsRows - 1) / kXsRows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(tiles, int64_t(device_sm_count()))));
  cfg.blockDim = dim3(XsWarps<NW>::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

}  // namespace

bool gemv_xs_ok(const MatArgs& a) {
  XsPlan plan;
  return xs_plan(a, &plan);
}

cudaError_t gemv_xs(const MatArgs& a, const PeerOut* po, cudaStream_t stream) {
  XsPlan plan;
  if (!xs_plan(a, &plan)) return cudaErrorNotSupported;
  XsParams p{};
  p.w = a.w;
  p.w_stride = a.w_stride;
  p.x = a.x;
  p.x_s8 = a.x_s8;
  p.x_sm = a.x_sm;
  p.y = a.y;
  p.y_s8 = a.y_s8;
  p.y_sm = a.y_sm;
  p.N = a.N;
  p.M = static_cast<int>(a.M);
  p.K = static_cast<int>(a.K);
  p.row_bytes = plan.row_bytes;
  p.pair_pitch = plan.pair_pitch;
  p.stages = plan.stages;
  p.pair_copies = a.w_stride == plan.row_bytes;
  p.y_bf16 = a.y_bf16;
  p.accumulate = a.accumulate;
  p.static_weights = a.static_weights;
  if (po != nullptr) {
    p.xchg_peers = po->xchg_peers;
    p.n_offset = po->n_offset;
    p.n_total = po->n_total;
    p.rank = po->rank;
    p.world = po->world;
  }
  const bool gather = po != nullptr;
  const bool w16 = plan.nw == 16;
  switch (a.fmt) {
    case kQ4_0:
      if (plan.gpw == 1)
        return w16 ? xs_launch_t<kQ4_0, 1, 16>(p, gather, a.ftz, plan.smem, stream)
                   : xs_launch_t<kQ4_0, 1, 12>(p, gather, a.ftz, plan.smem, stream);
      return w16 ? xs_launch_t<kQ4_0, 2, 16>(p, gather, a.ftz, plan.smem, stream)
                 : xs_launch_t<kQ4_0, 2, 12>(p, gather, a.ftz, plan.smem, stream);
    case kQ8_0:
      if (plan.gpw == 1)
        return w16 ? xs_launch_t<kQ8_0, 1, 16>(p, gather, a.ftz, plan.smem, stream)
                   : xs_launch_t<kQ8_0, 1, 12>(p, gather, a.ftz, plan.smem, stream);
      return w16 ? xs_launch_t<kQ8_0, 2, 16>(p, gather, a.ftz, plan.smem, stream)
                 : xs_launch_t<kQ8_0, 2, 12>(p, gather, a.ftz, plan.smem, stream);
    case kQ6_K:
      return w16 ? xs_launch_t<kQ6_K, 1, 16>(p, gather, a.ftz, plan.smem, stream)
                 : xs_launch_t<kQ6_K, 1, 12>(p, gather, a.ftz, plan.smem, stream);
  }
  return cudaErrorNotSupported;
}

}  // namespace spiral
