// gemv.cu — fused dequant-GEMV (decode, M <= 8 activation vectors) for sm_100a.
//
// B200 counterpart of the reference's fused unpack_mmul
// (src/quants/q4_0/mmul.aie.h:16-90, q8_0/mmul.aie.h:16-117,
// q6_k/mmul.aie.h:18-84): out[m][n] = sum_k in[m][k] * bf16(W[n][k]) with
// fp32 accumulation.  Weights stream from HBM exactly once.
//
// Structure (one persistent CTA per SM; two consumer groups of 8 warps plus
// one producer warp):
//  * A tile is 16 output features (one m16 MMA row block).  Tiles are dealt to
//    CTAs round-robin, and inside a CTA to its consumer groups round-robin, so
//    two tiles are being decoded while the producer prefetches the next ones.
//  * A pipeline stage holds the tile's rows over a K chunk (the whole row
//    whenever it fits, so one stage per tile).  The producer lane fills it
//    with one 1-D bulk (TMA) copy per row into a padded row pitch, completion
//    counted in bytes on an mbarrier; weights use an L2 evict-first policy.
//  * Consumer warp w of a group decodes the K groups w, w+8, ... of the stage
//    in registers straight into bf16 A fragments of mma.sync.m16n8k16 (rows
//    = features, n = 8 activation vectors, padded) and accumulates in fp32.
//    At the end of a tile the group's 8 partial 16x8 tiles are summed in a
//    fixed order (deterministic) and stored.
//  * Activations are staged once per CTA in shared memory in a k order
//    permuted to match each lane's A fragment, so a B fragment is one 8-byte
//    shared load.  The MMA contracts over k, so permuting k identically in A
//    and B leaves the sum unchanged.
//  * Programmatic dependent launch: each CTA lets the next kernel on the
//    stream launch at once, and reads activations / writes outputs only after
//    griddepcontrol.wait (the preceding kernel has completed).  With
//    SPIRAL_FLAG_STATIC_WEIGHTS the producer streams weights before that
//    wait, so this launch's ramp-up overlaps the previous kernel's tail.
//
// Dequantization (exact): a quant byte is placed in the mantissa of an fp32
// with one byte permute, f = 1 + q*2^-s, and one fused multiply-add computes
// f*(2^s*d) - (2^s + bias)*d = (q - bias)*d.  Both constants are exact in
// fp32 (at most 24 significant bits) and so is the result, so the FMA does
// not round; cvt.rn.bf16x2.f32 then rounds once to nearest even.  The A
// fragments therefore hold exactly the bf16 weights of the standalone
// dequant (bf16_rne(d*int), up to the sign of a zero weight, which cannot
// change a dot product), and the GEMV differs from the reference's
// dequant-then-fp32-matmul only by fp32 summation order.  Pairs of weights
// go through one fma.rn.f32x2.
#include <atomic>

#include "api_internal.h"
#include "decode.cuh"
#include "gemv_decode.cuh"
#include "gemv_generic.cuh"

namespace spiral {

constexpr int kGroupsPerCta = 2;  // consumer groups
constexpr int kWarpsPerGroup = 8;
constexpr int kConsumerWarps = kGroupsPerCta * kWarpsPerGroup;
constexpr int kGemvThreads = (kConsumerWarps + 1) * 32;
constexpr int kTileRows = 16;
constexpr int kBarrierBytes = 256;  // up to 15 mbarrier pairs + the abort word
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
  int chunk_groups;  // groups per full chunk
  int chunks_per_row;
  int stages;
  int row_pitch;  // bytes per row slot in a stage
  int x_pitch;    // bytes per activation vector in the permuted copy
  int y_bf16, accumulate, ftz;
  int static_weights;  // weights may be read before the preceding grid ends
  // Rows whose address or stride is not 16-byte aligned (e.g. Q6_K at
  // K = 1536: 1260-byte rows): each row is copied as the 16-byte aligned
  // window that holds it, and read at its offset inside the window.  The
  // window's extra bytes lie in the same 16-byte granules as the row's first
  // and last bytes, so they never reach another page.
  int window;
  // Gathered output (world > 0): y is this rank's full bf16 output
  // [M][y_sm]; the shard's rows are columns n_offset + n of it, and every
  // rank's exchange buffer (xchg_peers[r]) receives them as flagged units.
  uint8_t* const* xchg_peers;
  int64_t n_offset, n_total;
  int rank, world;
};

// Exchange buffer layout: kGemvXchgCtrlBytes / gemv_xchg_slot_bytes
// (api_internal.h).
constexpr int64_t kXchgCtrlBytes = kGemvXchgCtrlBytes;
__host__ __device__ constexpr int64_t xchg_slot_bytes(int64_t n_total) { return gemv_xchg_slot_bytes(n_total); }

__device__ __forceinline__ uint32_t xchg_flag(uint32_t calls) { return calls | 0x80000000u; }

__device__ __forceinline__ void st_pair_sys(uint8_t* dst, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(a), "l"(b) : "memory");
}

__device__ __forceinline__ void ld_pair_sys(const uint8_t* src, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
}

// ------------------------------------------------- activation staging ----

// Permuted activations: entry (m, group g, step s, lane column c) holds the
// 4 consecutive k that lane column c contracts at that step, at
//   xs + m*x_pitch + (g*kSteps + s)*32 + c*8.
// Fast path (contiguous 16-byte aligned rows, K <= kRawK): every thread loads
// its 16-byte pieces of all M rows at once (one L2 round trip), then row by
// row the raw copy goes through `raw` (the idle reduction buffer) and is
// permuted from there.  Otherwise each entry gathers from global memory.
constexpr int kRawK = kRedBytes / 2;
constexpr int kStageThreads = kConsumerWarps * 32;
constexpr int kRawPieces = (kRawK / 8 + kStageThreads - 1) / kStageThreads;

template <int FMT>
__device__ void stage_x(const GemvParams& p, uint8_t* xs, uint8_t* raw, int tid) {
  using F = GemvFmt<FMT>;
  constexpr int kStepShift = F::kSteps == 8 ? 3 : 4;
  const int per_m = static_cast<int>(p.K / F::kGroupK) * F::kSteps * 4;
  const bool fast = p.x_s8 == 8 && p.K <= kRawK && (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0 &&
                    (p.x_sm & 7) == 0;
  if (fast) {
    const int pieces = static_cast<int>(p.K / 8);  // 16-byte pieces per row
    uint4 v[8][kRawPieces];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
#pragma unroll
      for (int i = 0; i < kRawPieces; ++i) {
        const int q = tid + i * kStageThreads;
        if (m < p.M && q < pieces)
          v[m][i] = __ldg(reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(m) * p.x_sm) + q);
      }
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      if (m < p.M) {
#pragma unroll
        for (int i = 0; i < kRawPieces; ++i) {
          const int q = tid + i * kStageThreads;
          if (q < pieces) reinterpret_cast<uint4*>(raw)[q] = v[m][i];
        }
        named_bar_sync(kGroupsPerCta + 1, kStageThreads);
        const uint16_t* xr = reinterpret_cast<const uint16_t*>(raw);
        uint8_t* dst = xs + static_cast<int64_t>(m) * p.x_pitch;
        for (int e = tid; e < per_m; e += kStageThreads) {
          const int c = e & 3, gs = e >> 2, st = gs & (F::kSteps - 1), g = gs >> kStepShift;
          const int k = g * F::kGroupK + GroupDecoder<FMT>::xk(st, c);
          *reinterpret_cast<uint2*>(dst + gs * 32 + c * 8) =
              make_uint2(xr[k] | (static_cast<uint32_t>(xr[k + 1]) << 16),
                         xr[k + 2] | (static_cast<uint32_t>(xr[k + 3]) << 16));
        }
        named_bar_sync(kGroupsPerCta + 1, kStageThreads);
      }
    }
    return;
  }
  const int64_t total = static_cast<int64_t>(p.M) * per_m;
  for (int64_t e = tid; e < total; e += kStageThreads) {
    const int m = static_cast<int>(e / per_m);
    const int em = static_cast<int>(e - static_cast<int64_t>(m) * per_m);
    const int c = em & 3, gs = em >> 2, st = gs & (F::kSteps - 1), g = gs >> kStepShift;
    const int64_t k = static_cast<int64_t>(g) * F::kGroupK + GroupDecoder<FMT>::xk(st, c);
    const uint16_t* base = p.x + static_cast<int64_t>(m) * p.x_sm;
    uint32_t v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = base[((k + j) >> 3) * p.x_s8 + ((k + j) & 7)];
    *reinterpret_cast<uint2*>(xs + static_cast<int64_t>(m) * p.x_pitch + gs * 32 + c * 8) =
        make_uint2(v[0] | (v[1] << 16), v[2] | (v[3] << 16));
  }
}

// --------------------------------------------------------------- kernel ---

// GATHER: the row-sharded call with the all-gather fused in (p.world > 0);
// a separate instantiation so the plain GEMV carries none of its code.
// FTZ: the flush of subnormal scales, fixed at compile time so the decode
// loop carries no test for it (p.ftz is not read).
template <int FMT, bool GATHER, bool FTZ>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const GemvParams p) {
  using F = GemvFmt<FMT>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + p.stages;
  // Set when a bounded wait gave up: later waits are skipped (not retried) so
  // every warp still reaches every named barrier and the kernel ends.
  int& abort_flag = *reinterpret_cast<int*>(smem + kBarrierBytes - 8);
  float4* red = reinterpret_cast<float4*>(smem + kBarrierBytes);
  uint8_t* xs = smem + kBarrierBytes + kRedBytes;
  uint8_t* stages = xs + static_cast<int64_t>(p.M) * p.x_pitch;
  const int stage_bytes = kTileRows * p.row_pitch;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t tiles = (p.N + kTileRows - 1) / kTileRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarpsPerGroup);
    }
    abort_flag = 0;
    fence_mbar_init();
    griddep_launch_dependents();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------- producer ----
    if (lane == 0) {
      if (!p.static_weights) griddep_wait();
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
          const int64_t g0 = static_cast<int64_t>(ch) * p.chunk_groups;
          const int ng = static_cast<int>(::spiral::min64(p.chunk_groups, p.groups_per_row - g0));
          const uint32_t bytes = static_cast<uint32_t>(ng * F::kGroupBytes);
          uint8_t* dst = stages + s * stage_bytes;
          const uint8_t* src = src_tile + g0 * F::kGroupBytes;
          if (p.window) {
            uint32_t total = 0;
            for (int r = 0; r < rows; ++r) {
              const uint32_t off = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(src + r * p.w_stride) & 15u);
              total += (off + bytes + 15u) & ~15u;
            }
            mbar_arrive_expect_tx(&full[s], total);
            for (int r = 0; r < rows; ++r) {
              const uint8_t* row = src + r * p.w_stride;
              const uint32_t off = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(row) & 15u);
              bulk_g2s(dst + r * p.row_pitch, row - off, (off + bytes + 15u) & ~15u, &full[s], pol);
            }
          } else {
            mbar_arrive_expect_tx(&full[s], bytes * rows);
            for (int r = 0; r < rows; ++r)
              bulk_g2s(dst + r * p.row_pitch, src + r * p.w_stride, bytes, &full[s], pol);
          }
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
  griddep_wait();  // activations may come from the preceding kernel
  // calls completed on this rank: the parity and flag of this gathered call
  uint32_t calls = 0u;
  if constexpr (GATHER) calls = *reinterpret_cast<volatile const uint32_t*>(p.xchg_peers[p.rank]);
  stage_x<FMT>(p, xs, reinterpret_cast<uint8_t*>(red), threadIdx.x);
  named_bar_sync(kGroupsPerCta + 1, kConsumerWarps * 32);

  const int grp = warp / kWarpsPerGroup, gw = warp % kWarpsPerGroup;
  const int r = lane >> 2, c = lane & 3;
  const int mx = r < p.M ? r : 0;  // vectors >= M read vector 0; their columns are discarded
  const uint8_t* xcol = xs + static_cast<int64_t>(mx) * p.x_pitch + c * 8;
  float4* gred = red + grp * kWarpsPerGroup * 32;
  int64_t local = 0;  // tile index within this CTA
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++local) {
    if (local % kGroupsPerCta != grp) continue;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    uint32_t it = static_cast<uint32_t>(local * p.chunks_per_row);
    for (int ch = 0; ch < p.chunks_per_row; ++ch, ++it) {
      const int s = static_cast<int>(it % p.stages);
      const uint32_t ph = (it / p.stages) & 1u;
      bool ready = false;
      if (!*(volatile int*)&abort_flag) {
        ready = mbar_wait(&full[s], ph);
        if (!ready) abort_flag = 1;
      }
      const int64_t g0 = static_cast<int64_t>(ch) * p.chunk_groups;
      const int ng = static_cast<int>(::spiral::min64(p.chunk_groups, p.groups_per_row - g0));
      if (ready) {
        const uint8_t* st = stages + s * stage_bytes;
        const uint8_t* ra = st + r * p.row_pitch;
        const uint8_t* rb = st + (r + 8) * p.row_pitch;
        if (p.window) {  // the row's offset inside its window (rows past N: any)
          const uint8_t* row0 = p.w + tile * kTileRows * p.w_stride;
          ra += reinterpret_cast<uintptr_t>(row0 + r * p.w_stride) & 15u;
          rb += reinterpret_cast<uintptr_t>(row0 + (r + 8) * p.w_stride) & 15u;
        }
        auto decode = [&](int gl) {
          const uint8_t* xg = xcol + (g0 + gl) * F::kSteps * 32;
          if constexpr (FMT == kQ6_K) {
            GroupDecoder<FMT>::run(ra + gl * F::kGroupBytes, rb + gl * F::kGroupBytes, c, xg, FTZ, acc,
                                   (gl & 1) ? 16u : 0u);
          } else {
            GroupDecoder<FMT>::run(ra + gl * F::kGroupBytes, rb + gl * F::kGroupBytes, c, xg, FTZ, acc);
          }
        };
        // groups gw, gw + 8, ... < ng, two per iteration so the second
        // group's decode overlaps the first one's MMAs
        int gl = gw;
        for (; gl + kWarpsPerGroup < ng; gl += 2 * kWarpsPerGroup) {
          decode(gl);
          decode(gl + kWarpsPerGroup);
        }
        if (gl < ng) decode(gl);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    gred[gw * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    named_bar_sync(1 + grp, kWarpsPerGroup * 32);
    if (gw < 4) {
      const int t = gw * 32 + lane;  // 0..127: one output each
      const int l = t >> 2, j = t & 3;
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kWarpsPerGroup; ++w) sum += reinterpret_cast<const float*>(&gred[w * 32 + l])[j];
      const int row = (l >> 2) + 8 * (j >> 1);
      const int m = 2 * (l & 3) + (j & 1);
      const int64_t n = tile * kTileRows + row;
      if constexpr (GATHER) {
        // Gathered output: the tile's bf16 outputs are collected in shared
        // memory (the reduction slots, free once every sum is read) as
        // [m][16 rows]; 16-byte pieces then go to the local output and, as
        // flagged unit pairs, to every other rank's exchange slot.  Shards
        // are multiples of 8 rows, so a piece is either whole or absent.
        uint16_t* tile_out = reinterpret_cast<uint16_t*>(gred);
        named_bar_sync(kGroupsPerCta + 2 + grp, 128);
        tile_out[m * kTileRows + row] = static_cast<uint16_t>(pack_bf16x2(sum, 0.f) & 0xFFFFu);
        named_bar_sync(kGroupsPerCta + 2 + grp, 128);
        const int64_t r0 = tile * kTileRows;
        const int local_items = p.M * 2;
        const int items = *(volatile int*)&abort_flag ? local_items : local_items + p.M * 4 * (p.world - 1);
        for (int it = t; it < items; it += 128) {
          if (it < local_items) {
            const int half = it & 1, mm = it >> 1;
            if (r0 + half * 8 + 8 > p.N) continue;
            *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.y) + static_cast<int64_t>(mm) * p.y_sm + p.n_offset +
                                      r0 + half * 8) =
                *reinterpret_cast<const uint4*>(tile_out + mm * kTileRows + half * 8);
          } else {
            const int q = it - local_items;
            const int piece = q & 3, mm = (q >> 2) % p.M, k = (q >> 2) / p.M;
            if (r0 + piece * 4 + 4 > p.N) continue;
            const int rr = k < p.rank ? k : k + 1;
            const uint2 d = *reinterpret_cast<const uint2*>(tile_out + mm * kTileRows + piece * 4);
            const uint64_t hi = static_cast<uint64_t>(xchg_flag(calls)) << 32;
            const int64_t col = p.n_offset + r0 + piece * 4;
            st_pair_sys(p.xchg_peers[rr] + kXchgCtrlBytes + (calls & 1) * xchg_slot_bytes(p.n_total) +
                            mm * 4 * p.n_total + col * 4,
                        hi | d.x, hi | d.y);
          }
        }
      } else if (m < p.M && n < p.N) {
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
    named_bar_sync(1 + grp, kWarpsPerGroup * 32);
  }
  if constexpr (GATHER) {
    // Receive: the grid's consumer threads poll the other ranks' pieces of
    // the output in this rank's exchange slot (bounded) and copy them to the
    // local output; the grid completes only once the whole gathered output
    // is local, so stream order alone covers every later reader.  Every CTA
    // has sent all its pieces before it polls, and the grid (one CTA per SM)
    // is co-resident, so the waits cannot cycle.
    const int64_t pieces_per_row = p.n_total / 4;
    const int64_t total = static_cast<int64_t>(p.M) * pieces_per_row;
    const uint8_t* slot = p.xchg_peers[p.rank] + kXchgCtrlBytes + (calls & 1) * xchg_slot_bytes(p.n_total);
    const uint32_t flag = xchg_flag(calls);
    // After a rank failed to arrive the ranks' call counts no longer agree:
    // later calls skip their waits (the error stays set until the host reads
    // it) instead of each waiting out the limit.
    bool ok = !*(volatile int*)&abort_flag && !(*(volatile uint32_t*)&g_device_error & kDevErrPeerTimeout);
    for (int64_t q = static_cast<int64_t>(blockIdx.x) * kStageThreads + threadIdx.x; ok && q < total;
         q += static_cast<int64_t>(gridDim.x) * kStageThreads) {
      const int64_t mm = q / pieces_per_row, col = (q - mm * pieces_per_row) * 4;
      if (col >= p.n_offset && col < p.n_offset + p.N) continue;
      const uint8_t* src = slot + mm * 4 * p.n_total + col * 4;
      uint64_t a, b;
      const uint64_t t0 = globaltimer_ns();
      for (;;) {
        ld_pair_sys(src, a, b);
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
    // The last CTA to finish advances the call count (the parity and flag of
    // the next call); every CTA read it before adding itself here, and the
    // next call's CTAs read it only after this grid has completed.
    named_bar_sync(kGroupsPerCta + 1, kConsumerWarps * 32);
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

// ------------------------------------------------------------- launch ----

struct GemvPlan {
  int chunk_groups = 0, chunks = 0, stages = 0, row_pitch = 0, x_pitch = 0;
  bool window = false;
  size_t smem = 0;
};

// Largest chunk (preferably the whole row) and the most stages (>= 3, or
// >= 2 for the largest rows) that fit the shared memory.
template <int FMT>
static bool gemv_plan(const MatArgs& a, GemvPlan* out) {
  using F = GemvFmt<FMT>;
  if (a.M < 1 || a.M > 8) return false;
  const int64_t gpr = a.K / F::kGroupK;
  if (a.K % F::kGroupK != 0) return false;
  const bool aligned = reinterpret_cast<uintptr_t>(a.w) % 16 == 0 && a.w_stride % 16 == 0;
  if (!aligned || a.K % (static_cast<int64_t>(F::kGroupK) * F::kChunkAlign) != 0) {
    // window copies: whole rows only, each starting 4-byte aligned (the
    // decoders' alignment); the window holds up to 15 bytes around the row
    if (reinterpret_cast<uintptr_t>(a.w) % 4 != 0 || a.w_stride % 4 != 0) return false;
    const size_t avail = device_max_smem_optin();
    const int64_t x_pitch = a.K * 2 + 32;
    const size_t fixed = kBarrierBytes + kRedBytes + static_cast<size_t>(a.M) * x_pitch;
    const int64_t pitch = ((gpr * F::kGroupBytes + 15 + 15) / 16) * 16 + 16;
    const int64_t stage = kTileRows * pitch;
    if (fixed >= avail || static_cast<int64_t>(avail - fixed) / stage < 2) return false;
    out->chunk_groups = static_cast<int>(gpr);
    out->chunks = 1;
    out->stages = static_cast<int>(std::min<int64_t>(static_cast<int64_t>(avail - fixed) / stage, F::kMaxStages));
    out->row_pitch = static_cast<int>(pitch);
    out->x_pitch = static_cast<int>(x_pitch);
    out->smem = fixed + static_cast<size_t>(out->stages) * stage;
    out->window = true;
    return true;
  }
  const size_t avail = device_max_smem_optin();
  const int64_t x_pitch = a.K * 2 + 32;
  const size_t fixed = kBarrierBytes + kRedBytes + static_cast<size_t>(a.M) * x_pitch;
  if (fixed >= avail) return false;
  for (int min_stages : {3, 2}) {
    int64_t cg = gpr;
    while (cg >= F::kChunkAlign) {
      const int64_t pitch = ((cg * F::kGroupBytes + 15) / 16) * 16 + 16;  // +16: bank spread, over-read room
      const int64_t stage = kTileRows * pitch;
      const int64_t fit = static_cast<int64_t>(avail - fixed) / stage;
      if (fit >= min_stages) {
        out->chunk_groups = static_cast<int>(cg);
        out->chunks = static_cast<int>((gpr + cg - 1) / cg);
        out->stages = static_cast<int>(std::min<int64_t>(fit, F::kMaxStages));
        out->row_pitch = static_cast<int>(pitch);
        out->x_pitch = static_cast<int>(x_pitch);
        out->smem = fixed + static_cast<size_t>(out->stages) * stage;
        return true;
      }
      // halve the chunk, keeping it a multiple of the alignment
      cg = ((cg / 2) / F::kChunkAlign) * F::kChunkAlign;
    }
  }
  return false;
}

template <int FMT>
static bool gemv_fast_ok_t(const MatArgs& a) {
  GemvPlan plan;
  return gemv_plan<FMT>(a, &plan);
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
static cudaError_t gemv_t(const MatArgs& a, cudaStream_t stream, const PeerOut* po = nullptr) {
  using F = GemvFmt<FMT>;
  if constexpr (FMT == kQ6_K) {
    if (po == nullptr && gemv_xs6_ok(a)) return gemv_xs6(a, stream);
  }
  if (gemv_xs_ok(a)) return gemv_xs(a, po, stream);
  GemvPlan plan;
  if (!gemv_plan<FMT>(a, &plan) || (po != nullptr && plan.window)) {
    if (po != nullptr) return cudaErrorNotSupported;
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
  p.chunk_groups = plan.chunk_groups;
  p.chunks_per_row = plan.chunks;
  p.stages = plan.stages;
  p.row_pitch = plan.row_pitch;
  p.x_pitch = plan.x_pitch;
  p.y_bf16 = a.y_bf16;
  p.accumulate = a.accumulate;
  p.ftz = a.ftz;
  p.static_weights = a.static_weights;
  p.window = plan.window;
  if (po != nullptr) {
    p.xchg_peers = po->xchg_peers;
    p.n_offset = po->n_offset;
    p.n_total = po->n_total;
    p.rank = po->rank;
    p.world = po->world;
  }

  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = (FMT == kQ4_0 ? 0 : (FMT == kQ8_0 ? 1 : 2)) + (po != nullptr ? 3 : 0) + (a.ftz ? 6 : 0);
  static std::atomic<bool> configured[64][12];
  auto* kernel = po != nullptr ? (a.ftz ? gemv_kernel<FMT, true, true> : gemv_kernel<FMT, true, false>)
                               : (a.ftz ? gemv_kernel<FMT, false, true> : gemv_kernel<FMT, false, false>);
  if (!configured[dev & 63][slot].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(device_max_smem_optin()));
    if (e != cudaSuccess) return e;
    configured[dev & 63][slot].store(true, std::memory_order_release);
  }
  // One CTA per SM: the stages fill the shared memory by design.
  const int64_t tiles = (a.N + kTileRows - 1) / kTileRows;
  const int64_t grid = std::min<int64_t>(tiles, int64_t(device_sm_count()));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

cudaError_t gemv(const MatArgs& a, cudaStream_t stream) {
  switch (a.fmt) {
    case kQ4_0: return gemv_t<kQ4_0>(a, stream);
    case kQ8_0: return gemv_t<kQ8_0>(a, stream);
    case kQ6_K: return gemv_t<kQ6_K>(a, stream);
  }
  if (fmt_is_ext(a.fmt)) return gemv_ext(a, stream);
  return cudaErrorInvalidValue;
}

int64_t gemv_xchg_bytes(int64_t n_total) { return kXchgCtrlBytes + 2 * xchg_slot_bytes(n_total); }

cudaError_t gemv_allgather(const MatArgs& a, const PeerOut& po, cudaStream_t stream) {
  switch (a.fmt) {
    case kQ4_0: return gemv_t<kQ4_0>(a, stream, &po);
    case kQ8_0: return gemv_t<kQ8_0>(a, stream, &po);
    case kQ6_K: return gemv_t<kQ6_K>(a, stream, &po);
  }
  return cudaErrorInvalidValue;
}

}  // namespace spiral
