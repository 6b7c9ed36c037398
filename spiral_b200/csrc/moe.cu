// moe.cu — MoE FFN decode layer with quantized experts:
// for every token t and each of its top-k routed experts e_{t,j} with weight
// w_{t,j}:
//   h_{t,j} = bf16( silu(x_t Wg_e^T) * (x_t Wu_e^T) )          [I]
//   y_t     = sum_j w_{t,j} * (h_{t,j} Wd_e^T)                  [H]
// with gate/up [I rows x H] and down [H rows x I] canonical GGUF tensors per
// expert, fp32 accumulation everywhere and one bf16 rounding of h (the down
// projection consumes bf16 activations) and of y.
//
// Only experts in the local range [e0, e0 + E_local) contribute; others are
// skipped, so expert-parallel ranks each compute their share and the caller
// combines across ranks.
//
// Four stream-ordered kernels, each launched with programmatic stream
// serialization (every kernel waits for its predecessor before it reads
// anything that predecessor wrote):
//   1. moe_route   one CTA: bucket the (token, slot) pairs of local experts by
//                  expert (a parallel counting sort) and cut each expert's
//                  pairs into problems of at most 8 (the MMA N width).
//   2. moe_gemv<1> gate+up: work item = (problem, 16 intermediate features);
//                  a stage holds the 16 gate rows and the 16 up rows; the
//                  epilogue applies SwiGLU and stores h in bf16.
//   3. moe_gemv<2> down: work item = (problem, 64 output features: four MMA
//                  row blocks, each split over two warps by K); the
//                  epilogue stores w_{t,j} * y_e in fp32 per pair.
//   4. moe_combine y_t = sum over slots j in order (deterministic).
// The grouped GEMVs reuse the decode GEMV's machinery (gemv_decode.cuh): one
// persistent CTA per SM, a producer warp streaming whole weight rows with 1-D
// bulk copies, two groups of 8 consumer warps on mma.sync.  Work items are
// cut into one contiguous range per CTA; each group restages its activation
// rows only when its next item belongs to a different problem.
//
// Scratch (counts, pair lists, problem table, h, per-pair outputs) lives in a
// caller-provided workspace (spiral_moe_workspace_bytes).
#include <atomic>
#include <mutex>

#include "api_internal.h"
#include "gemv_decode.cuh"

namespace spiral {

namespace {

constexpr int kMoeGroups = 2;
constexpr int kMoeWarpsPerGroup = 8;
constexpr int kMoeGroupThreads = kMoeWarpsPerGroup * 32;
constexpr int kMoeConsumers = kMoeGroups * kMoeWarpsPerGroup;
constexpr int kMoeThreads = (kMoeConsumers + 1) * 32;
constexpr int kMoeMaxStages = 24;  // down-projection stages are small (16 rows x 432 B)
constexpr int kMoeBarrierBytes = 512;  // 24 mbarrier pairs + the abort word
constexpr int kRouteThreads = 1024;
constexpr int kTileRows = 16;

struct MoeProblem {
  int expert;  // local expert index
  int first;   // offset into the sorted pair list
  int nx;      // pairs (activation rows), 1..8
  int pad;
};

struct MoeLayout {
  // all offsets in bytes from the workspace base, 256-byte aligned
  size_t hdr, cnt, start, cursor, pairs, problems, h, part, total;
  int64_t max_pairs, max_problems;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

MoeLayout moe_layout(int64_t E_local, int64_t H, int64_t I, int64_t T, int64_t topk) {
  MoeLayout L{};
  L.max_pairs = T * topk;
  L.max_problems = L.max_pairs / 8 + E_local + 1;
  size_t off = 0;
  L.hdr = off;
  off = align256(off + 4 * sizeof(int));
  L.cnt = off;
  off = align256(off + E_local * sizeof(int));
  L.start = off;
  off = align256(off + E_local * sizeof(int));
  L.cursor = off;
  off = align256(off + E_local * sizeof(int));
  L.pairs = off;
  off = align256(off + L.max_pairs * sizeof(int));
  L.problems = off;
  off = align256(off + L.max_problems * sizeof(MoeProblem));
  L.h = off;
  off = align256(off + L.max_pairs * I * 2);
  L.part = off;
  off = align256(off + L.max_pairs * H * sizeof(float));
  L.total = off;
  return L;
}

struct MoeArgs {
  int fmt;
  const uint8_t* w_gate;  // [E_local][I][row_bytes(H)]
  const uint8_t* w_up;
  const uint8_t* w_down;  // [E_local][H][row_bytes(I)]
  int64_t rb_h, rb_i;     // row bytes of a gate/up row (K = H) and a down row (K = I)
  const uint16_t* x;      // [T][x_stride] bf16
  int64_t x_stride;
  const int32_t* ids;     // [T][topk] global expert ids
  const float* wts;       // [T][topk]
  void* y;                // [T][y_stride]
  int64_t y_stride;
  int y_bf16, accumulate, ftz;
  int T, topk, H, I, e0, E_local;
  uint8_t* ws;
  MoeLayout L;
  // Few pairs (T * topk <= kMoeDirectPairs): no routing kernel; pair p is
  // problem p (expert ids[p], one row), the pair list the identity.
  int direct;
};

constexpr int kMoeDirectPairs = 16;

// Problem pidx, pair-list entry idx and the problem count, routed or direct
// (a template parameter of the kernels, so the routed kernels carry no
// direct-mode code).
template <bool DIRECT>
__device__ __forceinline__ MoeProblem moe_problem(const MoeArgs& a, const MoeProblem* probs, int pidx) {
  if constexpr (DIRECT) {
    const int e = a.ids[pidx] - a.e0;
    const bool local = e >= 0 && e < a.E_local;
    return MoeProblem{local ? e : 0, pidx, local ? 1 : 0, 0};
  } else {
    return probs[pidx];
  }
}
template <bool DIRECT>
__device__ __forceinline__ int moe_pair(const int* pairs, int idx) {
  if constexpr (DIRECT) {
    return idx;
  } else {
    return pairs[idx];
  }
}
template <bool DIRECT>
__device__ __forceinline__ int moe_problem_count(const MoeArgs& a, const int* hdr) {
  if constexpr (DIRECT) {
    return a.T * a.topk;
  } else {
    return hdr[0];
  }
}

// ------------------------------------------------------------- routing ----

// Exclusive prefix sum of v over the block (kRouteThreads threads, one value
// each); returns this thread's prefix and sets `total`.
__device__ __forceinline__ int route_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < kRouteThreads / 32 ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive
  }
  __syncthreads();
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  total = warp_sums[kRouteThreads / 32 - 1];
  __syncthreads();  // warp_sums is reused by the next scan
  return before;
}

// Counting sort of the local (token, slot) pairs by expert, every step in
// parallel: counts by shared atomics, one block scan for each expert's first
// pair and one for its first problem, then each expert writes its own
// problems.  E_local is processed in chunks of kRouteThreads experts.
__global__ void __launch_bounds__(kRouteThreads) moe_route(const MoeArgs a) {
  extern __shared__ int sh[];
  int* scnt = sh;
  int* sstart = sh + a.E_local;
  int* scur = sh + 2 * a.E_local;
  __shared__ int warp_sums[32];
  griddep_launch_dependents();
  griddep_wait();
  int* hdr = reinterpret_cast<int*>(a.ws + a.L.hdr);
  int* pairs = reinterpret_cast<int*>(a.ws + a.L.pairs);
  MoeProblem* probs = reinterpret_cast<MoeProblem*>(a.ws + a.L.problems);
  const int np_total = a.T * a.topk;
  for (int e = threadIdx.x; e < a.E_local; e += blockDim.x) {
    scnt[e] = 0;
    scur[e] = 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < np_total; i += blockDim.x) {
    const int e = a.ids[i] - a.e0;
    if (e >= 0 && e < a.E_local) atomicAdd(&scnt[e], 1);
  }
  __syncthreads();
  int run = 0, np = 0;  // pairs and problems before this chunk
  for (int e0 = 0; e0 < a.E_local; e0 += kRouteThreads) {
    const int e = e0 + static_cast<int>(threadIdx.x);
    const int cnt = e < a.E_local ? scnt[e] : 0;
    int pairs_chunk = 0, probs_chunk = 0;
    const int pbefore = route_scan(cnt, warp_sums, pairs_chunk);
    const int qbefore = route_scan((cnt + 7) / 8, warp_sums, probs_chunk);
    if (e < a.E_local) {
      sstart[e] = run + pbefore;
      for (int c = 0, q = np + qbefore; c < cnt; c += 8, ++q) {
        MoeProblem pr;
        pr.expert = e;
        pr.first = run + pbefore + c;
        pr.nx = min(8, cnt - c);
        pr.pad = 0;
        probs[q] = pr;
      }
    }
    run += pairs_chunk;
    np += probs_chunk;
  }
  if (threadIdx.x == 0) {
    hdr[0] = np;
    hdr[1] = run;
  }
  __syncthreads();
  // Order inside an expert's list does not change any result: each pair is
  // its own MMA column, computed with the same summation order.
  for (int i = threadIdx.x; i < np_total; i += blockDim.x) {
    const int e = a.ids[i] - a.e0;
    if (e >= 0 && e < a.E_local) pairs[sstart[e] + atomicAdd(&scur[e], 1)] = i;
  }
}

// ------------------------------------------------------- grouped GEMV -----

template <int PHASE>
struct MoePhase;
template <>
struct MoePhase<1> {  // gate + up, K = H, 16 intermediate features per item
  static constexpr int kRows = 32;
};
template <>
struct MoePhase<2> {  // down, K = I, up to 64 output features per item
  static constexpr int kRows = 64;
};
// Output features per work item: 16 for gate/up (the stage holds those 16
// gate rows and 16 up rows); for down 64, 32 or 16 (the most that leaves
// three stages in shared memory): 1, 2 or 4 MMA row blocks, each split by K
// over 8, 4 or 2 warps, so every consumer warp decodes several groups.

// Stage the activation rows of one problem for one consumer group in the
// permuted fragment order of gemv_decode.cuh: row m (< nx) comes from
// src(m).  Four rows at a time, each thread first loads its 16-byte pieces of
// those rows (one L2 round trip), then each row goes through `raw` and is
// permuted.
template <int FMT, typename Src>
__device__ void moe_stage_rows(int nx, int K, Src src, uint8_t* xs, int x_pitch, uint8_t* raw, int gt, int bar_id) {
  using F = GemvFmt<FMT>;
  constexpr int kStepShift = F::kSteps == 8 ? 3 : 4;
  constexpr int kMaxPieces = 2;  // K <= 2 * 8 * 256 = 4096
  constexpr int kRowsPerRound = 4;
  const int pieces = K / 8;
  const int per_m = (K / F::kGroupK) * F::kSteps * 4;
  for (int m0 = 0; m0 < nx; m0 += kRowsPerRound) {
    uint4 v[kRowsPerRound][kMaxPieces];
#pragma unroll
    for (int mm = 0; mm < kRowsPerRound; ++mm) {
#pragma unroll
      for (int i = 0; i < kMaxPieces; ++i) {
        const int q = gt + i * kMoeGroupThreads;
        if (m0 + mm < nx && q < pieces) v[mm][i] = __ldg(reinterpret_cast<const uint4*>(src(m0 + mm)) + q);
      }
    }
#pragma unroll
    for (int mm = 0; mm < kRowsPerRound; ++mm) {
      const int m = m0 + mm;
      if (m < nx) {
#pragma unroll
        for (int i = 0; i < kMaxPieces; ++i) {
          const int q = gt + i * kMoeGroupThreads;
          if (q < pieces) reinterpret_cast<uint4*>(raw)[q] = v[mm][i];
        }
        named_bar_sync(bar_id, kMoeGroupThreads);
        const uint16_t* xr = reinterpret_cast<const uint16_t*>(raw);
        uint8_t* dst = xs + m * x_pitch;
        for (int e = gt; e < per_m; e += kMoeGroupThreads) {
          const int c = e & 3, gs = e >> 2, st = gs & (F::kSteps - 1), g = gs >> kStepShift;
          const int k = g * F::kGroupK + GroupDecoder<FMT>::xk(st, c);
          *reinterpret_cast<uint2*>(dst + gs * 32 + c * 8) =
              make_uint2(xr[k] | (static_cast<uint32_t>(xr[k + 1]) << 16),
                         xr[k + 2] | (static_cast<uint32_t>(xr[k + 3]) << 16));
        }
        named_bar_sync(bar_id, kMoeGroupThreads);
      }
    }
  }
}

template <int FMT>
__device__ __forceinline__ void moe_decode_group(const uint8_t* ra, const uint8_t* rb, int c, const uint8_t* xg,
                                                 bool ftz, float (&acc)[4], int gl) {
  if constexpr (FMT == kQ6_K) {
    GroupDecoder<FMT>::run(ra, rb, c, xg, ftz, acc, (gl & 1) ? 16u : 0u);
  } else {
    GroupDecoder<FMT>::run(ra, rb, c, xg, ftz, acc);
  }
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

template <int FMT, int PHASE>
__global__ void __launch_bounds__(kMoeThreads, 1)
    moe_gemv(const MoeArgs a, int stages, int row_pitch, int x_pitch, int item_rows) {
  using F = GemvFmt<FMT>;
  using P = MoePhase<PHASE>;
  constexpr int kAcc = PHASE == 1 ? 2 : 1;
  const int K = PHASE == 1 ? a.H : a.I;
  const int N = PHASE == 1 ? a.I : a.H;
  const int64_t rb = PHASE == 1 ? a.rb_h : a.rb_i;
  const int kItemRows = PHASE == 1 ? kTileRows : item_rows;
  const int stage_rows = PHASE == 1 ? P::kRows : item_rows;
  const int tiles = N / kItemRows;
  const int groups_per_row = K / F::kGroupK;

  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMoeMaxStages;
  int& abort_flag = *reinterpret_cast<int*>(smem + kMoeBarrierBytes - 8);
  float4* red = reinterpret_cast<float4*>(smem + kMoeBarrierBytes);  // [groups][kAcc][8 warps][32]
  uint8_t* xbuf = smem + kMoeBarrierBytes + kMoeConsumers * 32 * 16 * kAcc;  // [groups][8][x_pitch]
  uint8_t* stg = xbuf + kMoeGroups * 8 * x_pitch;
  const int stage_bytes = stage_rows * row_pitch;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kMoeWarpsPerGroup);
    }
    abort_flag = 0;
    fence_mbar_init();
    griddep_launch_dependents();
  }
  __syncthreads();
  griddep_wait();  // the route kernel (and for phase 2 the gate/up kernel) wrote what follows

  const int* hdr = reinterpret_cast<const int*>(a.ws + a.L.hdr);
  const int* pairs = reinterpret_cast<const int*>(a.ws + a.L.pairs);
  const MoeProblem* probs = reinterpret_cast<const MoeProblem*>(a.ws + a.L.problems);
  const int64_t items = static_cast<int64_t>(moe_problem_count<false>(a, hdr)) * tiles;
  const int64_t i_begin = blockIdx.x * items / gridDim.x, i_end = (blockIdx.x + 1) * items / gridDim.x;

  if (warp == kMoeConsumers) {
    // ------------------------------------------------------- producer ----
    // Lane 0 waits for a free stage and posts the byte count; then lane l
    // (< kRows) issues the copy of stage row l, so an item's 16 or 32 row
    // copies leave in one instruction (items are small: one thread issuing
    // them one by one would pace the down projection).
    const uint64_t pol = l2_evict_first_policy();
    const uint32_t bytes = static_cast<uint32_t>(rb);
    uint32_t it = 0;
    for (int64_t i = i_begin; i < i_end; ++i, ++it) {
      const MoeProblem pr = moe_problem<false>(a, probs, static_cast<int>(i / tiles));
      const int tile = static_cast<int>(i % tiles);
      const int s = static_cast<int>(it % stages);
      int go = 0;
      if (lane == 0) {
        go = mbar_wait(&empty[s], ((it / stages) & 1u) ^ 1u) && !*(volatile int*)&abort_flag;
        if (go) {
          mbar_arrive_expect_tx(&full[s], bytes * stage_rows);
        } else {
          abort_flag = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      const int64_t row0 = static_cast<int64_t>(pr.expert) * N + tile * kItemRows;
      for (int l = lane; l < stage_rows; l += 32) {
        uint8_t* dst = stg + s * stage_bytes + l * row_pitch;
        const uint8_t* src;
        if constexpr (PHASE == 1) {
          src = l < kTileRows ? a.w_gate + (row0 + l) * rb : a.w_up + (row0 + l - kTileRows) * rb;
        } else {
          src = a.w_down + (row0 + l) * rb;
        }
        bulk_g2s(dst, src, bytes, &full[s], pol);
      }
    }
    // Every issued stage must land before the CTA may exit.
    if (lane == 0) {
      const uint32_t first = it > static_cast<uint32_t>(stages) ? it - stages : 0u;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % stages], (j / stages) & 1u);
    }
    return;
  }

  // --------------------------------------------------------- consumers -----
  const int grp = warp / kMoeWarpsPerGroup, gw = warp % kMoeWarpsPerGroup;
  const int gt = gw * 32 + lane;
  const int r = lane >> 2, c = lane & 3;
  const bool ftz = a.ftz != 0;
  float4* gred = red + grp * (kAcc * kMoeWarpsPerGroup * 32);
  uint8_t* xs = xbuf + grp * 8 * x_pitch;
  const int bar_id = 1 + grp;
  int staged = -1;  // problem whose rows are in xs
  // The epilogue thread's activation column is the same in every item:
  // its pair (and routing weight) is read once per problem, not per item.
  const int my_m = 2 * ((gt >> 2) & 3) + (gt & 1);
  MoeProblem pr{};
  int my_pair = 0;
  float my_wt = 0.f;
  uint32_t it = 0;
  for (int64_t i = i_begin; i < i_end; ++i, ++it) {
    if (static_cast<int>((i - i_begin) % kMoeGroups) != grp) continue;
    const int pidx = static_cast<int>(i / tiles);
    const int tile = static_cast<int>(i % tiles);
    if (pidx != staged) {
      pr = moe_problem<false>(a, probs, pidx);
      my_pair = my_m < pr.nx ? moe_pair<false>(pairs, pr.first + my_m) : 0;
      if constexpr (PHASE == 2) my_wt = my_m < pr.nx ? a.wts[my_pair] : 0.f;
      if constexpr (PHASE == 1) {
        auto src = [&](int m) { return a.x + static_cast<int64_t>(moe_pair<false>(pairs, pr.first + m) / a.topk) * a.x_stride; };
        moe_stage_rows<FMT>(pr.nx, K, src, xs, x_pitch, reinterpret_cast<uint8_t*>(gred), gt, bar_id);
      } else {
        const uint16_t* h = reinterpret_cast<const uint16_t*>(a.ws + a.L.h);
        auto src = [&](int m) { return h + static_cast<int64_t>(moe_pair<false>(pairs, pr.first + m)) * a.I; };
        moe_stage_rows<FMT>(pr.nx, K, src, xs, x_pitch, reinterpret_cast<uint8_t*>(gred), gt, bar_id);
      }
      staged = pidx;
    }
    const int mx = r < pr.nx ? r : 0;  // columns >= nx read row 0 and are discarded
    const uint8_t* xcol = xs + mx * x_pitch + c * 8;
    const int s = static_cast<int>(it % stages);
    float acc[kAcc][4] = {};
    bool ready = false;
    if (!*(volatile int*)&abort_flag) {
      ready = mbar_wait(&full[s], (it / stages) & 1u);
      if (!ready) abort_flag = 1;
    }
    if (ready) {
      const uint8_t* st = stg + s * stage_bytes;
      if constexpr (PHASE == 1) {
        for (int gl = gw; gl < groups_per_row; gl += kMoeWarpsPerGroup) {
          const uint8_t* xg = xcol + gl * (F::kSteps * 32);
#pragma unroll
          for (int ac = 0; ac < kAcc; ++ac) {
            const uint8_t* base = st + ac * kTileRows * row_pitch + gl * F::kGroupBytes;
            moe_decode_group<FMT>(base + r * row_pitch, base + (r + 8) * row_pitch, c, xg, ftz, acc[ac], gl);
          }
        }
      } else {
        // warp gw: row block gw / wpr of the item, the (gw % wpr)-th part of K
        const int wpr = kMoeWarpsPerGroup / (item_rows / kTileRows);
        const int per = (groups_per_row + wpr - 1) / wpr;
        const int g_lo = (gw % wpr) * per, g_hi = min(groups_per_row, g_lo + per);
        const uint8_t* base = st + (gw / wpr) * kTileRows * row_pitch;
        for (int gl = g_lo; gl < g_hi; ++gl) {
          const uint8_t* xg = xcol + gl * (F::kSteps * 32);
          const uint8_t* gb = base + gl * F::kGroupBytes;
          moe_decode_group<FMT>(gb + r * row_pitch, gb + (r + 8) * row_pitch, c, xg, ftz, acc[0], gl);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
    for (int ac = 0; ac < kAcc; ++ac)
      gred[(ac * kMoeWarpsPerGroup + gw) * 32 + lane] = make_float4(acc[ac][0], acc[ac][1], acc[ac][2], acc[ac][3]);
    named_bar_sync(bar_id, kMoeGroupThreads);
    if constexpr (PHASE == 2) {
      // row blocks x 128 outputs: the K parts summed in order
      const int wpr = kMoeWarpsPerGroup / (item_rows / kTileRows);
      for (int idx = gt; idx < (item_rows / kTileRows) * 128; idx += kMoeGroupThreads) {
        const int rbk = idx >> 7, l = (idx >> 2) & 31, j = idx & 3;
        float v = 0.f;
        for (int q = 0; q < wpr; ++q) v += reinterpret_cast<const float*>(&gred[(rbk * wpr + q) * 32 + l])[j];
        const int row = rbk * kTileRows + (l >> 2) + 8 * (j >> 1);
        const int m = 2 * (l & 3) + (j & 1);
        if (ready && m < pr.nx) {  // m == my_m
          float* part = reinterpret_cast<float*>(a.ws + a.L.part);
          part[static_cast<int64_t>(my_pair) * a.H + tile * kItemRows + row] = my_wt * v;
        }
      }
    } else if (gw < 4) {
      const int l = gt >> 2, j = gt & 3;
      float v[kAcc];
#pragma unroll
      for (int ac = 0; ac < kAcc; ++ac) {
        v[ac] = 0.f;
#pragma unroll
        for (int w = 0; w < kMoeWarpsPerGroup; ++w)
          v[ac] += reinterpret_cast<const float*>(&gred[(ac * kMoeWarpsPerGroup + w) * 32 + l])[j];
      }
      const int row = (l >> 2) + 8 * (j >> 1);
      const int m = 2 * (l & 3) + (j & 1);
      if (ready && m < pr.nx) {  // m == my_m
        const int feat = tile * kTileRows + row;
        if constexpr (PHASE == 1) {
          uint16_t* h = reinterpret_cast<uint16_t*>(a.ws + a.L.h);
          h[static_cast<int64_t>(my_pair) * a.I + feat] =
              static_cast<uint16_t>(pack_bf16x2(silu(v[0]) * v[kAcc - 1], 0.f) & 0xFFFFu);
        } else {
          float* part = reinterpret_cast<float*>(a.ws + a.L.part);
          part[static_cast<int64_t>(my_pair) * a.H + feat] = my_wt * v[0];
        }
      }
    }
    named_bar_sync(bar_id, kMoeGroupThreads);  // gred is free again
  }
}

// Sum over token t's slots j whose expert is local, in slot order, of
// part[t*topk + j][n] (0 + the first such value, then the next, ...).  A
// chunk of 8 slots issues all its id and partial loads before the adds, so a
// thread waits about two memory latencies per chunk instead of two per slot.
__device__ __forceinline__ float moe_local_slot_sum(const MoeArgs& a, const float* part, int64_t t, int64_t n) {
  const int* ids = a.ids + t * a.topk;
  const float* pt = part + t * a.topk * static_cast<int64_t>(a.H) + n;
  float sum = 0.f;
  for (int j0 = 0; j0 < a.topk; j0 += 8) {
    float v[8];
    bool use[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u;
      const int ex = j < a.topk ? ids[j] - a.e0 : -1;
      use[u] = ex >= 0 && ex < a.E_local;
      v[u] = use[u] ? pt[static_cast<int64_t>(j) * a.H] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (use[u]) sum += v[u];
  }
  return sum;
}

// y[t][n] = sum over local slots j (in order) of part[t*topk + j][n].
__global__ void moe_combine(const MoeArgs a) {
  griddep_launch_dependents();
  griddep_wait();
  const float* part = reinterpret_cast<const float*>(a.ws + a.L.part);
  const int64_t total = static_cast<int64_t>(a.T) * a.H;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(e / a.H), n = static_cast<int>(e % a.H);
    const float sum = moe_local_slot_sum(a, part, t, n);
    const int64_t off = static_cast<int64_t>(t) * a.y_stride + n;
    if (a.y_bf16) {
      static_cast<uint16_t*>(a.y)[off] = static_cast<uint16_t>(pack_bf16x2(sum, 0.f) & 0xFFFFu);
    } else if (a.accumulate) {
      static_cast<float*>(a.y)[off] += sum;
    } else {
      static_cast<float*>(a.y)[off] = sum;
    }
  }
}

// ------------------------------------------------- expert-parallel combine --
//
// Expert-parallel layer (spiral_moe_ffn_ep): every rank holds all T tokens
// (x, ids and weights replicated, as after the preceding dense layer's
// all-gather) and the experts [e0, e0 + E_local); its partial y_r[t][h] is
// the sum over the token's slots whose expert is local.  The ranks' partials
// are combined inside this kernel over NVLink peer stores, in two exchanges
// that together are a reduce-scatter and an all-gather:
//  1. every rank sends its partial of column h to the column's owner
//     (owner = h / (H / world)) as 8-byte units {fp32 value, flag};
//  2. the owner sums the `world` partials of each of its columns in rank
//     order 0..world-1 (deterministic), writes the value to its own y and
//     sends it to every other rank as units {fp32, flag};
//  3. every rank copies the other ranks' columns into its y.
// A unit's flag is the call count | 2^31, stored with the value as one
// 64-bit access, so a reader that sees the flag sees the value; two slots
// alternate by call parity and the last CTA advances the call count, as in
// the gathered dense GEMV.  Waits are bounded (kWaitLimitNs); a rank that
// never arrives makes them give up with kDevErrPeerTimeout.  Step 1 has no
// waits and every CTA finishes it before it waits, and the grid (at most one
// CTA per SM, nothing else running) is co-resident, so the waits cannot
// cycle.
//
// Exchange buffer of a rank (moe_ep_xchg_bytes): a 256-byte control block
// (word 0: calls completed, word 1: CTA count of the running call) and two
// slots of [world][max_tokens][H / world] partial units followed by
// [max_tokens][H] result units.
struct MoeEp {
  uint8_t* const* peers;
  int rank, world;
  int64_t max_tokens;
};
constexpr int64_t kMoeEpCtrlBytes = 256;
__host__ __device__ constexpr int64_t moe_ep_slot_bytes(int64_t max_tokens, int64_t H) { return 16 * max_tokens * H; }

__device__ __forceinline__ void st_unit_sys(uint8_t* dst, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(dst), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_unit_sys(const uint8_t* src) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(src) : "memory");
  return v;
}
// Bounded poll for a unit carrying `flag`; false (and the device error) on
// giving up.
__device__ __forceinline__ bool wait_unit(const uint8_t* src, uint32_t flag, uint64_t& v) {
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    v = ld_unit_sys(src);
    if (static_cast<uint32_t>(v >> 32) == flag) return true;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_device_error(kDevErrPeerTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ void moe_store_y(const MoeArgs& a, int64_t t, int64_t h, float v) {
  const int64_t off = t * a.y_stride + h;
  if (a.y_bf16) {
    static_cast<uint16_t*>(a.y)[off] = static_cast<uint16_t>(pack_bf16x2(v, 0.f) & 0xFFFFu);
  } else if (a.accumulate) {
    static_cast<float*>(a.y)[off] += v;
  } else {
    static_cast<float*>(a.y)[off] = v;
  }
}

__global__ void __launch_bounds__(512) moe_ep_combine(const MoeArgs a, const MoeEp ep) {
  // every CTA is running before a dependent grid may start (co-residency)
  griddep_launch_dependents();
  griddep_wait();
  const float* part = reinterpret_cast<const float*>(a.ws + a.L.part);
  const int64_t T = a.T, H = a.H, Hs = H / ep.world;
  uint8_t* own = ep.peers[ep.rank];
  const uint32_t calls = *reinterpret_cast<volatile const uint32_t*>(own);
  const uint32_t flag = calls | 0x80000000u;
  const uint64_t hi = static_cast<uint64_t>(flag) << 32;
  const int64_t slot_off = kMoeEpCtrlBytes + (calls & 1) * moe_ep_slot_bytes(ep.max_tokens, H);
  const int64_t part_region = static_cast<int64_t>(ep.world) * ep.max_tokens * Hs * 8;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  // a rank that failed to arrive earlier leaves the call counts disagreeing:
  // skip the waits until the host has read the error
  bool ok = !(*(volatile uint32_t*)&g_device_error & kDevErrPeerTimeout);
  // 1. this rank's partials, to each column's owner
  for (int64_t e = tid; e < T * H; e += stride) {
    const int64_t t = e / H, h = e - t * H;
    const float sum = moe_local_slot_sum(a, part, t, h);
    const int q = static_cast<int>(h / Hs);
    st_unit_sys(ep.peers[q] + slot_off + ((static_cast<int64_t>(ep.rank) * ep.max_tokens + t) * Hs + (h - q * Hs)) * 8,
                hi | __float_as_uint(sum));
  }
  // 2. this rank's columns: every rank's partial, summed in rank order
  for (int64_t e = tid; ok && e < T * Hs; e += stride) {
    const int64_t t = e / Hs, hl = e - t * Hs;
    float sum = 0.f;
    for (int r = 0; r < ep.world && ok; ++r) {
      uint64_t v;
      ok = wait_unit(own + slot_off + ((static_cast<int64_t>(r) * ep.max_tokens + t) * Hs + hl) * 8, flag, v);
      sum += __uint_as_float(static_cast<uint32_t>(v));
    }
    if (!ok) break;
    const int64_t h = static_cast<int64_t>(ep.rank) * Hs + hl;
    moe_store_y(a, t, h, sum);
    for (int r = 0; r < ep.world; ++r)
      if (r != ep.rank) st_unit_sys(ep.peers[r] + slot_off + part_region + (t * H + h) * 8, hi | __float_as_uint(sum));
  }
  // 3. the other ranks' columns
  for (int64_t e = tid; ok && e < T * H; e += stride) {
    const int64_t t = e / H, h = e - t * H;
    if (h / Hs == ep.rank) continue;
    uint64_t v;
    ok = wait_unit(own + slot_off + part_region + (t * H + h) * 8, flag, v);
    if (ok) moe_store_y(a, t, h, __uint_as_float(static_cast<uint32_t>(v)));
  }
  // the last CTA to finish advances the call count (every CTA read it above;
  // the next call's CTAs read it only after this grid has completed)
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* ctrl = reinterpret_cast<uint32_t*>(own);
    uint32_t before;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(before) : "l"(ctrl + 1) : "memory");
    if (before == gridDim.x - 1) {
      ctrl[1] = 0u;
      ctrl[0] = calls + 1u;
    }
  }
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

template <int FMT, int PHASE>
cudaError_t launch_moe_gemv(const MoeArgs& a, cudaStream_t stream) {
  using F = GemvFmt<FMT>;
  constexpr int kAcc = PHASE == 1 ? 2 : 1;
  const int K = PHASE == 1 ? a.H : a.I;
  const int64_t rb = PHASE == 1 ? a.rb_h : a.rb_i;
  const int x_pitch = K * 2 + 32;
  const int row_pitch = static_cast<int>(rb) + 16;
  const size_t fixed = kMoeBarrierBytes + size_t(kMoeConsumers) * 32 * 16 * kAcc + size_t(kMoeGroups) * 8 * x_pitch;
  const size_t avail = device_max_smem_optin();
  // gate/up: 32 stage rows (16 gate + 16 up); down: the largest item of
  // 64 / 32 / 16 rows that leaves three stages (the output dimension H is a
  // multiple of 64)
  int rows = MoePhase<PHASE>::kRows;
  if constexpr (PHASE == 2) {
    while (rows > kTileRows && fixed + size_t(3) * rows * row_pitch > avail) rows /= 2;
  }
  if (fixed + size_t(2) * rows * row_pitch > avail) return cudaErrorInvalidValue;
  const int stages = static_cast<int>(std::min<size_t>(kMoeMaxStages, (avail - fixed) / (size_t(rows) * row_pitch)));
  const size_t smem = fixed + size_t(stages) * rows * row_pitch;
  (void)F::kGroupK;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<bool> configured[64];
  if (!configured[dev & 63].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(moe_gemv<FMT, PHASE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(avail));
    if (e != cudaSuccess) return e;
    configured[dev & 63].store(true, std::memory_order_release);
  }
  MoeArgs args = a;
  int st = stages, rp = row_pitch, xp = x_pitch, ir = rows;
  void* kargs[] = {&args, &st, &rp, &xp, &ir};
  return launch_pdl(reinterpret_cast<const void*>(moe_gemv<FMT, PHASE>), dim3(device_sm_count()), dim3(kMoeThreads),
                    smem, stream, kargs);
}

// ------------------------------------------- gate/up, activation-stationary --
//
// The gate/up GEMV of the layer with the decode GEMV's structure (gemv_xs.cu)
// for Q4_0 / Q8_0 at hidden = 16 x 128 x GPW: one CTA per SM, 16 consumer
// warps and a producer warp.  A work item is (problem, 16 intermediate
// features); its stage holds the 16 gate and the 16 up rows as 8 + 8 pairs of
// consecutive rows (pitch 2 rows + 16 bytes; MMA row g <-> row 2g, g + 8 <->
// 2g + 1).  Warp w owns the K slice [w K/16, (w+1) K/16) of every item; its
// activation fragments for the current problem's tokens stay in registers
// (reloaded from a shared staging buffer when the CTA's items move to the
// next problem) and serve gate and up alike.  The 16 warps' partial gate and
// up tiles go to 4 reducer warps (rotating per item) through a
// double-buffered shared array handed over with mbarriers; the reducers sum
// them in warp order, apply SwiGLU and store h in bf16.
constexpr int kGuWarps = 16;
constexpr int kGuWarpProducer = kGuWarps, kGuWarpReducer = kGuWarps + 1;
constexpr int kGuThreads = (kGuWarps + 2) * 32;  // + the producer and the reducer warp
constexpr int kGuMaxStages = 8;
constexpr int kGuHeader = 1024;
constexpr int kGuRedBytes = 2 * kGuWarps * 32 * 32;  // 2 buffers x 16 warps x 32 lanes x (gate, up) float4

template <int FMT, int GPW, bool DIRECT>
// 18 warps spread 5 + 5 + 4 + 4 over the sub-partitions: 96 registers per
// thread is the most that launches.
__global__ void __maxnreg__(96) moe_gateup_xs(const MoeArgs a, int stages, int pair_pitch) {
  using F = GemvFmt<FMT>;
  constexpr int kSteps = F::kSteps;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kGuMaxStages;
  uint64_t* red_full = empty + kGuMaxStages;
  uint64_t* red_empty = red_full + 2;
  int& abort_flag = *reinterpret_cast<int*>(smem + 512);
  float4* red = reinterpret_cast<float4*>(smem + kGuHeader);  // [2][16 warps][32 lanes][gate, up]
  uint8_t* xbuf = smem + kGuHeader + kGuRedBytes;              // [8 rows][H] bf16
  const int x_bytes = 8 * a.H * 2;
  uint8_t* stg = xbuf + x_bytes;
  const int stage_bytes = 16 * pair_pitch;
  const int rb = static_cast<int>(a.rb_h);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = a.I / kTileRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kGuWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&red_full[b], kGuWarps * 32);
      mbar_init(&red_empty[b], 32);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  griddep_wait();  // the route kernel wrote what follows
  // The down kernel may start once every CTA is past this point: the problem
  // list (or the ids) is then complete, so its producer can stream the down
  // weights while this kernel still runs.
  if (threadIdx.x == 0) griddep_launch_dependents();

  const int* hdr = reinterpret_cast<const int*>(a.ws + a.L.hdr);
  const int* pairs = reinterpret_cast<const int*>(a.ws + a.L.pairs);
  const MoeProblem* probs = reinterpret_cast<const MoeProblem*>(a.ws + a.L.problems);
  const int64_t items = static_cast<int64_t>(moe_problem_count<DIRECT>(a, hdr)) * tiles;
  const int64_t i_begin = blockIdx.x * items / gridDim.x, i_end = (blockIdx.x + 1) * items / gridDim.x;

  if (warp == kGuWarpProducer) {
    // ---------------------------------------------------------- producer --
    const uint64_t pol = l2_evict_first_policy();
    uint32_t it = 0;
    int stage = 0;
    uint32_t phase = 0u;
    for (int64_t i = i_begin; i < i_end; ++i, ++it) {
      const MoeProblem pr = moe_problem<DIRECT>(a, probs, static_cast<int>(i / tiles));
      const int tile = static_cast<int>(i % tiles);
      int go = 0;
      if (lane == 0) {
        go = !*(volatile int*)&abort_flag && mbar_wait(&empty[stage], phase ^ 1u);
        if (go) {
          mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(rb) * 2 * kTileRows);
        } else {
          abort_flag = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      if (lane < 16) {
        // lane q < 8: gate rows 2q, 2q + 1 of the tile; lane 8 + q: up rows
        const int q = lane & 7;
        const int64_t row = static_cast<int64_t>(pr.expert) * a.I + tile * kTileRows + 2 * q;
        const uint8_t* src = (lane < 8 ? a.w_gate : a.w_up) + row * rb;
        bulk_g2s(stg + stage * stage_bytes + lane * pair_pitch, src, static_cast<uint32_t>(rb) * 2, &full[stage],
                 pol);
      }
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    // Every issued copy must land before the CTA may exit.
    if (lane == 0) {
      const uint32_t first = it > static_cast<uint32_t>(stages) ? it - stages : 0u;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % stages], (j / stages) & 1u);
    }
    return;
  }

  if (warp == kGuWarpReducer) {
    // ---------------------------------------------------------- reducer --
    // Lane l sums the 16 warps' (gate, up) float4 partials of fragment lane
    // l in warp order: item rows (MMA rows l / 4, + 8) x problem vectors
    // 2 (l % 4), + 1; h = silu(gate) * up in bf16.
    uint16_t* h = reinterpret_cast<uint16_t*>(a.ws + a.L.h);
    const int m0 = 2 * (lane & 3);
    int staged = -1, nx = 0, pair0 = 0, pair1 = 0;
    int local = 0;
    for (int64_t i = i_begin; i < i_end; ++i, ++local) {
      const int pidx = static_cast<int>(i / tiles);
      const int tile = static_cast<int>(i % tiles);
      if (pidx != staged) {
        const MoeProblem pr = moe_problem<DIRECT>(a, probs, pidx);
        nx = pr.nx;
        pair0 = m0 < nx ? moe_pair<DIRECT>(pairs, pr.first + m0) : 0;
        pair1 = m0 + 1 < nx ? moe_pair<DIRECT>(pairs, pr.first + m0 + 1) : 0;
        staged = pidx;
      }
      const int rbuf = local & 1;
      if (!mbar_try_wait(&red_full[rbuf], static_cast<uint32_t>(local >> 1) & 1u) && !*(volatile int*)&abort_flag) {
        if (!mbar_wait(&red_full[rbuf], static_cast<uint32_t>(local >> 1) & 1u)) abort_flag = 1;
      }
      const float4* rp = red + (rbuf * kGuWarps * 32 + lane) * 2;
      float4 g = make_float4(0.f, 0.f, 0.f, 0.f), u = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kGuWarps; ++w) {
        const float4 gv = rp[w * 64], uv = rp[w * 64 + 1];
        g.x += gv.x;
        g.y += gv.y;
        g.z += gv.z;
        g.w += gv.w;
        u.x += uv.x;
        u.y += uv.y;
        u.z += uv.z;
        u.w += uv.w;
      }
      mbar_arrive(&red_empty[rbuf]);
      if (*(volatile int*)&abort_flag) continue;
      const float gs[4] = {g.x, g.y, g.z, g.w}, us[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int m = m0 + (j & 1);
        if (m >= nx) continue;
        const int rowp = (lane >> 2) + 8 * (j >> 1);                 // MMA row
        const int row = rowp < 8 ? 2 * rowp : 2 * (rowp - 8) + 1;  // weight row of the tile
        h[static_cast<int64_t>((j & 1) ? pair1 : pair0) * a.I + tile * kTileRows + row] =
            static_cast<uint16_t>(pack_bf16x2(silu(gs[j]) * us[j], 0.f) & 0xFFFFu);
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers --
  const int r = lane >> 2, c = lane & 3;
  const bool ftz = a.ftz != 0;
  const uint8_t* ra0 = stg + r * pair_pitch + warp * GPW * F::kGroupBytes;
  uint2 Bx[GPW][kSteps];
  int staged = -1;
  MoeProblem pr{};
  int stage = 0;
  uint32_t phase = 0u;
  int local = 0;
  for (int64_t i = i_begin; i < i_end; ++i, ++local) {
    const int pidx = static_cast<int>(i / tiles);
    if (pidx != staged) {
      // every warp has its fragments of the previous problem
      named_bar_sync(1, kGuWarps * 32);
      pr = moe_problem<DIRECT>(a, probs, pidx);
      // the problem's activation rows (nx <= 8), 16-byte pieces
      const int pieces = a.H / 8;
      for (int q = threadIdx.x; q < pr.nx * pieces; q += kGuWarps * 32) {
        const int m = q / pieces, pc = q - m * pieces;
        const int tok = moe_pair<DIRECT>(pairs, pr.first + m) / a.topk;
        reinterpret_cast<uint4*>(xbuf + m * a.H * 2)[pc] =
            __ldg(reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(tok) * a.x_stride) + pc);
      }
      named_bar_sync(1, kGuWarps * 32);
#pragma unroll
      for (int g = 0; g < GPW; ++g) {
#pragma unroll
        for (int st = 0; st < kSteps; ++st) {
          const int k = (warp * GPW + g) * F::kGroupK + GroupDecoder<FMT>::xk(st, c);
          Bx[g][st] = r < pr.nx ? *reinterpret_cast<const uint2*>(xbuf + r * a.H * 2 + k * 2) : make_uint2(0u, 0u);
        }
      }
      staged = pidx;
    }
    float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
    const int s = stage;
    bool ready = mbar_try_wait(&full[s], phase);
    if (!ready && !*(volatile int*)&abort_flag) {
      ready = mbar_wait(&full[s], phase);
      if (!ready) abort_flag = 1;
    }
    if (ready) {
      const uint8_t* ra = ra0 + s * stage_bytes;
#pragma unroll
      for (int g = 0; g < GPW; ++g) {
        auto bx = [&](int st) { return Bx[g][st]; };
        const uint8_t* ga = ra + g * F::kGroupBytes;
        GroupDecoder<FMT>::run_b(ga, ga + rb, c, bx, ftz, accg);
        const uint8_t* ua = ga + 8 * pair_pitch;
        GroupDecoder<FMT>::run_b(ua, ua + rb, c, bx, ftz, accu);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++stage == stages) {
      stage = 0;
      phase ^= 1u;
    }

    // hand the partials to the reducer warp
    const int rbuf = local & 1;
    if (local >= 2 && !mbar_try_wait(&red_empty[rbuf], static_cast<uint32_t>((local >> 1) - 1) & 1u) &&
        !*(volatile int*)&abort_flag) {
      if (!mbar_wait(&red_empty[rbuf], static_cast<uint32_t>((local >> 1) - 1) & 1u)) abort_flag = 1;
    }
    float4* my = red + ((rbuf * kGuWarps + warp) * 32 + lane) * 2;
    my[0] = make_float4(accg[0], accg[1], accg[2], accg[3]);
    my[1] = make_float4(accu[0], accu[1], accu[2], accu[3]);
    mbar_arrive(&red_full[rbuf]);
  }
}

// GPW (decode groups per warp) of the activation-stationary gate/up, or 0
// when the layer's shape is not served (then the grouped kernel runs).
int moe_gu_gpw(const MoeArgs& a) {
  if (a.fmt != kQ4_0 && a.fmt != kQ8_0) return 0;
  if (a.H == 2048) return 1;
  if (a.H == 4096) return 2;
  return 0;
}

// Whether the activation-stationary gate/up kernel serves this layer.
bool moe_gateup_xs_ok(const MoeArgs& a) {
  if (moe_gu_gpw(a) == 0) return false;
  // dense rows, 16-byte aligned, for the pair copies
  if (reinterpret_cast<uintptr_t>(a.w_gate) % 16 || reinterpret_cast<uintptr_t>(a.w_up) % 16 || a.rb_h % 16)
    return false;
  const size_t fixed = kGuHeader + kGuRedBytes + size_t(8) * a.H * 2;
  const size_t stage = size_t(16) * (2 * static_cast<size_t>(a.rb_h) + 16);
  return fixed + 3 * stage <= device_max_smem_optin();
}

template <int FMT>
cudaError_t launch_moe_gateup_xs(const MoeArgs& a, cudaStream_t stream, bool* launched) {
  *launched = false;
  if (!moe_gateup_xs_ok(a)) return cudaSuccess;
  const int gpw = moe_gu_gpw(a);
  const int pair_pitch = 2 * static_cast<int>(a.rb_h) + 16;
  const size_t fixed = kGuHeader + kGuRedBytes + size_t(8) * a.H * 2;
  const size_t avail = device_max_smem_optin();
  const size_t stage = size_t(16) * pair_pitch;
  const int stages = static_cast<int>(std::min<size_t>(kGuMaxStages, (avail - fixed) / stage));
  const size_t smem = fixed + size_t(stages) * stage;
  auto* kernel = a.direct ? (gpw == 1 ? moe_gateup_xs<FMT, 1, true> : moe_gateup_xs<FMT, 2, true>)
                          : (gpw == 1 ? moe_gateup_xs<FMT, 1, false> : moe_gateup_xs<FMT, 2, false>);
  const int slot = (gpw - 1) * 2 + (a.direct ? 1 : 0);
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<bool> configured[64][4];
  if (!configured[dev & 63][slot].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(avail));
    if (e != cudaSuccess) return e;
    configured[dev & 63][slot].store(true, std::memory_order_release);
  }
  MoeArgs args = a;
  int st = stages, pp = pair_pitch;
  void* kargs[] = {&args, &st, &pp};
  *launched = true;
  return launch_pdl(reinterpret_cast<const void*>(kernel), dim3(device_sm_count()), dim3(kGuThreads), smem, stream,
                    kargs);
}

// ---------------------------------------------- down, activation-stationary --
//
// The down GEMV (K = inter) with the same structure for Q4_0 / Q8_0 at
// inter = 6 x 128 (768): a work item is (problem, 64 output rows) copied as
// 32 pairs of consecutive rows.  12 consumer warps: warp w owns decode group
// g = w % 6 of K and the row blocks 2 (w / 6) and 2 (w / 6) + 1 of the item,
// so its activation fragments (the problem's h rows, one group) stay in
// registers and every warp issues 16 MMAs per item.  4 reducer warps
// (rotating over 3 sets) sum each output's 6 group partials in order and
// store w_{t,j} * y into the per-pair outputs.
constexpr int kDnGroups = 6;
constexpr int kDnWarps = 12;
constexpr int kDnWarpProducer = kDnWarps, kDnWarpReducer = kDnWarps + 1;
constexpr int kDnThreads = (kDnWarps + 2) * 32;  // + the producer and the reducer warp
constexpr int kDnMaxStages = 12;
constexpr int kDnItemRows = 64;
constexpr int kDnHeader = 1024;
constexpr int kDnRedBytes = 2 * kDnWarps * 32 * 32;  // 2 buffers x 12 warps x 32 lanes x 2 float4

template <int FMT, bool DIRECT>
// 14 warps spread 4 + 4 + 3 + 3 over the sub-partitions: 120 registers per
// thread still launches.
__global__ void __maxnreg__(120) moe_down_xs(const MoeArgs a, int stages, int pair_pitch) {
  using F = GemvFmt<FMT>;
  constexpr int kSteps = F::kSteps;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kDnMaxStages;
  uint64_t* red_full = empty + kDnMaxStages;
  uint64_t* red_empty = red_full + 2;
  int& abort_flag = *reinterpret_cast<int*>(smem + 512);
  float4* red = reinterpret_cast<float4*>(smem + kDnHeader);  // [2][12 warps][32 lanes][2 row blocks]
  uint8_t* xbuf = smem + kDnHeader + kDnRedBytes;             // [8 rows][I] bf16
  uint8_t* stg = xbuf + 8 * a.I * 2;
  const int stage_bytes = (kDnItemRows / 2) * pair_pitch;
  const int rb = static_cast<int>(a.rb_i);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = a.H / kDnItemRows;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDnWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&red_full[b], kDnWarps * 32);
      mbar_init(&red_empty[b], 32);
    }
    abort_flag = 0;
    fence_mbar_init();
    griddep_launch_dependents();
  }
  __syncthreads();
  // The problem list and the weights are final when this kernel starts (the
  // gate/up kernel releases it only after its own wait on the routing): the
  // producer streams weights at once; the consumers and the reducer wait for
  // the gate/up kernel to complete before reading h or writing outputs.
  if (warp != kDnWarpProducer) griddep_wait();

  const int* hdr = reinterpret_cast<const int*>(a.ws + a.L.hdr);
  const int* pairs = reinterpret_cast<const int*>(a.ws + a.L.pairs);
  const MoeProblem* probs = reinterpret_cast<const MoeProblem*>(a.ws + a.L.problems);
  const uint16_t* hbuf = reinterpret_cast<const uint16_t*>(a.ws + a.L.h);
  const int64_t items = static_cast<int64_t>(moe_problem_count<DIRECT>(a, hdr)) * tiles;
  const int64_t i_begin = blockIdx.x * items / gridDim.x, i_end = (blockIdx.x + 1) * items / gridDim.x;

  if (warp == kDnWarpProducer) {
    // ---------------------------------------------------------- producer --
    const uint64_t pol = l2_evict_first_policy();
    uint32_t it = 0;
    int stage = 0;
    uint32_t phase = 0u;
    for (int64_t i = i_begin; i < i_end; ++i, ++it) {
      const MoeProblem pr = moe_problem<DIRECT>(a, probs, static_cast<int>(i / tiles));
      const int tile = static_cast<int>(i % tiles);
      int go = 0;
      if (lane == 0) {
        go = !*(volatile int*)&abort_flag && mbar_wait(&empty[stage], phase ^ 1u);
        if (go) {
          mbar_arrive_expect_tx(&full[stage], static_cast<uint32_t>(rb) * kDnItemRows);
        } else {
          abort_flag = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      // lane q: rows 2q, 2q + 1 of the item
      const int64_t row = static_cast<int64_t>(pr.expert) * a.H + tile * kDnItemRows + 2 * lane;
      bulk_g2s(stg + stage * stage_bytes + lane * pair_pitch, a.w_down + row * rb, static_cast<uint32_t>(rb) * 2,
               &full[stage], pol);
      if (++stage == stages) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (lane == 0) {
      const uint32_t first = it > static_cast<uint32_t>(stages) ? it - stages : 0u;
      for (uint32_t j = first; j < it; ++j) mbar_wait(&full[j % stages], (j / stages) & 1u);
    }
    return;
  }

  if (warp == kDnWarpReducer) {
    // ---------------------------------------------------------- reducer --
    // Lane l sums, for each of the item's 4 row blocks b, the 6 group
    // partials (warps 6 (b / 2) + g, accumulator b % 2) of fragment lane l in
    // group order, and stores w_{t,j} * y into the per-pair outputs: rows of
    // MMA rows l / 4, + 8 of block b, problem vectors 2 (l % 4), + 1.
    float* part = reinterpret_cast<float*>(a.ws + a.L.part);
    const int m0 = 2 * (lane & 3);
    int staged = -1, nx = 0, pair0 = 0, pair1 = 0;
    float wt0 = 0.f, wt1 = 0.f;
    int local = 0;
    for (int64_t i = i_begin; i < i_end; ++i, ++local) {
      const int pidx = static_cast<int>(i / tiles);
      const int tile = static_cast<int>(i % tiles);
      if (pidx != staged) {
        const MoeProblem pr = moe_problem<DIRECT>(a, probs, pidx);
        nx = pr.nx;
        pair0 = m0 < nx ? moe_pair<DIRECT>(pairs, pr.first + m0) : 0;
        pair1 = m0 + 1 < nx ? moe_pair<DIRECT>(pairs, pr.first + m0 + 1) : 0;
        wt0 = m0 < nx ? a.wts[pair0] : 0.f;
        wt1 = m0 + 1 < nx ? a.wts[pair1] : 0.f;
        staged = pidx;
      }
      const int rbuf = local & 1;
      if (!mbar_try_wait(&red_full[rbuf], static_cast<uint32_t>(local >> 1) & 1u) && !*(volatile int*)&abort_flag) {
        if (!mbar_wait(&red_full[rbuf], static_cast<uint32_t>(local >> 1) & 1u)) abort_flag = 1;
      }
      float4 v[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const float4* rp = red + ((rbuf * kDnWarps + (b >> 1) * kDnGroups) * 32 + lane) * 2 + (b & 1);
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int gg = 0; gg < kDnGroups; ++gg) {
          const float4 q = rp[gg * 64];
          sum.x += q.x;
          sum.y += q.y;
          sum.z += q.z;
          sum.w += q.w;
        }
        v[b] = sum;
      }
      mbar_arrive(&red_empty[rbuf]);
      if (*(volatile int*)&abort_flag) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int m = m0 + (j & 1);
        if (m >= nx) continue;
        const int rowp = (lane >> 2) + 8 * (j >> 1);
        const int row16 = rowp < 8 ? 2 * rowp : 2 * (rowp - 8) + 1;
        const float wt = (j & 1) ? wt1 : wt0;
        float* dst = part + static_cast<int64_t>((j & 1) ? pair1 : pair0) * a.H + tile * kDnItemRows + row16;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const float val = j == 0 ? v[b].x : j == 1 ? v[b].y : j == 2 ? v[b].z : v[b].w;
          dst[16 * b] = wt * val;
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers --
  const int r = lane >> 2, c = lane & 3;
  const bool ftz = a.ftz != 0;
  const int g = warp % kDnGroups, rbp = warp / kDnGroups;  // decode group, row-block pair
  // MMA row r of row block b = pair 8b + r (weight rows 16b + 2r, +1)
  const uint8_t* ra0 = stg + (16 * rbp + r) * pair_pitch + g * F::kGroupBytes;
  uint2 Bx[kSteps];
  int staged = -1;
  MoeProblem pr{};
  int stage = 0;
  uint32_t phase = 0u;
  int local = 0;
  for (int64_t i = i_begin; i < i_end; ++i, ++local) {
    const int pidx = static_cast<int>(i / tiles);
    if (pidx != staged) {
      named_bar_sync(1, kDnWarps * 32);
      pr = moe_problem<DIRECT>(a, probs, pidx);
      const int pieces = a.I / 8;
      for (int q = threadIdx.x; q < pr.nx * pieces; q += kDnWarps * 32) {
        const int m = q / pieces, pc = q - m * pieces;
        reinterpret_cast<uint4*>(xbuf + m * a.I * 2)[pc] =
            __ldg(reinterpret_cast<const uint4*>(hbuf + static_cast<int64_t>(moe_pair<DIRECT>(pairs, pr.first + m)) * a.I) + pc);
      }
      named_bar_sync(1, kDnWarps * 32);
#pragma unroll
      for (int st = 0; st < kSteps; ++st) {
        const int k = g * F::kGroupK + GroupDecoder<FMT>::xk(st, c);
        Bx[st] = r < pr.nx ? *reinterpret_cast<const uint2*>(xbuf + r * a.I * 2 + k * 2) : make_uint2(0u, 0u);
      }
      staged = pidx;
    }
    float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
    const int s = stage;
    bool ready = mbar_try_wait(&full[s], phase);
    if (!ready && !*(volatile int*)&abort_flag) {
      ready = mbar_wait(&full[s], phase);
      if (!ready) abort_flag = 1;
    }
    if (ready) {
      auto bx = [&](int st) { return Bx[st]; };
      const uint8_t* b0 = ra0 + s * stage_bytes;
      GroupDecoder<FMT>::run_b(b0, b0 + rb, c, bx, ftz, acc0);
      const uint8_t* b1 = b0 + 8 * pair_pitch;
      GroupDecoder<FMT>::run_b(b1, b1 + rb, c, bx, ftz, acc1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++stage == stages) {
      stage = 0;
      phase ^= 1u;
    }

    // hand the partials to the reducer warp
    const int rbuf = local & 1;
    if (local >= 2 && !mbar_try_wait(&red_empty[rbuf], static_cast<uint32_t>((local >> 1) - 1) & 1u) &&
        !*(volatile int*)&abort_flag) {
      if (!mbar_wait(&red_empty[rbuf], static_cast<uint32_t>((local >> 1) - 1) & 1u)) abort_flag = 1;
    }
    float4* my = red + ((rbuf * kDnWarps + warp) * 32 + lane) * 2;
    my[0] = make_float4(acc0[0], acc0[1], acc0[2], acc0[3]);
    my[1] = make_float4(acc1[0], acc1[1], acc1[2], acc1[3]);
    mbar_arrive(&red_full[rbuf]);
  }
}

// Whether the activation-stationary down kernel serves this layer.
template <int FMT>
bool moe_down_xs_ok(const MoeArgs& a) {
  if (a.fmt != kQ4_0 && a.fmt != kQ8_0) return false;
  if (a.I != kDnGroups * GemvFmt<FMT>::kGroupK || a.H % kDnItemRows != 0) return false;
  if (reinterpret_cast<uintptr_t>(a.w_down) % 16 || a.rb_i % 16) return false;
  const size_t fixed = kDnHeader + kDnRedBytes + size_t(8) * a.I * 2;
  const size_t stage = size_t(kDnItemRows / 2) * (2 * static_cast<size_t>(a.rb_i) + 16);
  return fixed + 3 * stage <= device_max_smem_optin();
}

template <int FMT>
cudaError_t launch_moe_down_xs(const MoeArgs& a, cudaStream_t stream, bool* launched) {
  *launched = false;
  if (!moe_down_xs_ok<FMT>(a)) return cudaSuccess;
  const int pair_pitch = 2 * static_cast<int>(a.rb_i) + 16;
  const size_t fixed = kDnHeader + kDnRedBytes + size_t(8) * a.I * 2;
  const size_t avail = device_max_smem_optin();
  const size_t stage = size_t(kDnItemRows / 2) * pair_pitch;
  const int stages = static_cast<int>(std::min<size_t>(kDnMaxStages, (avail - fixed) / stage));
  const size_t smem = fixed + size_t(stages) * stage;
  auto* kernel = a.direct ? moe_down_xs<FMT, true> : moe_down_xs<FMT, false>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::atomic<bool> configured[64][2];
  if (!configured[dev & 63][a.direct ? 1 : 0].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(avail));
    if (e != cudaSuccess) return e;
    configured[dev & 63][a.direct ? 1 : 0].store(true, std::memory_order_release);
  }
  MoeArgs args = a;
  int st = stages, pp = pair_pitch;
  void* kargs[] = {&args, &st, &pp};
  *launched = true;
  return launch_pdl(reinterpret_cast<const void*>(kernel), dim3(device_sm_count()), dim3(kDnThreads), smem, stream,
                    kargs);
}

template <int FMT>
cudaError_t moe_run(const MoeArgs& a0, cudaStream_t stream, const MoeEp* ep = nullptr) {
  MoeArgs args = a0;
  // A few pairs: each is its own problem and the routing kernel (a launch
  // and a dependent step in front of the weight stream) is skipped; it
  // costs a second read of an expert's weights only when two of the pairs
  // pick the same expert.
  // Both expert kernels must be the activation-stationary ones (the grouped
  // fallback reads the routed problem list).
  if constexpr (FMT == kQ4_0 || FMT == kQ8_0)
    args.direct = ep == nullptr && static_cast<int64_t>(a0.T) * a0.topk <= kMoeDirectPairs &&
                  moe_gateup_xs_ok(a0) && moe_down_xs_ok<FMT>(a0);
  const MoeArgs& a = args;
  if (!a.direct) {
    void* kargs[] = {&args};
    const size_t smem = size_t(3) * a.E_local * sizeof(int);
    cudaError_t e = launch_pdl(reinterpret_cast<const void*>(moe_route), dim3(1), dim3(kRouteThreads), smem, stream,
                               kargs);
    if (e != cudaSuccess) return e;
  }
  bool gu_done = false;
  cudaError_t e = cudaSuccess;
  if constexpr (FMT == kQ4_0 || FMT == kQ8_0) e = launch_moe_gateup_xs<FMT>(a, stream, &gu_done);
  if (e != cudaSuccess) return e;
  if (!gu_done) e = launch_moe_gemv<FMT, 1>(a, stream);
  if (e != cudaSuccess) return e;
  bool dn_done = false;
  if constexpr (FMT == kQ4_0 || FMT == kQ8_0) e = launch_moe_down_xs<FMT>(a, stream, &dn_done);
  if (e != cudaSuccess) return e;
  if (!dn_done) e = launch_moe_gemv<FMT, 2>(a, stream);
  if (e != cudaSuccess) return e;
  const int64_t total = static_cast<int64_t>(a.T) * a.H;
  if (ep != nullptr) {
    // persistent and co-resident: at most one CTA per SM
    MoeEp epa = *ep;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 511) / 512, int64_t(device_sm_count())));
    void* kargs[] = {&args, &epa};
    return launch_pdl(reinterpret_cast<const void*>(moe_ep_combine), dim3(blocks), dim3(512), 0, stream, kargs);
  }
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, int64_t(device_sm_count()) * 8));
  void* kargs[] = {&args};
  return launch_pdl(reinterpret_cast<const void*>(moe_combine), dim3(blocks), dim3(256), 0, stream, kargs);
}

}  // namespace

size_t moe_workspace_bytes(int64_t E_local, int64_t H, int64_t I, int64_t T, int64_t topk) {
  return moe_layout(E_local, H, I, T, topk).total;
}

bool moe_shape_ok(int fmt, int64_t H, int64_t I) {
  // weight rows a whole number of 16-byte runs (bulk copies) and of decode
  // groups; an activation row fits the group's staging buffer (H <= 4096,
  // I <= 2048)
  const int64_t unit = fmt == kQ6_K ? 2048 : 256;
  if (H % unit != 0 || I % unit != 0) return false;
  return H <= 4096 && I <= 2048;
}

namespace {

MoeArgs moe_args(int fmt, const void* w_gate, const void* w_up, const void* w_down, const void* x, int64_t x_stride,
                 const int32_t* ids, const float* wts, void* y, int64_t y_stride, bool y_bf16, bool accumulate,
                 bool ftz, int64_t T, int64_t topk, int64_t H, int64_t I, int64_t e0, int64_t E_local, void* ws) {
  MoeArgs a{};
  a.fmt = fmt;
  a.w_gate = static_cast<const uint8_t*>(w_gate);
  a.w_up = static_cast<const uint8_t*>(w_up);
  a.w_down = static_cast<const uint8_t*>(w_down);
  const int64_t bk = fmt == kQ6_K ? 256 : 32, bb = fmt == kQ4_0 ? 18 : (fmt == kQ8_0 ? 34 : 210);
  a.rb_h = H / bk * bb;
  a.rb_i = I / bk * bb;
  a.x = static_cast<const uint16_t*>(x);
  a.x_stride = x_stride;
  a.ids = ids;
  a.wts = wts;
  a.y = y;
  a.y_stride = y_stride;
  a.y_bf16 = y_bf16;
  a.accumulate = accumulate;
  a.ftz = ftz;
  a.T = static_cast<int>(T);
  a.topk = static_cast<int>(topk);
  a.H = static_cast<int>(H);
  a.I = static_cast<int>(I);
  a.e0 = static_cast<int>(e0);
  a.E_local = static_cast<int>(E_local);
  a.ws = static_cast<uint8_t*>(ws);
  a.L = moe_layout(E_local, H, I, T, topk);
  return a;
}

cudaError_t moe_dispatch(const MoeArgs& a, cudaStream_t stream, const MoeEp* ep) {
  switch (a.fmt) {
    case kQ4_0: return moe_run<kQ4_0>(a, stream, ep);
    case kQ8_0: return moe_run<kQ8_0>(a, stream, ep);
    case kQ6_K: return moe_run<kQ6_K>(a, stream, ep);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t moe_ffn(int fmt, const void* w_gate, const void* w_up, const void* w_down, const void* x,
                    int64_t x_stride, const int32_t* ids, const float* wts, void* y, int64_t y_stride, bool y_bf16,
                    bool accumulate, bool ftz, int64_t T, int64_t topk, int64_t H, int64_t I, int64_t e0,
                    int64_t E_local, void* ws, cudaStream_t stream) {
  return moe_dispatch(moe_args(fmt, w_gate, w_up, w_down, x, x_stride, ids, wts, y, y_stride, y_bf16, accumulate,
                               ftz, T, topk, H, I, e0, E_local, ws),
                      stream, nullptr);
}

int64_t moe_ep_xchg_bytes(int64_t H, int64_t max_tokens) {
  return kMoeEpCtrlBytes + 2 * moe_ep_slot_bytes(max_tokens, H);
}

cudaError_t moe_ffn_ep(int fmt, const void* w_gate, const void* w_up, const void* w_down, const void* x,
                       int64_t x_stride, const int32_t* ids, const float* wts, void* y, int64_t y_stride, bool y_bf16,
                       bool accumulate, bool ftz, int64_t T, int64_t topk, int64_t H, int64_t I, int64_t e0,
                       int64_t E_local, void* ws, uint8_t* const* peers, int rank, int world, int64_t max_tokens,
                       cudaStream_t stream) {
  const MoeEp ep{peers, rank, world, max_tokens};
  return moe_dispatch(moe_args(fmt, w_gate, w_up, w_down, x, x_stride, ids, wts, y, y_stride, y_bf16, accumulate,
                               ftz, T, topk, H, I, e0, E_local, ws),
                      stream, &ep);
}

// ------------------------------------------------ allocation-free variant ----
//
// spiral_moe_ffn_noalloc serves callers that cannot allocate device memory
// at the point where they call in: a host without a device allocator of its
// own (a plain C program handed device pointers), a serving loop that must
// not hit cudaMalloc mid-step (it may synchronize the device), or code whose
// device memory is owned by a caching allocator or a pre-planned arena that
// a stray allocation would disturb.  Its scratch is this file-scope array,
// reserved on every GPU that loads the library until the process exits.
// Every call shares it and it keeps the last call's contents: the MoE layer
// reads only scratch bytes it wrote earlier in the same call, so nothing has
// to start at zero; calls that overlap on the GPU (different streams, or
// host threads without ordering between them) race on it.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per GPU
static __device__ __align__(256) uint8_t g_moe_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};
}  // namespace

size_t moe_noalloc_scratch_bytes() { return kNoAllocScratchBytes; }

// Device address of the array on the current device.  The first call on a
// device looks it up (cudaGetSymbolAddress, with that device current); in
// host code the array's name is only a stand-in for the symbol, never a
// device address.
cudaError_t moe_noalloc_scratch(void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_moe_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_addr[dev] = p;
  }
  *ptr = g_noalloc_addr[dev];
  return cudaSuccess;
}

}  // namespace spiral
