// dequant.cu — standalone GGUF dequant-to-bf16 kernels for sm_100a.
//
// B200 counterpart of the reference's per-format unpack_weights_chunk
// (src/quants/q4_0/unpack.aie.h:51-75, q8_0/unpack.aie.h:57-80,
// q6_k/unpack.aie.h:143-178) driven by quants_unpack_all
// (src/quants/tests/unpack.aie.cc:21-45).  The reference expands one 64- or
// 256-row chunk per call on one AIE core; here one warp expands a 16-byte
// aligned "unit" of canonical blocks per iteration:
//
//   Q4_0: 4 groups of 8 blocks (4 x 144 B, 1024 weights)
//   Q8_0: 4 groups of 8 blocks (4 x 272 B, 1024 weights)
//   Q6_K: 1 group of 8 super-blocks (1680 B, 2048 weights)
//
// The warp reads the unit with coalesced 128-bit loads into a private shared
// buffer, decodes from there with in-register bit tricks, and writes every
// 16-byte output chunk with one 128-bit store; lanes write consecutive chunks
// so each store instruction covers a contiguous 512-byte run.  Both sides are
// fully coalesced, so the kernel runs at the HBM write roofline (output bytes
// are 3.6x-4.6x the input bytes).
#include "api_internal.h"
#include "decode.cuh"

namespace spiral {

template <int FMT> struct DequantUnit;
template <> struct DequantUnit<kQ4_0> {
  static constexpr int kGroupBytes = 144, kGroupK = 256, kGroups = 4;
};
template <> struct DequantUnit<kQ8_0> {
  static constexpr int kGroupBytes = 272, kGroupK = 256, kGroups = 4;
};
template <> struct DequantUnit<kQ6_K> {
  static constexpr int kGroupBytes = 1680, kGroupK = 2048, kGroups = 1;
};

constexpr int kDequantWarps = 8;

// Offsets of a unit's groups: one 32-bit division per unit (the host
// guarantees total_groups < 2^32); the unit's later groups step along the row
// and wrap to the next rows.
template <int FMT>
__device__ __forceinline__ void dq_unit_offsets(int64_t unit, int64_t groups_per_row, int64_t total_groups,
                                                int64_t src_stride, int64_t dst_stride,
                                                int64_t (&src_off)[DequantUnit<FMT>::kGroups],
                                                int64_t (&dst_off)[DequantUnit<FMT>::kGroups],
                                                bool (&valid)[DequantUnit<FMT>::kGroups]) {
  using U = DequantUnit<FMT>;
  const int64_t g0 = unit * U::kGroups;
  const uint32_t gpr = static_cast<uint32_t>(groups_per_row);
  uint32_t row = static_cast<uint32_t>(g0) / gpr;
  uint32_t gi = static_cast<uint32_t>(g0) - row * gpr;
#pragma unroll
  for (int g = 0; g < U::kGroups; ++g) {
    valid[g] = g0 + g < total_groups;
    src_off[g] = static_cast<int64_t>(row) * src_stride + static_cast<int64_t>(gi) * U::kGroupBytes;
    dst_off[g] = static_cast<int64_t>(row) * dst_stride + static_cast<int64_t>(gi) * U::kGroupK;
    if (++gi == gpr) {
      gi = 0;
      ++row;
    }
  }
}

// Decode one unit staged in shared memory and store it: lanes write
// consecutive 16-byte chunks, so each store instruction covers a contiguous
// 512-byte run.
template <int FMT, bool FTZ>
__device__ __forceinline__ void dq_unit_store(const uint8_t* buf, int lane, uint16_t* __restrict__ dst,
                                              const int64_t (&dst_off)[DequantUnit<FMT>::kGroups],
                                              const bool (&valid)[DequantUnit<FMT>::kGroups]) {
  if constexpr (FMT == kQ4_0 || FMT == kQ8_0) {
    constexpr int kBB = Fmt<FMT>::kBlockBytes;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int oc = lane + 32 * i;  // output chunk of 8 weights, 0..127
      const int b = oc >> 2, part = oc & 3, g = b >> 3, blk = b & 7;
      if (!valid[g]) continue;
      const uint8_t* p = buf + kBB * b;
      const unsigned short h = fp16_scale_bits(lds_u16(p), FTZ);
      uint4 r;
      if constexpr (FMT == kQ4_0) {
        const uint8_t* qs = p + 2 + 8 * (part & 1);
        r = q4_0_decode8(lds_u32_a2(qs), lds_u32_a2(qs + 4), part >= 2, h);
      } else {
        const uint8_t* qs = p + 2 + 8 * part;
        r = q8_0_decode8(lds_u32_a2(qs), lds_u32_a2(qs + 4), h);
      }
      *reinterpret_cast<uint4*>(dst + dst_off[g] + 32 * blk + 8 * part) = r;
    }
  } else {
    // 64 tasks: super-block sb (0..7), half h, l0 in {0,8,16,24}; each task
    // emits the four 8-weight chunks y[128h + 32s + l0 .. +7], s = 0..3.
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int t = lane + 32 * i;
      const int sb = t >> 3, h = (t >> 2) & 1, l0 = 8 * (t & 3);
      const uint8_t* p = buf + 210 * sb;
      const float d = fp16_bits_to_f32(lds_u16(p + 208), FTZ);
      const uint32_t qla0 = lds_u32_a2(p + 64 * h + l0), qla1 = lds_u32_a2(p + 64 * h + l0 + 4);
      const uint32_t qlb0 = lds_u32_a2(p + 64 * h + 32 + l0), qlb1 = lds_u32_a2(p + 64 * h + 32 + l0 + 4);
      const uint32_t qh0 = lds_u32_a2(p + 128 + 32 * h + l0), qh1 = lds_u32_a2(p + 128 + 32 * h + l0 + 4);
      uint16_t* out = dst + dst_off[0] + 256 * sb + 128 * h + l0;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int8_t sc = static_cast<int8_t>(p[192 + 8 * h + 2 * s + (l0 >> 4)]);
        const float ds = d * static_cast<float>(sc);
        const uint2 a = q6_k_scale4(q6_k_assemble4((s & 1) ? qlb0 : qla0, qh0, s), ds);
        const uint2 b = q6_k_scale4(q6_k_assemble4((s & 1) ? qlb1 : qla1, qh1, s), ds);
        *reinterpret_cast<uint4*>(out + 32 * s) = make_uint4(a.x, a.y, b.x, b.y);
      }
    }
  }
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Row-major output, fast path.  Preconditions (checked on the host): src,
// dst 16-byte aligned; src_stride and dst_stride*2 multiples of 16; K a
// multiple of kGroupK.  A resident grid: every warp walks the units
// gw, gw + nw, ... and keeps kDqDepth of them in flight in a private ring of
// shared buffers (16-byte cp.async per lane), so the reads of the next units
// overlap the decode and the stores of this one.
constexpr int kDqDepth = 3;
template <int FMT, bool FTZ>
__global__ void __launch_bounds__(kDequantWarps * 32)
    dequant_rows_pipe(const uint8_t* __restrict__ src, int64_t src_stride, uint16_t* __restrict__ dst,
                      int64_t dst_stride, int64_t groups_per_row, int64_t total_groups, int64_t units) {
  using U = DequantUnit<FMT>;
  constexpr int kUnitBytes = U::kGroupBytes * U::kGroups;
  constexpr int kLoads = kUnitBytes / 16;
  constexpr int kPieces = U::kGroupBytes / 16;
  // +16: lds_u32_a2 may read one word past the last used byte.
  constexpr int kSlot = kUnitBytes + 16;
  __shared__ __align__(16) uint8_t sbuf[kDequantWarps][kDqDepth][kSlot];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kDequantWarps + warp;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * kDequantWarps;
  // programmatic dependent launch: the next kernel may be scheduled now; this
  // one touches global memory only after its predecessor has completed
  griddep_launch_dependents();
  griddep_wait();

  // one commit group per unit slot, empty past the last unit
  auto issue = [&](int64_t u, int slot) {
    if (u < units) {
      int64_t so[U::kGroups], dof[U::kGroups];
      bool v[U::kGroups];
      dq_unit_offsets<FMT>(u, groups_per_row, total_groups, src_stride, 0, so, dof, v);
      uint8_t* buf = sbuf[warp][slot];
#pragma unroll
      for (int q = lane; q < kLoads; q += 32) {
        const int g = q / kPieces, piece = q - g * kPieces;
        // select the group's offset without indexing the arrays by a
        // run-time value (which would put them in local memory)
        int64_t off = so[0];
        bool ok = v[0];
#pragma unroll
        for (int gg = 1; gg < U::kGroups; ++gg) {
          if (g == gg) {
            off = so[gg];
            ok = v[gg];
          }
        }
        if (ok) cp_async16(buf + 16 * q, src + off + 16 * piece);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int s = 0; s < kDqDepth; ++s) issue(gw + s * nw, s);

  int slot = 0;
  for (int64_t u = gw; u < units; u += nw) {
    cp_async_wait<kDqDepth - 1>();  // this lane's pieces of unit u have landed ...
    __syncwarp();                   // ... and every other lane's
    int64_t so[U::kGroups], dof[U::kGroups];
    bool v[U::kGroups];
    dq_unit_offsets<FMT>(u, groups_per_row, total_groups, 0, dst_stride, so, dof, v);
    dq_unit_store<FMT, FTZ>(sbuf[warp][slot], lane, dst, dof, v);
    __syncwarp();  // the slot is read by every lane before it is refilled
    issue(u + kDqDepth * nw, slot);
    slot = slot + 1 == kDqDepth ? 0 : slot + 1;
  }
  cp_async_wait<0>();
}

// Row-major output, fast path, one unit per warp (no ring): the better
// choice for Q6_K, whose units are large (2048 weights) and whose decode
// needs more registers than a resident ring of units allows.
template <int FMT, bool FTZ>
__global__ void __launch_bounds__(kDequantWarps * 32)
    dequant_rows_unit(const uint8_t* __restrict__ src, int64_t src_stride, uint16_t* __restrict__ dst,
                      int64_t dst_stride, int64_t groups_per_row, int64_t total_groups, int64_t units) {
  using U = DequantUnit<FMT>;
  constexpr int kUnitBytes = U::kGroupBytes * U::kGroups;
  constexpr int kLoads = kUnitBytes / 16;
  constexpr int kPieces = U::kGroupBytes / 16;
  __shared__ __align__(16) uint8_t sbuf[kDequantWarps][kUnitBytes + 16];
  griddep_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = static_cast<int64_t>(blockIdx.x) * kDequantWarps + warp;
  if (unit >= units) return;
  int64_t so[U::kGroups], dof[U::kGroups];
  bool v[U::kGroups];
  dq_unit_offsets<FMT>(unit, groups_per_row, total_groups, src_stride, dst_stride, so, dof, v);
  griddep_wait();
  uint8_t* buf = sbuf[warp];
#pragma unroll
  for (int q = lane; q < kLoads; q += 32) {
    const int g = q / kPieces, piece = q - g * kPieces;
    int64_t off = so[0];
    bool ok = v[0];
#pragma unroll
    for (int gg = 1; gg < U::kGroups; ++gg) {
      if (g == gg) {
        off = so[gg];
        ok = v[gg];
      }
    }
    if (ok) *reinterpret_cast<uint4*>(buf + 16 * q) = __ldg(reinterpret_cast<const uint4*>(src + off + 16 * piece));
  }
  __syncwarp();
  dq_unit_store<FMT, FTZ>(buf, lane, dst, dof, v);
}

// Row-major output, any valid shape/alignment: one thread per 8-weight
// chunk, 2-byte loads, 2-byte stores.
template <int FMT, bool FTZ>
__global__ void __launch_bounds__(256)
    dequant_rows_generic(const uint8_t* __restrict__ src, int64_t src_stride, uint16_t* __restrict__ dst,
                         int64_t dst_stride, int64_t K, int64_t N) {
  constexpr int kBK = Fmt<FMT>::kBlockK, kBB = Fmt<FMT>::kBlockBytes;
  const int64_t chunks_per_row = K / 8;
  const int64_t total = chunks_per_row * N;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = c / chunks_per_row, kc = c - n * chunks_per_row;
    const int64_t blk = (kc * 8) / kBK;
    const int k8 = static_cast<int>(kc - blk * (kBK / 8));
    const uint4 r = decode8_generic<FMT>(src + n * src_stride + blk * kBB, k8, FTZ);
    uint16_t* o = dst + n * dst_stride + kc * 8;
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      o[2 * j] = static_cast<uint16_t>(w[j] & 0xFFFFu);
      o[2 * j + 1] = static_cast<uint16_t>(w[j] >> 16);
    }
  }
}

// Reference stream order [N/8][K][8] (formats/<fmt>.py reference_weights).
// One thread per (column tile of 8 rows, 8-weight chunk along K): decodes the
// chunk for the 8 rows and writes 8 outputs of 16 B (one per k), each the 8
// rows' values at that k.
template <int FMT, bool FTZ>
__global__ void __launch_bounds__(256)
    dequant_tiles(const uint8_t* __restrict__ src, int64_t src_stride, uint16_t* __restrict__ dst, int64_t K,
                  int64_t N) {
  constexpr int kBK = Fmt<FMT>::kBlockK, kBB = Fmt<FMT>::kBlockBytes;
  const int64_t chunks_per_row = K / 8;
  const int64_t total = chunks_per_row * (N / 8);
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tile = c / chunks_per_row, kc = c - tile * chunks_per_row;
    const int64_t blk = (kc * 8) / kBK;
    const int k8 = static_cast<int>(kc - blk * (kBK / 8));
    uint32_t v[8][4];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const uint4 q = decode8_generic<FMT>(src + (tile * 8 + r) * src_stride + blk * kBB, k8, FTZ);
      v[r][0] = q.x;
      v[r][1] = q.y;
      v[r][2] = q.z;
      v[r][3] = q.w;
    }
    uint4* o = reinterpret_cast<uint4*>(dst + (tile * K + kc * 8) * 8);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int sh = (j & 1) * 16, wi = j >> 1;
      uint32_t e[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) e[r] = (v[r][wi] >> sh) & 0xFFFFu;
      o[j] = make_uint4(e[0] | (e[1] << 16), e[2] | (e[3] << 16), e[4] | (e[5] << 16), e[6] | (e[7] << 16));
    }
  }
}

// ------------------------------------------------------------ launchers --

template <int FMT, bool FTZ>
static cudaError_t launch_rows(const uint8_t* src, int64_t src_stride, uint16_t* dst, int64_t dst_stride, int64_t K,
                               int64_t N, bool fast, cudaStream_t stream) {
  using U = DequantUnit<FMT>;
  if (fast) {
    const int64_t gpr = K / U::kGroupK;
    const int64_t total_groups = gpr * N;
    const int64_t units = (total_groups + U::kGroups - 1) / U::kGroups;
    int64_t blocks = (units + kDequantWarps - 1) / kDequantWarps;
    auto* kernel = FMT == kQ6_K ? dequant_rows_unit<FMT, FTZ> : dequant_rows_pipe<FMT, FTZ>;
    if (FMT != kQ6_K) {
      static int per_sm[2] = {0, 0};  // resident CTAs per SM (same on every B200)
      const int slot = FMT == kQ4_0 ? 0 : 1;
      if (per_sm[slot] == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kDequantWarps * 32, 0) != cudaSuccess || n < 1)
          n = 1;
        per_sm[slot] = n;
      }
      blocks = std::min<int64_t>(blocks, int64_t(device_sm_count()) * per_sm[slot]);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(kDequantWarps * 32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, src, src_stride, dst, dst_stride, gpr, total_groups, units);
  } else {
    const int64_t total = (K / 8) * N;
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, int64_t(148) * 64);
    dequant_rows_generic<FMT, FTZ><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, src_stride, dst,
                                                                                       dst_stride, K, N);
  }
  return cudaGetLastError();
}

template <int FMT, bool FTZ>
static cudaError_t launch_tiles(const uint8_t* src, int64_t src_stride, uint16_t* dst, int64_t K, int64_t N,
                                cudaStream_t stream) {
  const int64_t total = (K / 8) * (N / 8);
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, int64_t(148) * 64);
  dequant_tiles<FMT, FTZ><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, src_stride, dst, K, N);
  return cudaGetLastError();
}

bool dequant_fast_ok(int fmt, const void* src, int64_t src_stride, const void* dst, int64_t dst_stride, int64_t K) {
  const int64_t gk = fmt == kQ6_K ? 2048 : 256;
  return (reinterpret_cast<uintptr_t>(src) % 16 == 0) && (reinterpret_cast<uintptr_t>(dst) % 16 == 0) &&
         (src_stride % 16 == 0) && ((dst_stride * 2) % 16 == 0) && (K % gk == 0);
}

static bool dequant_fast_fits(int fmt, int64_t K, int64_t N) {
  const int64_t gk = fmt == kQ6_K ? 2048 : 256;
  return (K / gk) * N < (int64_t(1) << 32) - 8;  // 32-bit group indices
}

cudaError_t dequant_rows(int fmt, const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int64_t K,
                         int64_t N, bool ftz, cudaStream_t stream) {
  const auto* s = static_cast<const uint8_t*>(src);
  auto* d = static_cast<uint16_t*>(dst);
  const bool fast = dequant_fast_ok(fmt, src, src_stride, dst, dst_stride, K) && dequant_fast_fits(fmt, K, N);
#define SPIRAL_DQ(F)                                                                   \
  return ftz ? launch_rows<F, true>(s, src_stride, d, dst_stride, K, N, fast, stream) \
             : launch_rows<F, false>(s, src_stride, d, dst_stride, K, N, fast, stream)
  switch (fmt) {
    case kQ4_0: SPIRAL_DQ(kQ4_0);
    case kQ8_0: SPIRAL_DQ(kQ8_0);
    case kQ6_K: SPIRAL_DQ(kQ6_K);
  }
#undef SPIRAL_DQ
  if (fmt_is_ext(fmt)) return dequant_rows_ext(fmt, src, src_stride, dst, dst_stride, K, N, ftz, stream);
  return cudaErrorInvalidValue;
}

cudaError_t dequant_tiles_ref(int fmt, const void* src, int64_t src_stride, void* dst, int64_t K, int64_t N, bool ftz,
                              cudaStream_t stream) {
  const auto* s = static_cast<const uint8_t*>(src);
  auto* d = static_cast<uint16_t*>(dst);
#define SPIRAL_DT(F) \
  return ftz ? launch_tiles<F, true>(s, src_stride, d, K, N, stream) : launch_tiles<F, false>(s, src_stride, d, K, N, stream)
  switch (fmt) {
    case kQ4_0: SPIRAL_DT(kQ4_0);
    case kQ8_0: SPIRAL_DT(kQ8_0);
    case kQ6_K: SPIRAL_DT(kQ6_K);
  }
#undef SPIRAL_DT
  return cudaErrorInvalidValue;
}

}  // namespace spiral
