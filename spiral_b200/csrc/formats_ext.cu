// formats_ext.cu — dequant-to-bf16 and MUL_MAT for the extended GGUF
// formats (Q4_K, Q5_K, IQ4_NL, IQ4_XS, F16, BF16), the reference's "more
// formats" next step (src/quants/TODO.md:16-22, 80-130).
//
// Both paths are built on the exact 8-weight decoders of decode_ext.cuh:
//  * dequant: one thread per 8-weight chunk of a row, grid-stride, one
//    16-byte store per chunk when the destination allows it (2-byte stores
//    otherwise);
//  * MUL_MAT: the generic warp-per-row GEMV (gemv_generic.cuh) for up to 8
//    activation vectors per launch; the host loops over batches of 8.
// These formats are not on the configs' hot path; the kernels favour one
// simple exact path over the pipelined designs of the three reference
// formats.
#include "api_internal.h"
#include "decode_ext.cuh"
#include "gemv_generic.cuh"

namespace spiral {
namespace {

template <int FMT, bool FTZ, bool VEC>
__global__ void __launch_bounds__(256)
    dequant_rows_ext(const uint8_t* __restrict__ src, int64_t src_stride, uint16_t* __restrict__ dst,
                     int64_t dst_stride, int64_t K, int64_t N) {
  constexpr int kBK = Fmt<FMT>::kBlockK, kBB = Fmt<FMT>::kBlockBytes;
  griddep_launch_dependents();
  griddep_wait();
  const int64_t chunks_per_row = K / 8;
  const int64_t total = chunks_per_row * N;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = c / chunks_per_row, kc = c - n * chunks_per_row;
    const int64_t blk = (kc * 8) / kBK;
    const int k8 = static_cast<int>(kc - blk * (kBK / 8));
    const uint4 r = decode8_generic<FMT>(src + n * src_stride + blk * kBB, k8, FTZ);
    uint16_t* o = dst + n * dst_stride + kc * 8;
    if constexpr (VEC) {
      *reinterpret_cast<uint4*>(o) = r;
    } else {
      const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[2 * j] = static_cast<uint16_t>(w[j] & 0xFFFFu);
        o[2 * j + 1] = static_cast<uint16_t>(w[j] >> 16);
      }
    }
  }
}

template <int FMT>
cudaError_t dequant_ext_t(const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int64_t K, int64_t N,
                          bool ftz, cudaStream_t stream) {
  const bool vec = (reinterpret_cast<uintptr_t>(dst) % 16 == 0) && (dst_stride % 8 == 0);
  auto* kernel = ftz ? (vec ? dequant_rows_ext<FMT, true, true> : dequant_rows_ext<FMT, true, false>)
                     : (vec ? dequant_rows_ext<FMT, false, true> : dequant_rows_ext<FMT, false, false>);
  const int64_t total = (K / 8) * N;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, int64_t(device_sm_count()) * 16);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(std::max<int64_t>(blocks, 1)));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<const uint8_t*>(src), src_stride, static_cast<uint16_t*>(dst),
                            dst_stride, K, N);
}

template <int FMT>
cudaError_t gemv_ext_t(const MatArgs& a, cudaStream_t stream) {
  const int64_t blocks = std::min<int64_t>((a.N + 7) / 8, int64_t(device_sm_count()) * 16);
  gemv_generic<FMT><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

bool fmt_is_ext(int fmt) {
  return fmt == kQ4_K || fmt == kQ5_K || fmt == kIQ4_NL || fmt == kIQ4_XS || fmt == kF16 || fmt == kBF16;
}

cudaError_t dequant_rows_ext(int fmt, const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int64_t K,
                             int64_t N, bool ftz, cudaStream_t stream) {
  switch (fmt) {
    case kQ4_K: return dequant_ext_t<kQ4_K>(src, src_stride, dst, dst_stride, K, N, ftz, stream);
    case kQ5_K: return dequant_ext_t<kQ5_K>(src, src_stride, dst, dst_stride, K, N, ftz, stream);
    case kIQ4_NL: return dequant_ext_t<kIQ4_NL>(src, src_stride, dst, dst_stride, K, N, ftz, stream);
    case kIQ4_XS: return dequant_ext_t<kIQ4_XS>(src, src_stride, dst, dst_stride, K, N, ftz, stream);
    case kF16: return dequant_ext_t<kF16>(src, src_stride, dst, dst_stride, K, N, ftz, stream);
    case kBF16: return dequant_ext_t<kBF16>(src, src_stride, dst, dst_stride, K, N, ftz, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t gemv_ext(const MatArgs& a, cudaStream_t stream) {
  switch (a.fmt) {
    case kQ4_K: return gemv_ext_t<kQ4_K>(a, stream);
    case kQ5_K: return gemv_ext_t<kQ5_K>(a, stream);
    case kIQ4_NL: return gemv_ext_t<kIQ4_NL>(a, stream);
    case kIQ4_XS: return gemv_ext_t<kIQ4_XS>(a, stream);
    case kF16: return gemv_ext_t<kF16>(a, stream);
    case kBF16: return gemv_ext_t<kBF16>(a, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace spiral
