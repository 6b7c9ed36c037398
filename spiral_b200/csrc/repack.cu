// repack.cu — device-side repack of a canonical GGUF tensor view into the
// dense canonical layout every kernel here reads, with the reference's repack
// semantics (src/quants/q4_0/repack.h:27-111, q8_0/repack.h:26-91,
// q6_k/repack.h:28-115, common/repack.h:9-61):
//  * subnormal fp16 scales (exponent 0, mantissa != 0) are flushed to +0,
//    because the reference's device path decodes exponent 0 as zero;
//  * Q8_0 quants equal to -128 (0x80) are kept but reported;
//  * at most one warning line per call, worded as the reference's
//    RepackWarnings::warn, through a caller-replaceable hook (the reference's
//    QUANTS_REPACK_WARN macro; here a runtime callback, default stderr).
// The NPU record layout itself is not reproduced: the B200 kernels read
// canonical blocks in place, so the "record" is the canonical block.
#include <atomic>
#include <cstdio>
#include <mutex>

#include "api_internal.h"
#include "common.cuh"

namespace spiral {

enum : uint32_t { kRepackSubnormalScale = 1u, kRepackMinInt8 = 2u };

namespace {

// Per-call event words: a call takes slot (counter mod 64), so calls in
// flight on different streams (up to 64) do not share a word.
constexpr int kRepackSlots = 64;
__device__ uint32_t g_repack_events[kRepackSlots];
std::atomic<uint32_t> g_repack_next{0};

// One thread per block: copy it (2-byte granules: every block size and
// scale offset is even), flushing a subnormal scale and noting -128 quants.
template <int FMT>
__global__ void repack_blocks(const uint8_t* src, int64_t src_stride, uint8_t* dst, int64_t blocks_per_row,
                              int64_t rows, int slot) {
  constexpr int kBB = Fmt<FMT>::kBlockBytes;
  constexpr int kScaleAt = FMT == kQ6_K ? 208 : 0;
  const int64_t total = blocks_per_row * rows;
  uint32_t events = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / blocks_per_row, b = i - row * blocks_per_row;
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src + row * src_stride + b * kBB);
    uint16_t* d = reinterpret_cast<uint16_t*>(dst + (row * blocks_per_row + b) * kBB);
#pragma unroll 4
    for (int h = 0; h < kBB / 2; ++h) {
      uint32_t v = s[h];
      if (h == kScaleAt / 2) {
        if ((v & 0x7C00u) == 0u && (v & 0x03FFu) != 0u) {
          v = 0u;
          events |= kRepackSubnormalScale;
        }
      } else if (FMT == kQ8_0) {
        if ((v & 0xFFu) == 0x80u || (v >> 8) == 0x80u) events |= kRepackMinInt8;
      }
      d[h] = static_cast<uint16_t>(v);
    }
  }
  if (events) atomicOr(&g_repack_events[slot], events);
}

void default_warn(const char* line, void*) { fputs(line, stderr); }

std::mutex g_warn_mu;
spiral_repack_warn_fn_t g_warn_fn = default_warn;
void* g_warn_user = nullptr;

}  // namespace

void repack_set_warn(spiral_repack_warn_fn_t fn, void* user) {
  std::lock_guard<std::mutex> lk(g_warn_mu);
  g_warn_fn = fn;
  g_warn_user = user;
}

// One line per call, as the reference's RepackWarnings::warn words it.
static void repack_warn(const char* format, uint32_t events) {
  if (!(events & (kRepackSubnormalScale | kRepackMinInt8))) return;
  char line[160];
  if ((events & kRepackSubnormalScale) && (events & kRepackMinInt8)) {
    snprintf(line, sizeof line,
             "quants: %s repack flushed subnormal fp16 scales to zero and found -128 int8 weights\n", format);
  } else if (events & kRepackSubnormalScale) {
    snprintf(line, sizeof line, "quants: %s repack flushed subnormal fp16 scales to zero\n", format);
  } else {
    snprintf(line, sizeof line, "quants: %s repack found -128 int8 weights\n", format);
  }
  std::lock_guard<std::mutex> lk(g_warn_mu);
  if (g_warn_fn != nullptr) g_warn_fn(line, g_warn_user);
}

cudaError_t repack(int fmt, const void* src, int64_t src_stride, void* dst, int64_t K, int64_t N,
                   cudaStream_t stream) {
  const int slot = static_cast<int>(g_repack_next.fetch_add(1, std::memory_order_relaxed) % kRepackSlots);
  const uint32_t zero = 0;
  cudaError_t e = cudaMemcpyToSymbolAsync(g_repack_events, &zero, sizeof(zero), slot * sizeof(uint32_t),
                                          cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return e;
  const int64_t bk = fmt == kQ6_K ? 256 : 32;
  const int64_t bpr = K / bk, total = bpr * N;
  const int threads = 256;
  const int64_t grid = std::min<int64_t>((total + threads - 1) / threads, int64_t(device_sm_count()) * 16);
  const auto* s = static_cast<const uint8_t*>(src);
  auto* d = static_cast<uint8_t*>(dst);
  const char* name = "Q4_0";
  switch (fmt) {
    case kQ4_0: repack_blocks<kQ4_0><<<static_cast<unsigned>(grid), threads, 0, stream>>>(s, src_stride, d, bpr, N, slot); break;
    case kQ8_0: name = "Q8_0"; repack_blocks<kQ8_0><<<static_cast<unsigned>(grid), threads, 0, stream>>>(s, src_stride, d, bpr, N, slot); break;
    case kQ6_K: name = "Q6_K"; repack_blocks<kQ6_K><<<static_cast<unsigned>(grid), threads, 0, stream>>>(s, src_stride, d, bpr, N, slot); break;
    default: return cudaErrorInvalidValue;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  uint32_t events = 0;
  e = cudaMemcpyFromSymbolAsync(&events, g_repack_events, sizeof(events), slot * sizeof(uint32_t),
                                cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return e;
  repack_warn(name, events);
  return cudaSuccess;
}

}  // namespace spiral
