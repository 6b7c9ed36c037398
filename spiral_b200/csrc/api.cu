// api.cu — the extern "C" boundary of libspiral_b200.so.
//
// Host code is plain C-style: every entry point validates its arguments,
// picks a kernel, queues it on the caller's stream and returns a status.
// There is no host-side fallback: if a kernel cannot be launched the call
// fails with SPIRAL_ERR_CUDA and a message from spiral_last_error().
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "../../include/spiral_b200.h"
#include "api_internal.h"
#include "common.cuh"

namespace spiral {

__device__ uint32_t g_device_error = 0;

namespace {

thread_local char g_last_error[512] = {0};

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SPIRAL_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// The reference's three formats (every entry point) ...
bool fmt_valid(int fmt) { return fmt == kQ4_0 || fmt == kQ8_0 || fmt == kQ6_K; }
// ... and the extended ones (dequant and MUL_MAT only).
bool fmt_valid_any(int fmt) { return fmt_valid(fmt) || fmt_is_ext(fmt); }

// ggml's block size (weights) and type size (bytes) of each format.
int64_t block_k(int fmt) {
  switch (fmt) {
    case kQ4_0: return 32;
    case kQ8_0: return 32;
    case kQ6_K: return 256;
    case kQ4_K: return 256;
    case kQ5_K: return 256;
    case kIQ4_NL: return 32;
    case kIQ4_XS: return 256;
    case kF16: return 1;
    case kBF16: return 1;
  }
  return 0;
}
int64_t block_bytes(int fmt) {
  switch (fmt) {
    case kQ4_0: return 18;
    case kQ8_0: return 34;
    case kQ6_K: return 210;
    case kQ4_K: return 144;
    case kQ5_K: return 176;
    case kIQ4_NL: return 18;
    case kIQ4_XS: return 136;
    case kF16: return 2;
    case kBF16: return 2;
  }
  return 0;
}

int64_t row_bytes(int fmt, int64_t K) { return (K / block_k(fmt)) * block_bytes(fmt); }

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<int> g_smem_optin[kMaxDevices];

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 0;
  return dev;
}

// any_fmt: the entry point also takes the extended formats (whose kernels
// work in 8-weight chunks, so K must be a multiple of 8 for F16/BF16 too).
int check_shape(int fmt, int64_t K, int64_t N, bool any_fmt = false) {
  if (!(any_fmt ? fmt_valid_any(fmt) : fmt_valid(fmt))) {
    if (fmt_valid_any(fmt))
      return fail(SPIRAL_ERR_UNSUPPORTED, "format %d is supported by dequant and MUL_MAT only", fmt);
    return fail(SPIRAL_ERR_INVALID_FORMAT, "unknown quantized format %d", fmt);
  }
  if (K <= 0 || N <= 0) return fail(SPIRAL_ERR_INVALID_SHAPE, "dims must be positive (K=%lld N=%lld)", (long long)K,
                                    (long long)N);
  const int64_t unit = std::max<int64_t>(block_k(fmt), 8);
  if (K % unit != 0)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "K=%lld is not a multiple of the block size %lld", (long long)K,
                (long long)unit);
  return SPIRAL_OK;
}

}  // namespace

int device_sm_count() {
  const int dev = current_device();
  int v = g_sm_count[dev].load(std::memory_order_relaxed);
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    g_sm_count[dev].store(v, std::memory_order_relaxed);
  }
  return v;
}

size_t device_max_smem_optin() {
  const int dev = current_device();
  int v = g_smem_optin[dev].load(std::memory_order_relaxed);
  if (v <= 0) {
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0)
      v = 232448;
    g_smem_optin[dev].store(v, std::memory_order_relaxed);
  }
  return static_cast<size_t>(v);
}

}  // namespace spiral

using namespace spiral;

extern "C" {

int spiral_version(void) { return 100; }

const char* spiral_status_string(int status) {
  switch (status) {
    case SPIRAL_OK: return "ok";
    case SPIRAL_ERR_INVALID_FORMAT: return "invalid format";
    case SPIRAL_ERR_INVALID_SHAPE: return "invalid shape";
    case SPIRAL_ERR_NULL_POINTER: return "null pointer";
    case SPIRAL_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case SPIRAL_ERR_CAPACITY: return "buffer too small";
    case SPIRAL_ERR_CUDA: return "CUDA error";
    case SPIRAL_ERR_NCCL: return "NCCL error";
    case SPIRAL_ERR_TIMEOUT: return "timeout";
    case SPIRAL_ERR_UNSUPPORTED: return "unsupported";
    case SPIRAL_ERR_INVALID_ARGUMENT: return "invalid argument";
  }
  return "unknown status";
}

const char* spiral_last_error(void) { return g_last_error; }

int64_t spiral_quants_block_rows(int fmt) { return fmt_valid_any(fmt) ? block_k(fmt) : 0; }
int64_t spiral_quants_block_bytes(int fmt) { return fmt_valid_any(fmt) ? block_bytes(fmt) : 0; }

int64_t spiral_quants_record_count(int fmt, int64_t weights_rows, int64_t weights_cols) {
  if (!fmt_valid(fmt) || weights_rows <= 0 || weights_cols <= 0 || weights_rows % block_k(fmt) != 0) return 0;
  return (weights_rows / block_k(fmt)) * weights_cols;
}

int64_t spiral_quants_packed_bytes(int fmt, int64_t weights_rows, int64_t weights_cols) {
  return spiral_quants_record_count(fmt, weights_rows, weights_cols) * (fmt_valid(fmt) ? block_bytes(fmt) : 0);
}

int64_t spiral_quants_repack(int fmt, const void* src, int64_t src_col_stride_bytes, void* dst, int64_t dst_capacity,
                             int64_t weights_rows, int64_t weights_cols, void* stream) {
  g_last_error[0] = 0;
  const int64_t bytes = spiral_quants_packed_bytes(fmt, weights_rows, weights_cols);
  if (bytes == 0 || src == nullptr || dst == nullptr || bytes > dst_capacity) return 0;
  const int64_t rb = row_bytes(fmt, weights_rows);
  if (src_col_stride_bytes < rb) return 0;
  if ((reinterpret_cast<uintptr_t>(src) & 1u) || (reinterpret_cast<uintptr_t>(dst) & 1u) ||
      (src_col_stride_bytes & 1))
    return 0;
  const cudaError_t e = repack(fmt, src, src_col_stride_bytes, dst, weights_rows, weights_cols,
                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    cuda_fail(e, "repack");
    return 0;
  }
  return bytes;
}

void spiral_set_repack_warn(spiral_repack_warn_fn_t fn, void* user) { repack_set_warn(fn, user); }

int spiral_dequant_bf16(int fmt, const void* src, int64_t src_row_stride_bytes, void* dst,
                        int64_t dst_row_stride_elems, int64_t K, int64_t N, unsigned flags, void* stream) {
  g_last_error[0] = 0;
  if (int st = check_shape(fmt, K, N, true)) return st;
  if (src == nullptr || dst == nullptr) return fail(SPIRAL_ERR_NULL_POINTER, "null src or dst");
  if (src_row_stride_bytes < row_bytes(fmt, K))
    return fail(SPIRAL_ERR_INVALID_SHAPE, "src row stride %lld < row bytes %lld", (long long)src_row_stride_bytes,
                (long long)row_bytes(fmt, K));
  if (dst_row_stride_elems < K)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "dst row stride %lld < K %lld", (long long)dst_row_stride_elems,
                (long long)K);
  if ((reinterpret_cast<uintptr_t>(src) & 1u) || (src_row_stride_bytes & 1) || (reinterpret_cast<uintptr_t>(dst) & 1u))
    return fail(SPIRAL_ERR_ALIGNMENT, "src/dst and the src row stride must be 2-byte aligned");
  const cudaError_t e = dequant_rows(fmt, src, src_row_stride_bytes, dst, dst_row_stride_elems, K, N,
                                     (flags & SPIRAL_FLAG_FTZ_SCALES) != 0, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dequant launch");
  return SPIRAL_OK;
}

int spiral_quants_unpack_all(int fmt, const void* packed, void* weights_bf16, int64_t weights_rows,
                             int64_t weights_cols, unsigned flags, void* stream) {
  g_last_error[0] = 0;
  if (int st = check_shape(fmt, weights_rows, weights_cols)) return st;
  if (weights_cols % 8 != 0)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "weights_cols=%lld must be a multiple of 8", (long long)weights_cols);
  if (packed == nullptr || weights_bf16 == nullptr) return fail(SPIRAL_ERR_NULL_POINTER, "null packed or output");
  if ((reinterpret_cast<uintptr_t>(packed) & 1u) || (reinterpret_cast<uintptr_t>(weights_bf16) & 15u))
    return fail(SPIRAL_ERR_ALIGNMENT, "packed must be 2-byte and output 16-byte aligned");
  const cudaError_t e = dequant_tiles_ref(fmt, packed, row_bytes(fmt, weights_rows), weights_bf16, weights_rows,
                                          weights_cols, (flags & SPIRAL_FLAG_FTZ_SCALES) != 0,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "unpack_all launch");
  return SPIRAL_OK;
}

}  // extern "C"

namespace {

// Runs y = x W^T.  M <= 8: the fused GEMV.  Larger M: the tcgen05 GEMM when
// the operands allow it (row-major, 16-byte aligned, K % 256 == 0), else the
// GEMV over batches of at most 8 activation vectors.
int run_mat(MatArgs a, cudaStream_t stream) {
  const int64_t M = a.M;
  if (M > 8 && gemm_supported(a)) {
    const cudaError_t e = gemm(a, stream);
    if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
    return SPIRAL_OK;
  }
  for (int64_t m0 = 0; m0 < M; m0 += 8) {
    MatArgs b = a;
    b.M = std::min<int64_t>(8, M - m0);
    b.x = a.x + m0 * a.x_sm;
    if (a.y_bf16)
      b.y = static_cast<uint16_t*>(a.y) + m0 * a.y_sm;
    else
      b.y = static_cast<float*>(a.y) + m0 * a.y_sm;
    const cudaError_t e = gemv(b, stream);
    if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
  }
  return SPIRAL_OK;
}

}  // namespace

extern "C" {

int spiral_mul_mat(int fmt, const void* w, int64_t w_row_stride_bytes, const void* x, int64_t x_row_stride_elems,
                   void* y, int y_dtype, int64_t y_row_stride_elems, int64_t M, int64_t N, int64_t K, unsigned flags,
                   void* stream) {
  g_last_error[0] = 0;
  if (int st = check_shape(fmt, K, N, true)) return st;
  if (M <= 0) return fail(SPIRAL_ERR_INVALID_SHAPE, "M=%lld must be positive", (long long)M);
  if (w == nullptr || x == nullptr || y == nullptr) return fail(SPIRAL_ERR_NULL_POINTER, "null w, x or y");
  if (y_dtype != SPIRAL_DTYPE_BF16 && y_dtype != SPIRAL_DTYPE_F32)
    return fail(SPIRAL_ERR_INVALID_ARGUMENT, "y_dtype %d is neither F32 nor BF16", y_dtype);
  if ((flags & SPIRAL_FLAG_ACCUMULATE) && y_dtype != SPIRAL_DTYPE_F32)
    return fail(SPIRAL_ERR_INVALID_ARGUMENT, "ACCUMULATE needs an F32 destination");
  if (w_row_stride_bytes < row_bytes(fmt, K))
    return fail(SPIRAL_ERR_INVALID_SHAPE, "w row stride %lld < row bytes %lld", (long long)w_row_stride_bytes,
                (long long)row_bytes(fmt, K));
  if (x_row_stride_elems < K || y_row_stride_elems < N)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "x/y row strides smaller than K/N");
  if ((reinterpret_cast<uintptr_t>(w) & 1u) || (w_row_stride_bytes & 1) || (reinterpret_cast<uintptr_t>(x) & 1u) ||
      (reinterpret_cast<uintptr_t>(y) & (y_dtype == SPIRAL_DTYPE_F32 ? 3u : 1u)))
    return fail(SPIRAL_ERR_ALIGNMENT, "w/x/y misaligned for their element types");
  MatArgs a{};
  a.fmt = fmt;
  a.w = static_cast<const uint8_t*>(w);
  a.w_stride = w_row_stride_bytes;
  a.x = static_cast<const uint16_t*>(x);
  a.x_s8 = 8;
  a.x_sm = x_row_stride_elems;
  a.y = y;
  a.y_s8 = 8;
  a.y_sm = y_row_stride_elems;
  a.y_bf16 = y_dtype == SPIRAL_DTYPE_BF16;
  a.accumulate = (flags & SPIRAL_FLAG_ACCUMULATE) != 0;
  a.ftz = (flags & SPIRAL_FLAG_FTZ_SCALES) != 0;
  a.static_weights = (flags & SPIRAL_FLAG_STATIC_WEIGHTS) != 0;
  a.M = M;
  a.N = N;
  a.K = K;
  return run_mat(a, static_cast<cudaStream_t>(stream));
}

int spiral_quants_unpack_mmul_all(int fmt, const void* packed, const void* inputs_bf16, float* outputs,
                                  int64_t weights_rows, int64_t weights_cols, int64_t inputs_vecs, unsigned flags,
                                  void* stream) {
  g_last_error[0] = 0;
  if (int st = check_shape(fmt, weights_rows, weights_cols)) return st;
  if (weights_cols % 8 != 0 || weights_rows % 8 != 0)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "weights_rows and weights_cols must be multiples of 8");
  if (inputs_vecs <= 0) return fail(SPIRAL_ERR_INVALID_SHAPE, "inputs_vecs must be positive");
  if (packed == nullptr || inputs_bf16 == nullptr || outputs == nullptr)
    return fail(SPIRAL_ERR_NULL_POINTER, "null packed, inputs or outputs");
  if ((reinterpret_cast<uintptr_t>(packed) & 1u) || (reinterpret_cast<uintptr_t>(inputs_bf16) & 1u) ||
      (reinterpret_cast<uintptr_t>(outputs) & 3u))
    return fail(SPIRAL_ERR_ALIGNMENT, "packed/inputs/outputs misaligned");
  MatArgs a{};
  a.fmt = fmt;
  a.w = static_cast<const uint8_t*>(packed);
  a.w_stride = row_bytes(fmt, weights_rows);
  a.x = static_cast<const uint16_t*>(inputs_bf16);
  a.x_s8 = 8 * inputs_vecs;
  a.x_sm = 8;
  a.y = outputs;
  a.y_s8 = 8 * inputs_vecs;
  a.y_sm = 8;
  a.y_bf16 = false;
  a.accumulate = true;
  a.ftz = (flags & SPIRAL_FLAG_FTZ_SCALES) != 0;
  a.M = inputs_vecs;
  a.N = weights_cols;
  a.K = weights_rows;
  return run_mat(a, static_cast<cudaStream_t>(stream));
}

int64_t spiral_allgather_exchange_bytes(int64_t N_total) {
  if (N_total <= 0 || (N_total & 7)) return 0;
  return gemv_xchg_bytes(N_total);
}

int spiral_allgather_exchange_reset(void* exchange, int64_t N_total, void* stream) {
  g_last_error[0] = 0;
  const int64_t bytes = spiral_allgather_exchange_bytes(N_total);
  if (bytes == 0) return fail(SPIRAL_ERR_INVALID_SHAPE, "N_total=%lld: not a positive multiple of 8", (long long)N_total);
  if (!exchange) return fail(SPIRAL_ERR_NULL_POINTER, "null exchange");
  const cudaError_t e = cudaMemsetAsync(exchange, 0, static_cast<size_t>(bytes), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(SPIRAL_ERR_CUDA, "exchange reset: %s", cudaGetErrorString(e));
  return SPIRAL_OK;
}

int spiral_mul_mat_allgather(int fmt, const void* w_shard, int64_t w_row_stride_bytes, const void* x,
                             int64_t x_row_stride_elems, void* y, int64_t y_row_stride_elems, int64_t n_offset,
                             int64_t M, int64_t N_shard, int64_t N_total, int64_t K, void* const* exchange_peers,
                             int rank, int world, unsigned flags, void* stream) {
  g_last_error[0] = 0;
  if (int st = check_shape(fmt, K, N_shard)) return st;
  if (M <= 0 || M > 8) return fail(SPIRAL_ERR_INVALID_SHAPE, "M=%lld: the gathered GEMV takes 1..8 vectors", (long long)M);
  if (world < 1 || world > 64 || rank < 0 || rank >= world)
    return fail(SPIRAL_ERR_INVALID_ARGUMENT, "rank %d / world %d", rank, world);
  if (!w_shard || !x || !y || !exchange_peers) return fail(SPIRAL_ERR_NULL_POINTER, "null operand");
  if (n_offset < 0 || N_total < n_offset + N_shard || y_row_stride_elems < N_total)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "shard columns [%lld, %lld) outside the output of %lld (row stride %lld)",
                (long long)n_offset, (long long)(n_offset + N_shard), (long long)N_total,
                (long long)y_row_stride_elems);
  if (w_row_stride_bytes < row_bytes(fmt, K) || x_row_stride_elems < K)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "w/x row strides smaller than a row");
  if ((reinterpret_cast<uintptr_t>(w_shard) & 15u) || (w_row_stride_bytes & 15) || (reinterpret_cast<uintptr_t>(x) & 1u))
    return fail(SPIRAL_ERR_ALIGNMENT, "weights need 16-byte aligned rows");
  if ((reinterpret_cast<uintptr_t>(y) & 15u) || (y_row_stride_elems & 7) || (n_offset & 7) || (N_shard & 7) ||
      (N_total & 7))
    return fail(SPIRAL_ERR_ALIGNMENT,
                "gathered output: 16-byte aligned, row stride, shard offset, shard and total multiples of 8");
  MatArgs a{};
  a.fmt = fmt;
  a.w = static_cast<const uint8_t*>(w_shard);
  a.w_stride = w_row_stride_bytes;
  a.x = static_cast<const uint16_t*>(x);
  a.x_s8 = 8;
  a.x_sm = x_row_stride_elems;
  a.y = y;
  a.y_s8 = 8;
  a.y_sm = y_row_stride_elems;
  a.y_bf16 = true;
  a.ftz = (flags & SPIRAL_FLAG_FTZ_SCALES) != 0;
  a.static_weights = (flags & SPIRAL_FLAG_STATIC_WEIGHTS) != 0;
  a.M = M;
  a.N = N_shard;
  a.K = K;
  PeerOut po{reinterpret_cast<uint8_t* const*>(exchange_peers), n_offset, N_total, rank, world};
  const cudaError_t e = gemv_allgather(a, po, static_cast<cudaStream_t>(stream));
  if (e == cudaErrorNotSupported)
    return fail(SPIRAL_ERR_UNSUPPORTED, "shape not served by the pipelined GEMV (K=%lld)", (long long)K);
  if (e != cudaSuccess) return cuda_fail(e, "gathered gemv launch");
  return SPIRAL_OK;
}

int64_t spiral_moe_workspace_bytes(int64_t n_experts_local, int64_t hidden, int64_t inter, int64_t tokens,
                                   int64_t topk) {
  if (n_experts_local <= 0 || hidden <= 0 || inter <= 0 || tokens <= 0 || topk <= 0) return 0;
  if (tokens > (int64_t(1) << 24) || topk > 64 || n_experts_local > 4096) return 0;
  return static_cast<int64_t>(moe_workspace_bytes(n_experts_local, hidden, inter, tokens, topk));
}

int spiral_moe_ffn(int fmt, const void* w_gate, const void* w_up, const void* w_down, int64_t n_experts_local,
                   int64_t expert_first, int64_t hidden, int64_t inter, const void* x, int64_t x_row_stride_elems,
                   int64_t tokens, const int32_t* expert_ids, const float* expert_weights, int64_t topk, void* y,
                   int y_dtype, int64_t y_row_stride_elems, void* workspace, int64_t workspace_bytes, unsigned flags,
                   void* stream) {
  g_last_error[0] = 0;
  if (!fmt_valid(fmt)) return fail(SPIRAL_ERR_INVALID_FORMAT, "unknown quantized format %d", fmt);
  if (n_experts_local <= 0 || expert_first < 0 || tokens <= 0 || topk <= 0 || topk > 64 || hidden <= 0 ||
      inter <= 0 || n_experts_local > 4096 || tokens > (int64_t(1) << 24))
    return fail(SPIRAL_ERR_INVALID_SHAPE, "bad MoE dims (experts %lld, tokens %lld, topk %lld)",
                (long long)n_experts_local, (long long)tokens, (long long)topk);
  if (!moe_shape_ok(fmt, hidden, inter))
    return fail(SPIRAL_ERR_INVALID_SHAPE,
                "hidden=%lld / inter=%lld: need multiples of %d, hidden <= 4096 and inter <= 2048",
                (long long)hidden, (long long)inter, fmt == SPIRAL_QFMT_Q6_K ? 2048 : 256);
  if (!w_gate || !w_up || !w_down || !x || !expert_ids || !expert_weights || !y || !workspace)
    return fail(SPIRAL_ERR_NULL_POINTER, "null MoE operand");
  if (y_dtype != SPIRAL_DTYPE_BF16 && y_dtype != SPIRAL_DTYPE_F32)
    return fail(SPIRAL_ERR_INVALID_ARGUMENT, "y_dtype %d is neither F32 nor BF16", y_dtype);
  if ((flags & SPIRAL_FLAG_ACCUMULATE) && y_dtype != SPIRAL_DTYPE_F32)
    return fail(SPIRAL_ERR_INVALID_ARGUMENT, "ACCUMULATE needs an F32 destination");
  if (x_row_stride_elems < hidden || y_row_stride_elems < hidden)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "x/y row strides smaller than hidden");
  const auto al = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
  if (!al(w_gate, 16) || !al(w_up, 16) || !al(w_down, 16) || !al(x, 16) || (x_row_stride_elems % 8) != 0 ||
      !al(expert_ids, 4) || !al(expert_weights, 4) || !al(workspace, 256) ||
      !al(y, y_dtype == SPIRAL_DTYPE_F32 ? 4 : 2))
    return fail(SPIRAL_ERR_ALIGNMENT, "MoE operands misaligned (weights, x rows 16 B; workspace 256 B)");
  const int64_t need = spiral_moe_workspace_bytes(n_experts_local, hidden, inter, tokens, topk);
  if (workspace_bytes < need)
    return fail(SPIRAL_ERR_CAPACITY, "workspace %lld bytes < %lld needed", (long long)workspace_bytes,
                (long long)need);
  const cudaError_t e =
      moe_ffn(fmt, w_gate, w_up, w_down, x, x_row_stride_elems, expert_ids, expert_weights, y, y_row_stride_elems,
              y_dtype == SPIRAL_DTYPE_BF16, (flags & SPIRAL_FLAG_ACCUMULATE) != 0,
              (flags & SPIRAL_FLAG_FTZ_SCALES) != 0, tokens, topk, hidden, inter, expert_first, n_experts_local,
              workspace, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "moe launch");
  return SPIRAL_OK;
}

int64_t spiral_moe_ep_exchange_bytes(int64_t hidden, int64_t max_tokens) {
  if (hidden <= 0 || max_tokens <= 0 || max_tokens > (int64_t(1) << 24) || hidden > (int64_t(1) << 20)) return 0;
  return moe_ep_xchg_bytes(hidden, max_tokens);
}

int spiral_moe_ep_exchange_reset(void* exchange, int64_t hidden, int64_t max_tokens, void* stream) {
  g_last_error[0] = 0;
  const int64_t bytes = spiral_moe_ep_exchange_bytes(hidden, max_tokens);
  if (bytes == 0)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "hidden=%lld max_tokens=%lld", (long long)hidden, (long long)max_tokens);
  if (!exchange) return fail(SPIRAL_ERR_NULL_POINTER, "null exchange");
  const cudaError_t e = cudaMemsetAsync(exchange, 0, static_cast<size_t>(bytes), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(SPIRAL_ERR_CUDA, "exchange reset: %s", cudaGetErrorString(e));
  return SPIRAL_OK;
}

int spiral_moe_ffn_ep(int fmt, const void* w_gate, const void* w_up, const void* w_down, int64_t n_experts_local,
                      int64_t expert_first, int64_t hidden, int64_t inter, const void* x, int64_t x_row_stride_elems,
                      int64_t tokens, int64_t max_tokens, const int32_t* expert_ids, const float* expert_weights,
                      int64_t topk, void* y, int y_dtype, int64_t y_row_stride_elems, void* const* exchange_peers,
                      int rank, int world, void* workspace, int64_t workspace_bytes, unsigned flags, void* stream) {
  g_last_error[0] = 0;
  if (world < 1 || world > 64 || rank < 0 || rank >= world)
    return fail(SPIRAL_ERR_INVALID_ARGUMENT, "rank %d / world %d", rank, world);
  if (exchange_peers == nullptr) return fail(SPIRAL_ERR_NULL_POINTER, "null exchange_peers");
  if (tokens > max_tokens) return fail(SPIRAL_ERR_CAPACITY, "tokens %lld > max_tokens %lld", (long long)tokens,
                                        (long long)max_tokens);
  if (hidden % world != 0)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "hidden %lld is not a multiple of world %d", (long long)hidden, world);
  // the remaining rules are spiral_moe_ffn's
  if (!fmt_valid(fmt)) return fail(SPIRAL_ERR_INVALID_FORMAT, "unknown quantized format %d", fmt);
  if (n_experts_local <= 0 || expert_first < 0 || tokens <= 0 || topk <= 0 || topk > 64 || hidden <= 0 ||
      inter <= 0 || n_experts_local > 4096 || tokens > (int64_t(1) << 24))
    return fail(SPIRAL_ERR_INVALID_SHAPE, "bad MoE dims (experts %lld, tokens %lld, topk %lld)",
                (long long)n_experts_local, (long long)tokens, (long long)topk);
  if (!moe_shape_ok(fmt, hidden, inter))
    return fail(SPIRAL_ERR_INVALID_SHAPE,
                "hidden=%lld / inter=%lld: need multiples of %d, hidden <= 4096 and inter <= 2048",
                (long long)hidden, (long long)inter, fmt == SPIRAL_QFMT_Q6_K ? 2048 : 256);
  if (!w_gate || !w_up || !w_down || !x || !expert_ids || !expert_weights || !y || !workspace)
    return fail(SPIRAL_ERR_NULL_POINTER, "null MoE operand");
  if (y_dtype != SPIRAL_DTYPE_BF16 && y_dtype != SPIRAL_DTYPE_F32)
    return fail(SPIRAL_ERR_INVALID_ARGUMENT, "y_dtype %d is neither F32 nor BF16", y_dtype);
  if ((flags & SPIRAL_FLAG_ACCUMULATE) && y_dtype != SPIRAL_DTYPE_F32)
    return fail(SPIRAL_ERR_INVALID_ARGUMENT, "ACCUMULATE needs an F32 destination");
  if (x_row_stride_elems < hidden || y_row_stride_elems < hidden)
    return fail(SPIRAL_ERR_INVALID_SHAPE, "x/y row strides smaller than hidden");
  const auto al = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
  if (!al(w_gate, 16) || !al(w_up, 16) || !al(w_down, 16) || !al(x, 16) || (x_row_stride_elems % 8) != 0 ||
      !al(expert_ids, 4) || !al(expert_weights, 4) || !al(workspace, 256) ||
      !al(y, y_dtype == SPIRAL_DTYPE_F32 ? 4 : 2))
    return fail(SPIRAL_ERR_ALIGNMENT, "MoE operands misaligned (weights, x rows 16 B; workspace 256 B)");
  const int64_t need = spiral_moe_workspace_bytes(n_experts_local, hidden, inter, tokens, topk);
  if (workspace_bytes < need)
    return fail(SPIRAL_ERR_CAPACITY, "workspace %lld bytes < %lld needed", (long long)workspace_bytes,
                (long long)need);
  const cudaError_t e = moe_ffn_ep(fmt, w_gate, w_up, w_down, x, x_row_stride_elems, expert_ids, expert_weights, y,
                                   y_row_stride_elems, y_dtype == SPIRAL_DTYPE_BF16,
                                   (flags & SPIRAL_FLAG_ACCUMULATE) != 0, (flags & SPIRAL_FLAG_FTZ_SCALES) != 0,
                                   tokens, topk, hidden, inter, expert_first, n_experts_local, workspace,
                                   reinterpret_cast<uint8_t* const*>(exchange_peers), rank, world, max_tokens,
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "moe ep launch");
  return SPIRAL_OK;
}

int spiral_moe_ffn_noalloc(int fmt, const void* w_gate, const void* w_up, const void* w_down, int64_t n_experts_local,
                           int64_t expert_first, int64_t hidden, int64_t inter, const void* x,
                           int64_t x_row_stride_elems, int64_t tokens, const int32_t* expert_ids,
                           const float* expert_weights, int64_t topk, void* y, int y_dtype,
                           int64_t y_row_stride_elems, unsigned flags, void* stream) {
  g_last_error[0] = 0;
  const int64_t need = spiral_moe_workspace_bytes(n_experts_local, hidden, inter, tokens, topk);
  const int64_t cap = static_cast<int64_t>(moe_noalloc_scratch_bytes());
  if (need > cap)
    return fail(SPIRAL_ERR_CAPACITY,
                "these dims need %lld bytes of scratch; the allocation-free entry point has %lld (use "
                "spiral_moe_ffn with a workspace)",
                (long long)need, (long long)cap);
  void* scratch = nullptr;
  const cudaError_t e = moe_noalloc_scratch(&scratch);
  if (e != cudaSuccess) return cuda_fail(e, "static scratch address");
  return spiral_moe_ffn(fmt, w_gate, w_up, w_down, n_experts_local, expert_first, hidden, inter, x,
                        x_row_stride_elems, tokens, expert_ids, expert_weights, topk, y, y_dtype, y_row_stride_elems,
                        scratch, cap, flags, stream);
}

int spiral_device_status(void* stream, uint32_t* code) {
  g_last_error[0] = 0;
  if (code == nullptr) return fail(SPIRAL_ERR_NULL_POINTER, "null code");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "stream sync");
  uint32_t v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "read device error word");
  *code = v;
  if (v != 0) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "clear device error word");
    return fail(SPIRAL_ERR_TIMEOUT, "device reported error bits 0x%x", v);
  }
  return SPIRAL_OK;
}

}  // extern "C"
