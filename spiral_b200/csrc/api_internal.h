// api_internal.h — launcher declarations shared between the kernel files and
// the C-ABI layer (api.cu).  Launchers validate nothing: api.cu checks every
// argument before calling them.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "../../include/spiral_b200.h"

namespace spiral {

// dequant.cu
bool dequant_fast_ok(int fmt, const void* src, int64_t src_stride, const void* dst, int64_t dst_stride, int64_t K);
cudaError_t dequant_rows(int fmt, const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int64_t K,
                         int64_t N, bool ftz, cudaStream_t stream);
cudaError_t dequant_tiles_ref(int fmt, const void* src, int64_t src_stride, void* dst, int64_t K, int64_t N, bool ftz,
                              cudaStream_t stream);

// Generalised strided operands shared by the GEMV and GEMM paths:
//   x[m][k] at x + (k/8)*x_s8 + m*x_sm + (k%8)     (bf16 elements)
//   y[m][n] at y + (n/8)*y_s8 + m*y_sm + (n%8)     (y_dtype elements)
// Row-major operands use s8 = 8 and sm = row stride; the reference's tiled
// orders ([K/8][M][8], [N/8][M][8]) use s8 = 8*M and sm = 8.
struct MatArgs {
  int fmt;
  const uint8_t* w;
  int64_t w_stride;  // bytes between output-feature rows
  const uint16_t* x;
  int64_t x_s8, x_sm;
  void* y;
  int64_t y_s8, y_sm;
  bool y_bf16;
  bool accumulate;
  bool ftz;
  bool static_weights;  // weights are not written by the preceding kernel
  int64_t M, N, K;
};

// formats_ext.cu — Q4_K, Q5_K, IQ4_NL, IQ4_XS, F16, BF16.
bool fmt_is_ext(int fmt);
cudaError_t dequant_rows_ext(int fmt, const void* src, int64_t src_stride, void* dst, int64_t dst_stride, int64_t K,
                             int64_t N, bool ftz, cudaStream_t stream);
cudaError_t gemv_ext(const MatArgs& a, cudaStream_t stream);

// gemv.cu — M <= 8.
bool gemv_fast_ok(const MatArgs& a);
cudaError_t gemv(const MatArgs& a, cudaStream_t stream);

// Row-sharded GEMV with the all-gather fused in (gemv.cu): a.y is this
// rank's full bf16 output [M][a.y_sm]; the shard's rows are its columns
// [n_offset, n_offset + a.N); xchg_peers is a device array of `world`
// exchange buffers (gemv_xchg_bytes(n_total) each, zeroed before first use).
struct PeerOut {
  uint8_t* const* xchg_peers;
  int64_t n_offset, n_total;
  int rank, world;
};
int64_t gemv_xchg_bytes(int64_t n_total);
cudaError_t gemv_allgather(const MatArgs& a, const PeerOut& po, cudaStream_t stream);

// Exchange buffer of the gathered GEMV (one per rank, peer-mapped): a
// 256-byte control block (word 0: calls completed on this rank, word 1: CTA
// count of the running call) and two slots (call parity) of [8][n_total / 2]
// units.  A unit is 8 bytes, two bf16 outputs (columns 2u, 2u + 1) in the
// low word and the call's flag (call count | 2^31) in the high word, stored
// and loaded as one 64-bit access, so a reader that sees the flag sees the
// data: no fence is needed on either side.  Units travel in 16-byte pairs.
constexpr int64_t kGemvXchgCtrlBytes = 256;
__host__ __device__ constexpr int64_t gemv_xchg_slot_bytes(int64_t n_total) { return 8 * n_total * 4; }

// gemv_xs.cu — activation-stationary GEMV for Q4_0 / Q8_0 at K in {1536,
// 2048, 3072, 4096} and Q6_K at K = 4096; gemv() and gemv_allgather() use it
// whenever it applies.
// po == nullptr: plain MUL_MAT; else the row-sharded call with the
// all-gather fused in (same exchange protocol as above).
bool gemv_xs_ok(const MatArgs& a);
cudaError_t gemv_xs(const MatArgs& a, const PeerOut* po, cudaStream_t stream);

// gemv_xs6.cu — activation-stationary GEMV for Q6_K at K = 1536 with dense
// 1260-byte rows and N a multiple of 32 (the Gemma output head shape).
bool gemv_xs6_ok(const MatArgs& a);
cudaError_t gemv_xs6(const MatArgs& a, cudaStream_t stream);

// gemm.cu — tcgen05 dequant-GEMM for larger M.
bool gemm_supported(const MatArgs& a);
cudaError_t gemm(const MatArgs& a, cudaStream_t stream);

// repack.cu — canonical view -> dense canonical tensor with the reference's
// subnormal-scale flush and -128 report; synchronizes `stream` and emits at
// most one warning line through the hook.
cudaError_t repack(int fmt, const void* src, int64_t src_stride, void* dst, int64_t K, int64_t N,
                   cudaStream_t stream);
void repack_set_warn(spiral_repack_warn_fn_t fn, void* user);

// moe.cu — MoE FFN decode layer over quantized experts.
size_t moe_workspace_bytes(int64_t E_local, int64_t H, int64_t I, int64_t T, int64_t topk);
bool moe_shape_ok(int fmt, int64_t H, int64_t I);
cudaError_t moe_ffn(int fmt, const void* w_gate, const void* w_up, const void* w_down, const void* x,
                    int64_t x_stride, const int32_t* ids, const float* wts, void* y, int64_t y_stride, bool y_bf16,
                    bool accumulate, bool ftz, int64_t T, int64_t topk, int64_t H, int64_t I, int64_t e0,
                    int64_t E_local, void* ws, cudaStream_t stream);

// Expert-parallel MoE layer: the local experts' layer plus a fused combine
// of every rank's fp32 partial over peer-mapped exchange buffers
// (moe_ep_xchg_bytes each, zeroed before first use); y gets the whole layer.
int64_t moe_ep_xchg_bytes(int64_t H, int64_t max_tokens);
cudaError_t moe_ffn_ep(int fmt, const void* w_gate, const void* w_up, const void* w_down, const void* x,
                       int64_t x_stride, const int32_t* ids, const float* wts, void* y, int64_t y_stride, bool y_bf16,
                       bool accumulate, bool ftz, int64_t T, int64_t topk, int64_t H, int64_t I, int64_t e0,
                       int64_t E_local, void* ws, uint8_t* const* peers, int rank, int world, int64_t max_tokens,
                       cudaStream_t stream);

// Allocation-free MoE: capacity and device address (current device) of the
// library's static scratch array.
size_t moe_noalloc_scratch_bytes();
cudaError_t moe_noalloc_scratch(void** ptr);

// Device properties cached per device.
int device_sm_count();
size_t device_max_smem_optin();

}  // namespace spiral
