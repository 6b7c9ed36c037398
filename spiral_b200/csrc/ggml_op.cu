// ggml_op.cu — the ggml backend boundary: MUL_MAT on ggml-style tensor
// descriptors (type, ne[4], nb[4], data), the call a ggml backend's graph
// compute makes for a GGML_OP_MUL_MAT node whose src0 is quantized (the
// reference's planned llama.cpp backend, README.md:11-14, TODO.md:49-55).
//
// ggml semantics (4-D, src0 broadcast over the batch dims):
//   dst[i3][i2][i1][i0] = sum_k src0[i3/r3][i2/r2][i0][k] * src1[i3][i2][i1][k]
//   with r2 = ne12 / ne02, r3 = ne13 / ne03,
// i.e. each (i2, i3) batch is one spiral_mul_mat with K = ne00, N = ne01,
// M = ne11.  Host code only: it validates and loops the batches.
#include "api_internal.h"

namespace {

// ggml's block size / type size; 0 for a type spiral_mul_mat does not take
// (every quantized format of spiral_qfmt and the F16 / BF16 pass-through).
int64_t ggml_block_k(int t) { return spiral_quants_block_rows(t); }
int64_t ggml_block_bytes(int t) { return spiral_quants_block_bytes(t); }

// 0 when the node is served, else the spiral_status that refuses it.
int ggml_check(const spiral_ggml_tensor* a, const spiral_ggml_tensor* b, const spiral_ggml_tensor* d) {
  if (a == nullptr || b == nullptr || d == nullptr) return SPIRAL_ERR_NULL_POINTER;
  if (ggml_block_k(a->type) <= 0) return SPIRAL_ERR_INVALID_FORMAT;
  if (b->type != SPIRAL_DTYPE_BF16) return SPIRAL_ERR_UNSUPPORTED;
  if (d->type != SPIRAL_DTYPE_BF16 && d->type != SPIRAL_DTYPE_F32) return SPIRAL_ERR_UNSUPPORTED;
  for (int i = 0; i < 4; ++i)
    if (a->ne[i] <= 0 || b->ne[i] <= 0 || d->ne[i] <= 0) return SPIRAL_ERR_INVALID_SHAPE;
  const int64_t K = a->ne[0];
  // whole blocks, and whole 8-weight chunks for the 2-byte types
  if (b->ne[0] != K || K % ggml_block_k(a->type) != 0 || K % 8 != 0) return SPIRAL_ERR_INVALID_SHAPE;
  if (d->ne[0] != a->ne[1] || d->ne[1] != b->ne[1] || d->ne[2] != b->ne[2] || d->ne[3] != b->ne[3])
    return SPIRAL_ERR_INVALID_SHAPE;
  if (b->ne[2] % a->ne[2] != 0 || b->ne[3] % a->ne[3] != 0) return SPIRAL_ERR_INVALID_SHAPE;
  // contiguous along K (one block / one element per step), rows at nb[1]
  const int64_t esize = d->type == SPIRAL_DTYPE_F32 ? 4 : 2;
  if (static_cast<int64_t>(a->nb[0]) != ggml_block_bytes(a->type) || static_cast<int64_t>(b->nb[0]) != 2 ||
      static_cast<int64_t>(d->nb[0]) != esize)
    return SPIRAL_ERR_UNSUPPORTED;
  if (b->nb[1] % 2 != 0 || d->nb[1] % esize != 0) return SPIRAL_ERR_ALIGNMENT;
  if (a->data == nullptr || b->data == nullptr || d->data == nullptr) return SPIRAL_ERR_NULL_POINTER;
  return SPIRAL_OK;
}

}  // namespace

extern "C" {

int spiral_ggml_supports_mul_mat(const spiral_ggml_tensor* src0, const spiral_ggml_tensor* src1,
                                 const spiral_ggml_tensor* dst) {
  return ggml_check(src0, src1, dst) == SPIRAL_OK ? 1 : 0;
}

int spiral_ggml_mul_mat(const spiral_ggml_tensor* src0, const spiral_ggml_tensor* src1, spiral_ggml_tensor* dst,
                        unsigned flags, void* stream) {
  if (int st = ggml_check(src0, src1, dst)) return st;
  const int64_t K = src0->ne[0], N = src0->ne[1], M = src1->ne[1];
  const int64_t r2 = src1->ne[2] / src0->ne[2], r3 = src1->ne[3] / src0->ne[3];
  const int64_t esize = dst->type == SPIRAL_DTYPE_F32 ? 4 : 2;
  for (int64_t i3 = 0; i3 < src1->ne[3]; ++i3) {
    for (int64_t i2 = 0; i2 < src1->ne[2]; ++i2) {
      const uint8_t* w = static_cast<const uint8_t*>(src0->data) + (i2 / r2) * src0->nb[2] + (i3 / r3) * src0->nb[3];
      const uint8_t* x = static_cast<const uint8_t*>(src1->data) + i2 * src1->nb[2] + i3 * src1->nb[3];
      uint8_t* y = static_cast<uint8_t*>(dst->data) + i2 * dst->nb[2] + i3 * dst->nb[3];
      const int st = spiral_mul_mat(src0->type, w, static_cast<int64_t>(src0->nb[1]), x,
                                    static_cast<int64_t>(src1->nb[1]) / 2, y, dst->type,
                                    static_cast<int64_t>(dst->nb[1]) / esize, M, N, K, flags, stream);
      if (st != SPIRAL_OK) return st;
    }
  }
  return SPIRAL_OK;
}

}  // extern "C"
