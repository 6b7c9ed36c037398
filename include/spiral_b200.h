/*
 * spiral_b200.h — C-ABI of the B200 (sm_100a) quantized-weight library.
 *
 * The library dequantizes canonical GGUF Q4_0, Q8_0 and Q6_K weights to bf16
 * and runs the quantized MUL_MAT (quantized src0 x bf16 src1) that consumes
 * them, on NVIDIA B200 GPUs.  Everything here is plain C: pointers, sizes,
 * integer enums.  Device pointers are CUDA device (or managed) pointers; a
 * `stream` argument is a cudaStream_t passed as `void*` (NULL = legacy default
 * stream).  Calls are stream-ordered and return as soon as the work is queued.
 *
 * Naming follows the reference's weight-matrix vocabulary
 * (spiral src/quants/TODO.md:246-266):
 *   weights_rows = K  (reduction length, = inputs_len)
 *   weights_cols = N  (output features, = outputs_len)
 *   inputs_vecs  = M  (number of activation vectors)
 * GGUF stores the weight matrix "column-major" in that vocabulary: each of
 * the N output features holds its K weights as consecutive blocks.  In ggml
 * terms that is src0 with ne0 = K, ne1 = N, one row per output feature.
 *
 * Numerics (all formats): a weight is fp16 scale x integer, computed exactly
 * in fp32 and rounded once to bf16 round-to-nearest-even.  This equals the
 * reference oracle (src/quants/tests/formats/q4_0.py:42-62, q8_0.py:43-60,
 * q6_k.py:55-112, cast with ml_dtypes bfloat16) bit for bit.  Subnormal fp16
 * scales are decoded exactly by default (GGUF semantics); SPIRAL_FLAG_FTZ_SCALES
 * flushes them to +0 as the reference NPU device path does
 * (src/quants/common/repack.h:29-34, common/scale.aie.h:9-13).
 *
 * Errors: every int-returning call returns SPIRAL_OK (0) or a negative
 * spiral_status.  Size queries and the repack return 0 on invalid input,
 * exactly like the reference's record_count / packed_bytes / repack_weights
 * (src/quants/q4_0/repack.h:10-41, TODO.md:331-334).  Nothing throws or traps.
 *
 * Per-device state: the first call on a device sets the kernels' shared-memory
 * limits and caches the device's SM count and attributes (and, for
 * spiral_moe_ffn_noalloc, its scratch address) for the process.  None of it
 * survives cudaDeviceReset or any other reset of the device's primary
 * context: after one, load the library into a new process before calling it.
 */
#ifndef SPIRAL_B200_H
#define SPIRAL_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SPIRAL_API __attribute__((visibility("default")))
#else
#define SPIRAL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Quantized formats.  The values are ggml's `enum ggml_type` ids, so a ggml
 * backend can pass src0->type straight through. */
typedef enum spiral_qfmt {
  SPIRAL_QFMT_Q4_0 = 2,  /* 18-byte block: fp16 d, 16 B nibbles; w=(q-8)*d   */
  SPIRAL_QFMT_Q8_0 = 8,  /* 34-byte block: fp16 d, 32 int8;      w=q*d       */
  SPIRAL_QFMT_Q6_K = 14, /* 210-byte super-block of 256: ql[128] qh[64]
                            sc[16] d; w=d*sc*(q-32)                          */
  /* Extended formats (ggml's layouts; spiral_dequant_bf16, spiral_mul_mat
   * and the ggml boundary only, K a multiple of the block size and of 8):  */
  SPIRAL_QFMT_F16 = 1,     /* 2 bytes per weight; w = bf16_rne(f16)          */
  SPIRAL_QFMT_Q4_K = 12,   /* 144-byte super-block of 256: fp16 d, dmin,
                              12 B of 6-bit (scale, min) pairs, 128 B nibbles;
                              w = (d*sc)*q - dmin*m                          */
  SPIRAL_QFMT_Q5_K = 13,   /* 176 bytes: Q4_K plus qh[32] (the fifth bit)    */
  SPIRAL_QFMT_IQ4_NL = 20, /* 18-byte block of 32: fp16 d, 16 B codebook
                              nibbles; w = d * kvalues[q]                    */
  SPIRAL_QFMT_IQ4_XS = 23, /* 136-byte super-block of 256: fp16 d, 6-bit
                              sub-scales ls; w = (d*(ls-32)) * kvalues[q]    */
  SPIRAL_QFMT_BF16 = 30    /* 2 bytes per weight, used as is                 */
} spiral_qfmt;

/* Output element types (ggml type ids). */
typedef enum spiral_dtype {
  SPIRAL_DTYPE_F32 = 0,
  SPIRAL_DTYPE_BF16 = 30
} spiral_dtype;

typedef enum spiral_status {
  SPIRAL_OK = 0,
  SPIRAL_ERR_INVALID_FORMAT = -1,  /* fmt is not one of spiral_qfmt          */
  SPIRAL_ERR_INVALID_SHAPE = -2,   /* non-positive dims, K not a block multiple,
                                      stride smaller than a row               */
  SPIRAL_ERR_NULL_POINTER = -3,
  SPIRAL_ERR_ALIGNMENT = -4,       /* pointer/stride alignment the op needs   */
  SPIRAL_ERR_CAPACITY = -5,        /* caller buffer or workspace too small    */
  SPIRAL_ERR_CUDA = -6,            /* a CUDA runtime call failed              */
  SPIRAL_ERR_NCCL = -7,            /* a NCCL call failed                      */
  SPIRAL_ERR_TIMEOUT = -8,         /* a bounded device or host wait gave up   */
  SPIRAL_ERR_UNSUPPORTED = -9,     /* valid request this build cannot serve   */
  SPIRAL_ERR_INVALID_ARGUMENT = -10
} spiral_status;

/* Flags (bit set). */
#define SPIRAL_FLAG_FTZ_SCALES 0x1u  /* flush subnormal fp16 scales to +0      */
#define SPIRAL_FLAG_ACCUMULATE 0x2u  /* mul_mat: dst += result (f32 dst only)  */
/* mul_mat, M <= 8: the weights are not written by the kernel queued just
 * before this call on the stream (true for inference weights), so the GEMV
 * may start streaming them while that kernel finishes.  Activations are
 * always read, and outputs written, only after the preceding kernel ends. */
#define SPIRAL_FLAG_STATIC_WEIGHTS 0x4u

/* ---------------------------------------------------------------- info --- */

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
SPIRAL_API int spiral_version(void);

/* Static text for a status code. */
SPIRAL_API const char* spiral_status_string(int status);

/* Detail text of the last error raised on the calling host thread ("" when
 * none).  Valid until the next library call on the same thread. */
SPIRAL_API const char* spiral_last_error(void);

/* Synchronizes `stream`, then reads and clears the device-side error word of
 * the current device into *code.  Kernels never trap: a bounded wait (an
 * mbarrier or peer flag) that gives up sets a bit (1 = pipeline wait timeout,
 * 2 = tensor-memory allocation failure, 4 = bad launch geometry, 8 = a
 * rank's gathered-GEMV pieces never arrived) and the kernel ends early.  Returns SPIRAL_ERR_TIMEOUT when any bit was set.
 * No reference counterpart: the reference's only device watchdog is the XRT
 * run.wait2(5000 ms) host timeout (tests/poc/invoke.cc:25-26, 126-131). */
SPIRAL_API int spiral_device_status(void* stream, uint32_t* code);

/* Weights per block (32, 32, 256) and bytes per block (18, 34, 210); 0 for an
 * unknown format.  Mirrors the per-format kBlockRows / kBlockBytes constants
 * of src/quants/<fmt>/layout.h (q4_0/layout.h:10-12, q8_0/layout.h:10-13,
 * q6_k/layout.h:10-15).  The extended formats report ggml's block and type
 * sizes (Q4_K 256/144, Q5_K 256/176, IQ4_NL 32/18, IQ4_XS 256/136, F16 and
 * BF16 1/2). */
SPIRAL_API int64_t spiral_quants_block_rows(int fmt);
SPIRAL_API int64_t spiral_quants_block_bytes(int fmt);

/* ------------------------------------------------- size queries / repack -- */

/* Number of canonical blocks of a weights_rows x weights_cols tensor, or 0 if
 * the shape is invalid (non-positive, or weights_rows not a multiple of the
 * block's weight count).
 * Replaces: extern "C" int64_t quants_record_count(rows, cols)
 *           (src/quants/tests/repack.cc:13-16).  The reference counts NPU
 *           records; the B200 kernels read canonical GGUF blocks directly, so
 *           the record here is the canonical block. */
SPIRAL_API int64_t spiral_quants_record_count(int fmt, int64_t weights_rows,
                                   int64_t weights_cols);

/* Dense canonical bytes of the tensor (record_count * block bytes), 0 if
 * invalid.
 * Replaces: extern "C" int64_t quants_packed_bytes(rows, cols)
 *           (src/quants/tests/repack.cc:18-21). */
SPIRAL_API int64_t spiral_quants_packed_bytes(int fmt, int64_t weights_rows,
                                   int64_t weights_cols);

/* Device-side repack of a (possibly padded) canonical tensor view into the
 * dense device layout every kernel here reads: weights_cols rows of
 * packed_bytes/weights_cols bytes.  `src` and `dst` are device pointers
 * (2-byte aligned); src_col_stride_bytes >= the dense row size and even.
 * As the reference's repack does, subnormal fp16 scales are flushed to +0
 * (its device path decodes exponent 0 as zero; q4_0/repack.h:75-80,
 * q6_k/repack.h:64-67) and Q8_0 quants of -128 are kept but reported
 * (q8_0/repack.h:76-78): at most one warning line per call, worded as the
 * reference's (common/repack.h:36-58), goes to the hook set by
 * spiral_set_repack_warn (default: stderr).  The call synchronizes `stream`
 * (it must read the device's report before it returns, as the reference's
 * host repack returns only when done).  Returns bytes written, or 0 on
 * invalid dims, insufficient capacity, null or misaligned pointers or a CUDA
 * error.
 * Replaces: extern "C" int64_t quants_repack(src, src_col_stride_bytes, dst,
 *           dst_capacity, rows, cols) (src/quants/tests/repack.cc:23-32,
 *           q4_0/repack.h:27-41).  Same argument meaning and return contract;
 *           the destination layout is canonical GGUF instead of NPU records. */
SPIRAL_API int64_t spiral_quants_repack(int fmt, const void* src,
                             int64_t src_col_stride_bytes, void* dst,
                             int64_t dst_capacity, int64_t weights_rows,
                             int64_t weights_cols, void* stream);

/* Receiver of the repack's one-line warnings ('\n'-terminated text).
 * Replaces the reference's overridable QUANTS_REPACK_WARN macro
 * (src/quants/common/repack.h:9-14): pass a function to route the line into
 * the caller's logger, or NULL to suppress it; the default writes to stderr.
 * Process-wide; the hook may be called from any host thread that repacks. */
typedef void (*spiral_repack_warn_fn_t)(const char* line, void* user);
SPIRAL_API void spiral_set_repack_warn(spiral_repack_warn_fn_t fn, void* user);

/* ------------------------------------------------------ dequant-to-bf16 -- */

/* ggml-style dequantize (to_float / dequantize_row_* semantics):
 *   dst[n * dst_row_stride_elems + k] = bf16(W[n][k]),  n < N, k < K
 * src: device pointer to N rows of K/blk canonical blocks, row n at
 * src + n * src_row_stride_bytes.  dst: device bf16 (uint16_t) buffer.
 * Bit-exact against the reference oracle (see header comment).
 * Fast path: 16-byte aligned src/dst, 16-byte multiple strides and
 * K % 256 == 0 (Q4_0/Q8_0) or K % 2048 == 0 (Q6_K); other valid shapes run a
 * slower scalar-load kernel with the same results. */
SPIRAL_API int spiral_dequant_bf16(int fmt, const void* src, int64_t src_row_stride_bytes,
                        void* dst, int64_t dst_row_stride_elems, int64_t K,
                        int64_t N, unsigned flags, void* stream);

/* Dequantize a dense canonical tensor into the reference's bf16 weights
 * stream order [weights_cols/8][weights_rows][8] (the order of
 * formats/<fmt>.py reference_weights: [cols_tile][rows_record][chunk]
 * [kUnpackTileRows][kTileCols], which flattens to [cols/8][rows][8]).
 * weights_cols must be a multiple of 8 (kTileCols).
 * Replaces: extern "C" void quants_unpack_all(const uint8_t* packed,
 *           bfloat16* out) (src/quants/tests/unpack.aie.cc:21-45), whose
 *           format and shape are compile-time macros there and arguments here.
 */
SPIRAL_API int spiral_quants_unpack_all(int fmt, const void* packed, void* weights_bf16,
                             int64_t weights_rows, int64_t weights_cols,
                             unsigned flags, void* stream);

/* ------------------------------------------------------------ MUL_MAT ---- */

/* ggml MUL_MAT with a quantized src0 and a bf16 src1:
 *   y[m][n] = sum_k bf16(W[n][k]) * x[m][k],   m < M, n < N
 * accumulated in fp32 and stored as y_dtype (BF16 rounds once, RNE; F32 with
 * SPIRAL_FLAG_ACCUMULATE adds into y).
 * w: N rows of canonical blocks at w_row_stride_bytes; x: M rows of K bf16 at
 * x_row_stride_elems; y: M rows of N at y_row_stride_elems.
 * M <= 8 runs the fused dequant-GEMV (decode); larger M runs the tcgen05
 * dequant-GEMM (prefill).  Results are within fp32-summation-order error of
 * the reference's dequant-then-fp32-matmul (src/quants/tests/mmul.py:104-121)
 * and identical from run to run (fixed summation order).  Nothing is
 * allocated.  The GEMV is launched with programmatic stream serialization
 * so that the next kernel on the stream can be scheduled while it finishes.
 */
SPIRAL_API int spiral_mul_mat(int fmt, const void* w, int64_t w_row_stride_bytes,
                   const void* x, int64_t x_row_stride_elems, void* y,
                   int y_dtype, int64_t y_row_stride_elems, int64_t M,
                   int64_t N, int64_t K, unsigned flags, void* stream);

/* Row-sharded MUL_MAT with the output all-gather fused into the kernel, for
 * one process per GPU (BASELINE config 2 at 2..8 GPUs; the reference has no
 * multi-device path — its multi-tile pattern splits weights by output column
 * and broadcasts the input, src/quants/tests/poc/calc.py:1-11, 154-215).
 * This rank computes y[m][n_offset + n] = sum_k bf16(Wshard[n][k]) x[m][k],
 * n < N_shard, m < M <= 8, into its full bf16 output y [M][N_total] (row
 * stride y_row_stride_elems) and sends the same values to every other
 * rank's exchange buffer over NVLink; it then copies the other ranks'
 * columns from its own exchange buffer into y.  The kernel completes only
 * with all N_total columns in y, so work queued after it on the stream sees
 * the whole gathered output; y itself is never written by another rank.
 * exchange_peers: DEVICE array of `world` device pointers, rank r's
 * exchange buffer (spiral_allgather_exchange_bytes(N_total) bytes, 16-byte
 * aligned, peer-mapped on every rank, e.g. by a symmetric-memory rendezvous,
 * zeroed once before the first call).  Shards must be disjoint and cover
 * [0, N_total); n_offset, N_shard, N_total and the row stride multiples of
 * 8, y 16-byte aligned.  Every rank makes the same calls in the same order,
 * with no other kernel running on its GPU meanwhile (the grid, one CTA per
 * SM, must be co-resident), and calls on one exchange never overlap (one
 * stream, or streams ordered by events).  A rank that does not arrive makes
 * the others' bounded waits (2 s) give up with bit 8 of spiral_device_status;
 * the ranks' call counts then disagree, so later calls skip their waits
 * until the status is read, and the exchanges must be zeroed again on every
 * rank before further use (spiral_allgather_exchange_reset).  The gathered
 * columns of every call since the timeout are invalid; each rank's own
 * columns are complete. */
SPIRAL_API int64_t spiral_allgather_exchange_bytes(int64_t N_total);
/* Zero this rank's exchange buffer on the stream, as before the first call:
 * the recovery after a peer timeout.  Peers read and write this buffer, so
 * every rank first finishes its calls on the exchange (stream synchronize,
 * then a host barrier), resets its own exchange, and the ranks meet at a
 * host barrier again before the next gathered call. */
SPIRAL_API int spiral_allgather_exchange_reset(void* exchange, int64_t N_total, void* stream);
SPIRAL_API int spiral_mul_mat_allgather(int fmt, const void* w_shard, int64_t w_row_stride_bytes,
                                        const void* x, int64_t x_row_stride_elems,
                                        void* y, int64_t y_row_stride_elems, int64_t n_offset,
                                        int64_t M, int64_t N_shard, int64_t N_total, int64_t K,
                                        void* const* exchange_peers, int rank, int world,
                                        unsigned flags, void* stream);

/* ggml backend boundary.  A tensor as a ggml backend sees it: ggml type id,
 * elements per dimension (ne[0] innermost) and bytes between consecutive
 * elements of each dimension (nb[0] = block bytes for a quantized row,
 * element size otherwise), data on the device.  Field meaning as ggml's
 * struct ggml_tensor, so a backend fills it from its node's tensors. */
typedef struct spiral_ggml_tensor {
  int32_t type;
  int64_t ne[4];
  size_t nb[4];
  void* data;
} spiral_ggml_tensor;

/* supports_op for GGML_OP_MUL_MAT: 1 when spiral_ggml_mul_mat serves the
 * node (src0 Q4_0 / Q8_0 / Q6_K, src1 BF16, dst F32 or BF16, rows
 * contiguous along K, ggml's shape and broadcast rules), else 0.  The
 * reference's planned llama.cpp backend (README.md:11-14, TODO.md:49-55)
 * offers these src0 types to ggml the same way. */
SPIRAL_API int spiral_ggml_supports_mul_mat(const spiral_ggml_tensor* src0, const spiral_ggml_tensor* src1,
                                            const spiral_ggml_tensor* dst);

/* GGML_OP_MUL_MAT with ggml's semantics: for every batch (i2, i3) of src1,
 *   dst[i3][i2][i1][i0] = sum_k src0[i3/r3][i2/r2][i0][k] * src1[i3][i2][i1][k]
 * (r2 = ne12/ne02, r3 = ne13/ne03: src0 broadcast over the batch dims), each
 * batch one spiral_mul_mat (same numerics and flags).  Returns the first
 * non-zero status, or the status that supports_mul_mat refuses with. */
SPIRAL_API int spiral_ggml_mul_mat(const spiral_ggml_tensor* src0, const spiral_ggml_tensor* src1,
                                   spiral_ggml_tensor* dst, unsigned flags, void* stream);

/* Fused unpack + mmul in the reference's tiled I/O orders:
 *   inputs  bf16 [weights_rows/8][inputs_vecs][8]
 *   outputs f32  [weights_cols/8][inputs_vecs][8], ACCUMULATED (+=); the
 *           caller zeroes them, as the reference shim does.
 * weights: dense canonical tensor.  weights_rows % 8 == 0 and
 * weights_cols % 8 == 0 are required by the tiled orders.
 * Replaces: extern "C" void quants_unpack_mmul_all(const uint8_t* packed,
 *           const bfloat16* inputs, float* outputs)
 *           (src/quants/tests/mmul.aie.cc:20-35; layouts mmul.py:22-35,
 *           113-118), with format/shape as arguments instead of macros. */
SPIRAL_API int spiral_quants_unpack_mmul_all(int fmt, const void* packed,
                                  const void* inputs_bf16, float* outputs,
                                  int64_t weights_rows, int64_t weights_cols,
                                  int64_t inputs_vecs, unsigned flags,
                                  void* stream);

/* ------------------------------------------------------------ MoE FFN ---- */

/* Bytes of scratch spiral_moe_ffn needs for these dims (0 if invalid).  The
 * caller allocates it once (device memory, 256-byte aligned) and may reuse it
 * for every call with the same or smaller dims on one stream. */
SPIRAL_API int64_t spiral_moe_workspace_bytes(int64_t n_experts_local, int64_t hidden,
                                              int64_t inter, int64_t tokens, int64_t topk);

/* MoE FFN decode layer with quantized SwiGLU experts (the
 * reference has no MoE operator — this is the expert FFN built from its
 * quantized MUL_MAT, src/quants/q4_0/mmul.aie.h:16-90):
 *   for each token t and slot j < topk with global expert id e = ids[t][j]
 *   in [expert_first, expert_first + n_experts_local):
 *     h = bf16( silu(x_t Wg_e^T) * (x_t Wu_e^T) )       (inter values)
 *     y_t += weights[t][j] * (h Wd_e^T)                  (hidden values)
 *   accumulated in fp32, summed over slots in order j = 0..topk-1, stored as
 *   y_dtype (BF16 rounds once; F32 with SPIRAL_FLAG_ACCUMULATE adds into y).
 * Ids outside the local range (or negative) are skipped, so expert-parallel
 * ranks each produce their partial y and combine them.
 * w_gate, w_up: n_experts_local x [inter rows][hidden] canonical tensors,
 * back to back; w_down: n_experts_local x [hidden rows][inter].  Rows dense
 * (row bytes = K / block * block bytes).  hidden and inter multiples of 256
 * (Q6_K: 2048), hidden <= 4096, inter <= 2048.  x: [tokens][x_row_stride]
 * bf16, 16-byte aligned rows.  ids int32 / weights f32: [tokens][topk]. */
SPIRAL_API int spiral_moe_ffn(int fmt, const void* w_gate, const void* w_up, const void* w_down,
                              int64_t n_experts_local, int64_t expert_first, int64_t hidden,
                              int64_t inter, const void* x, int64_t x_row_stride_elems,
                              int64_t tokens, const int32_t* expert_ids,
                              const float* expert_weights, int64_t topk, void* y, int y_dtype,
                              int64_t y_row_stride_elems, void* workspace,
                              int64_t workspace_bytes, unsigned flags, void* stream);

/* Bytes of one rank's exchange buffer for spiral_moe_ffn_ep (0 if invalid:
 * non-positive dims).  Sized for up to max_tokens tokens per call. */
SPIRAL_API int64_t spiral_moe_ep_exchange_bytes(int64_t hidden, int64_t max_tokens);
/* Zero this rank's spiral_moe_ffn_ep exchange buffer on the stream, as
 * before the first call: the recovery after a peer timeout, with the same
 * barriers around it as spiral_allgather_exchange_reset. */
SPIRAL_API int spiral_moe_ep_exchange_reset(void* exchange, int64_t hidden, int64_t max_tokens, void* stream);

/* Expert-parallel MoE FFN layer, one process per GPU (BASELINE config 4 at
 * 2..8 GPUs; the reference has no MoE and no multi-device path, its
 * multi-tile pattern splits weights and broadcasts the input,
 * src/quants/tests/poc/calc.py:1-11, 154-215).  Every rank passes the same
 * tokens: x [tokens][hidden], expert_ids and expert_weights [tokens][topk]
 * (global expert ids), as they are after the preceding dense layer's
 * all-gather; rank r holds the experts [expert_first, expert_first +
 * n_experts_local) in w_gate / w_up / w_down as spiral_moe_ffn takes them.
 * Each rank runs its local experts (spiral_moe_ffn's kernels, ids of other
 * ranks' experts skipped), then one kernel combines the ranks' fp32 partial
 * layers over NVLink: the partials of each column go to the column's owner
 * (hidden / world columns each), which sums them in rank order and sends
 * the sum to every rank.  On return every rank's y holds the whole layer
 * output, identical on all ranks: for every token, the sum over all its topk
 * slots (slots of one rank in slot order, ranks in rank order), stored as
 * y_dtype (ACCUMULATE adds into an F32 y).  With top-8 of 128 experts over
 * at most 8 ranks nearly every token reaches every rank, so the tokens are
 * replicated rather than dispatched with an all-to-all.
 * exchange_peers: DEVICE array of `world` device pointers, rank r's exchange
 * buffer (spiral_moe_ep_exchange_bytes(hidden, max_tokens) bytes, 16-byte
 * aligned, peer-mapped on every rank, zeroed once before the first call);
 * tokens <= max_tokens; hidden a multiple of world.  Every rank makes the
 * same calls in the same order with no other kernel running on its GPU
 * meanwhile, and calls on one exchange never overlap.  A rank that does not
 * arrive makes the others' bounded waits (2 s) give up with bit 8 of
 * spiral_device_status; y is then invalid, later calls skip their waits until
 * the status is read, and the exchanges must be zeroed again on every rank.
 * Other arguments and the workspace as spiral_moe_ffn. */
SPIRAL_API int spiral_moe_ffn_ep(int fmt, const void* w_gate, const void* w_up, const void* w_down,
                                 int64_t n_experts_local, int64_t expert_first, int64_t hidden,
                                 int64_t inter, const void* x, int64_t x_row_stride_elems,
                                 int64_t tokens, int64_t max_tokens, const int32_t* expert_ids,
                                 const float* expert_weights, int64_t topk, void* y, int y_dtype,
                                 int64_t y_row_stride_elems, void* const* exchange_peers, int rank,
                                 int world, void* workspace, int64_t workspace_bytes, unsigned flags,
                                 void* stream);

/* The same MoE layer for callers that cannot allocate device memory when they
 * call in: a plain C host handed device pointers with no allocator of its own,
 * a serving loop that must not hit cudaMalloc mid-step (it may synchronize the
 * device), or code whose device memory belongs to a caching allocator or a
 * pre-planned arena.  No counterpart in the reference (it has no MoE and its
 * shims allocate nothing device-side).
 * Scratch is a static 8 MiB array inside the library, reserved on every GPU
 * that loads the library until the process exits; this call allocates
 * nothing.  Dims whose spiral_moe_workspace_bytes exceeds 8 MiB are rejected
 * with SPIRAL_ERR_CAPACITY (config-4 dims, 128 experts x hidden 2048 x inter
 * 768 at top-8, fit up to 107 tokens).  The first call on a device looks up
 * the array's device address; make that first call before any stream
 * capture.  The looked-up address is kept for the process: after
 * cudaDeviceReset (or any other reset of the device's primary context) do not
 * call this entry point again in the same process.  All calls share the
 * array: calls that overlap on the GPU race on it, so order them (one
 * stream, or events).  As with spiral_moe_ffn, y is valid only while
 * spiral_device_status reports no error bits: a pipeline wait that gave up
 * (bit 1) leaves parts of the layer, and so of y, uncomputed.  Arguments as
 * spiral_moe_ffn without the workspace. */
SPIRAL_API int spiral_moe_ffn_noalloc(int fmt, const void* w_gate, const void* w_up,
                                      const void* w_down, int64_t n_experts_local,
                                      int64_t expert_first, int64_t hidden, int64_t inter,
                                      const void* x, int64_t x_row_stride_elems, int64_t tokens,
                                      const int32_t* expert_ids, const float* expert_weights,
                                      int64_t topk, void* y, int y_dtype,
                                      int64_t y_row_stride_elems, unsigned flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPIRAL_B200_H */
