"""spiral_b200 — B200-native GGUF dequant / quantized MUL_MAT.

Python mirror of the C-ABI in include/spiral_b200.h (loaded with ctypes, the
way the reference's harness loads its host shim: src/quants/tests/common.py
:308-341).  The compute runs in libspiral_b200.so (hand-written sm_100a CUDA);
there is no Python or CPU fallback: if the library is missing, every entry
point raises.

Tensors may be torch CUDA tensors or raw device pointers (ints).  Shapes use
ggml's convention: a quantized weight has N rows (output features) of K
weights; activations are [M][K]; outputs [M][N].
"""

from __future__ import annotations

import ctypes
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libspiral_b200.so"

Q4_0, Q8_0, Q6_K = 2, 8, 14
# extended formats (spiral_dequant_bf16 / spiral_mul_mat / the ggml boundary)
F16, Q4_K, Q5_K, IQ4_NL, IQ4_XS = 1, 12, 13, 20, 23
F32, BF16 = 0, 30
FLAG_FTZ_SCALES = 0x1
FLAG_ACCUMULATE = 0x2
FLAG_STATIC_WEIGHTS = 0x4
FORMATS = {"q4_0": Q4_0, "q8_0": Q8_0, "q6_k": Q6_K, "q4_k": Q4_K, "q5_k": Q5_K, "iq4_nl": IQ4_NL,
           "iq4_xs": IQ4_XS, "f16": F16, "bf16": BF16}
BLOCK_K = {Q4_0: 32, Q8_0: 32, Q6_K: 256, Q4_K: 256, Q5_K: 256, IQ4_NL: 32, IQ4_XS: 256, F16: 1, BF16: 1}
BLOCK_BYTES = {Q4_0: 18, Q8_0: 34, Q6_K: 210, Q4_K: 144, Q5_K: 176, IQ4_NL: 18, IQ4_XS: 136, F16: 2, BF16: 2}

# Every symbol include/spiral_b200.h declares, with (argtypes, restype).
_i64, _i32, _vp, _u32 = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint
_SIGNATURES = {
    "spiral_version": ([], _i32),
    "spiral_status_string": ([_i32], ctypes.c_char_p),
    "spiral_last_error": ([], ctypes.c_char_p),
    "spiral_device_status": ([_vp, ctypes.POINTER(ctypes.c_uint32)], _i32),
    "spiral_quants_block_rows": ([_i32], _i64),
    "spiral_quants_block_bytes": ([_i32], _i64),
    "spiral_quants_record_count": ([_i32, _i64, _i64], _i64),
    "spiral_quants_packed_bytes": ([_i32, _i64, _i64], _i64),
    "spiral_quants_repack": ([_i32, _vp, _i64, _vp, _i64, _i64, _i64, _vp], _i64),
    "spiral_set_repack_warn": ([_vp, _vp], None),
    "spiral_dequant_bf16": ([_i32, _vp, _i64, _vp, _i64, _i64, _i64, _u32, _vp], _i32),
    "spiral_quants_unpack_all": ([_i32, _vp, _vp, _i64, _i64, _u32, _vp], _i32),
    "spiral_mul_mat": ([_i32, _vp, _i64, _vp, _i64, _vp, _i32, _i64, _i64, _i64, _i64, _u32, _vp], _i32),
    "spiral_ggml_supports_mul_mat": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p], _i32),
    "spiral_ggml_mul_mat": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _u32, _vp], _i32),
    "spiral_quants_unpack_mmul_all": ([_i32, _vp, _vp, _vp, _i64, _i64, _i64, _u32, _vp], _i32),
    "spiral_allgather_exchange_bytes": ([_i64], _i64),
    "spiral_allgather_exchange_reset": ([_vp, _i64, _vp], _i32),
    "spiral_mul_mat_allgather": ([_i32, _vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i32,
                                  _i32, _u32, _vp], _i32),
    "spiral_moe_workspace_bytes": ([_i64, _i64, _i64, _i64, _i64], _i64),
    "spiral_moe_ffn": ([_i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _i32,
                        _i64, _vp, _i64, _u32, _vp], _i32),
    "spiral_moe_ep_exchange_bytes": ([_i64, _i64], _i64),
    "spiral_moe_ep_exchange_reset": ([_vp, _i64, _i64, _vp], _i32),
    "spiral_moe_ffn_ep": ([_i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _i64, _vp,
                           _i32, _i64, _vp, _i32, _i32, _vp, _i64, _u32, _vp], _i32),
    "spiral_moe_ffn_noalloc": ([_i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _vp,
                                _i32, _i64, _u32, _vp], _i32),
}



class GgmlTensor(ctypes.Structure):
    """spiral_ggml_tensor: ggml type id, ne[4], nb[4] (bytes), device data."""

    _fields_ = [("type", ctypes.c_int32), ("ne", ctypes.c_int64 * 4), ("nb", ctypes.c_size_t * 4),
                ("data", ctypes.c_void_p)]


_lib = None


class SpiralError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"spiral status {status}: {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    """The loaded C-ABI library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m spiral_b200.build` "
                "(this package has no CPU fallback)"
            )
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (args, res) in _SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def fmt_id(fmt) -> int:
    return FORMATS[fmt] if isinstance(fmt, str) else int(fmt)


def _check(status: int) -> None:
    if status != 0:
        msg = lib().spiral_last_error().decode() or lib().spiral_status_string(status).decode()
        raise SpiralError(status, msg)


def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    return int(t.data_ptr())


def _stream(stream) -> int:
    if stream is None:
        try:
            import torch

            if torch.cuda.is_available():
                return int(torch.cuda.current_stream().cuda_stream)
        except Exception:
            pass
        return 0
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


# ------------------------------------------------------------ size queries


def record_count(fmt, weights_rows: int, weights_cols: int) -> int:
    return lib().spiral_quants_record_count(fmt_id(fmt), weights_rows, weights_cols)


def packed_bytes(fmt, weights_rows: int, weights_cols: int) -> int:
    return lib().spiral_quants_packed_bytes(fmt_id(fmt), weights_rows, weights_cols)


def row_bytes(fmt, K: int) -> int:
    f = fmt_id(fmt)
    return (K // BLOCK_K[f]) * BLOCK_BYTES[f]


def repack(fmt, src, src_col_stride_bytes: int, dst, dst_capacity: int, weights_rows: int, weights_cols: int,
           stream=None) -> int:
    """Bytes written, 0 on invalid input (reference repack contract)."""
    return lib().spiral_quants_repack(fmt_id(fmt), _ptr(src), src_col_stride_bytes, _ptr(dst), dst_capacity,
                                      weights_rows, weights_cols, _stream(stream))


# C signature of the repack warning hook: void (*)(const char* line, void* user)
REPACK_WARN_FN = ctypes.CFUNCTYPE(None, ctypes.c_char_p, ctypes.c_void_p)
_warn_keep = None  # the installed ctypes callback must outlive its use


def set_repack_warn(fn=None, *, to_stderr: bool = False) -> None:
    """Route the repack's one-line warnings: fn(line: str) receives each
    line; fn=None suppresses them; to_stderr=True writes them to sys.stderr
    (the library's own default, before any call here, is the C stderr)."""
    global _warn_keep
    if to_stderr:
        import sys

        fn = sys.stderr.write
    cb = None if fn is None else REPACK_WARN_FN(lambda line, user: fn(line.decode()))
    _warn_keep = cb
    lib().spiral_set_repack_warn(ctypes.cast(cb, ctypes.c_void_p) if cb is not None else None, None)


def device_status(stream=None) -> int:
    code = ctypes.c_uint32(0)
    st = lib().spiral_device_status(_stream(stream), ctypes.byref(code))
    if st not in (0, -8):
        _check(st)
    return code.value


# ------------------------------------------------------------------ ops


def dequant_bf16(fmt, w, K: int, N: int, out=None, *, w_row_stride: int | None = None,
                 out_row_stride: int | None = None, ftz: bool = False, stream=None):
    """ggml-style dequantize: out[n][k] = bf16(W[n][k])."""
    f = fmt_id(fmt)
    if out is None:
        import torch

        out = torch.empty((N, K), dtype=torch.bfloat16, device=w.device)
    _check(lib().spiral_dequant_bf16(f, _ptr(w), w_row_stride or row_bytes(f, K), _ptr(out), out_row_stride or K,
                                     K, N, FLAG_FTZ_SCALES if ftz else 0, _stream(stream)))
    return out


def unpack_all(fmt, packed, weights_rows: int, weights_cols: int, out=None, *, ftz: bool = False, stream=None):
    """Reference-order dequant: out = [weights_cols/8][weights_rows][8] bf16."""
    f = fmt_id(fmt)
    if out is None:
        import torch

        out = torch.empty((weights_rows * weights_cols,), dtype=torch.bfloat16, device=packed.device)
    _check(lib().spiral_quants_unpack_all(f, _ptr(packed), _ptr(out), weights_rows, weights_cols,
                                          FLAG_FTZ_SCALES if ftz else 0, _stream(stream)))
    return out


def mul_mat(fmt, w, x, N: int, K: int, y=None, *, y_dtype: int = BF16, w_row_stride: int | None = None,
            x_row_stride: int | None = None, y_row_stride: int | None = None, accumulate: bool = False,
            ftz: bool = False, stream=None, M: int | None = None, static_weights: bool = False):
    """ggml MUL_MAT: y[m][n] = sum_k bf16(W[n][k]) * x[m][k] (fp32 accumulate).

    static_weights: the weights are not written by the kernel queued just
    before on the stream, so the decode GEMV may start streaming them early."""
    f = fmt_id(fmt)
    if M is None:
        M = int(x.shape[0])
    if y is None:
        import torch

        y = torch.empty((M, N), dtype=torch.bfloat16 if y_dtype == BF16 else torch.float32, device=x.device)
    flags = ((FLAG_FTZ_SCALES if ftz else 0) | (FLAG_ACCUMULATE if accumulate else 0)
             | (FLAG_STATIC_WEIGHTS if static_weights else 0))
    _check(lib().spiral_mul_mat(f, _ptr(w), w_row_stride or row_bytes(f, K), _ptr(x), x_row_stride or K, _ptr(y),
                                y_dtype, y_row_stride or N, M, N, K, flags, _stream(stream)))
    return y


def unpack_mmul_all(fmt, packed, inputs_tiled, outputs, weights_rows: int, weights_cols: int, inputs_vecs: int, *,
                    ftz: bool = False, stream=None):
    """Reference fused op: outputs[N/8][M][8] (f32) += unpack(W) x inputs[K/8][M][8]."""
    _check(lib().spiral_quants_unpack_mmul_all(fmt_id(fmt), _ptr(packed), _ptr(inputs_tiled), _ptr(outputs),
                                               weights_rows, weights_cols, inputs_vecs,
                                               FLAG_FTZ_SCALES if ftz else 0, _stream(stream)))
    return outputs


def allgather_exchange_bytes(n_total: int) -> int:
    """Bytes of one rank's exchange buffer for mul_mat_allgather (0 if
    n_total is not a positive multiple of 8)."""
    return int(lib().spiral_allgather_exchange_bytes(n_total))


def allgather_exchange_reset(exchange, n_total: int, *, stream=None) -> None:
    """Zero this rank's exchange buffer (a device tensor) on the stream:
    the recovery after a gathered wait timed out.  Every rank resets its own,
    then the ranks meet at a barrier before the next gathered call."""
    _check(lib().spiral_allgather_exchange_reset(_ptr(exchange), n_total, _stream(stream)))


def mul_mat_allgather(fmt, w_shard, x, N_shard: int, K: int, y, n_offset: int, exchange_peers_dev, rank: int,
                      world: int, *, w_row_stride: int | None = None, ftz: bool = False, static_weights: bool = True,
                      stream=None):
    """Row-sharded MUL_MAT with the all-gather fused in: y (bf16
    [M][N_total], this rank's) receives every rank's shard; see
    spiral_b200.dist.AllGatherExchange for the exchange buffers."""
    import torch

    f = fmt_id(fmt)
    M, n_total = int(x.shape[0]), int(y.shape[1])
    if y.dtype != torch.bfloat16 or y.shape[0] < M:
        raise ValueError("y must be bf16 with at least M rows")
    flags = (FLAG_FTZ_SCALES if ftz else 0) | (FLAG_STATIC_WEIGHTS if static_weights else 0)
    _check(lib().spiral_mul_mat_allgather(f, _ptr(w_shard), w_row_stride or row_bytes(f, K), _ptr(x),
                                          int(x.stride(0)), _ptr(y), int(y.stride(0)), n_offset, M, N_shard,
                                          n_total, K, _ptr(exchange_peers_dev), rank, world, flags,
                                          _stream(stream)))


# ---------------------------------------------------------------- MoE FFN


def moe_workspace_bytes(n_experts_local: int, hidden: int, inter: int, tokens: int, topk: int) -> int:
    return lib().spiral_moe_workspace_bytes(n_experts_local, hidden, inter, tokens, topk)


def moe_ffn(fmt, w_gate, w_up, w_down, x, expert_ids, expert_weights, *, hidden: int, inter: int,
            n_experts_local: int, expert_first: int = 0, y=None, y_dtype: int = BF16, workspace=None,
            accumulate: bool = False, ftz: bool = False, stream=None):
    """MoE FFN decode layer (SwiGLU experts, quantized gate/up/down):
    y[t] (+)= sum_j w[t][j] * down_e(bf16(silu(gate_e x_t) * up_e x_t)) over the
    slots j whose expert e = ids[t][j] lies in [expert_first,
    expert_first + n_experts_local).  x: [T][hidden] bf16; ids int32 and
    weights f32: [T][topk]."""
    import torch

    f = fmt_id(fmt)
    T, topk = int(expert_ids.shape[0]), int(expert_ids.shape[1])
    if y is None:
        y = torch.empty((T, hidden), dtype=torch.bfloat16 if y_dtype == BF16 else torch.float32, device=x.device)
    need = moe_workspace_bytes(n_experts_local, hidden, inter, T, topk)
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    flags = (FLAG_FTZ_SCALES if ftz else 0) | (FLAG_ACCUMULATE if accumulate else 0)
    _check(lib().spiral_moe_ffn(f, _ptr(w_gate), _ptr(w_up), _ptr(w_down), n_experts_local, expert_first, hidden,
                                inter, _ptr(x), int(x.stride(0)), T, _ptr(expert_ids), _ptr(expert_weights), topk,
                                _ptr(y), y_dtype, int(y.stride(0)), _ptr(workspace), int(workspace.numel()),
                                flags, _stream(stream)))
    return y


def moe_ep_exchange_bytes(hidden: int, max_tokens: int) -> int:
    return int(lib().spiral_moe_ep_exchange_bytes(hidden, max_tokens))


def moe_ep_exchange_reset(exchange, hidden: int, max_tokens: int, *, stream=None) -> None:
    """Zero this rank's moe_ffn_ep exchange buffer on the stream (the
    recovery after a timed-out wait; every rank resets, then a barrier)."""
    _check(lib().spiral_moe_ep_exchange_reset(_ptr(exchange), hidden, max_tokens, _stream(stream)))


def moe_ffn_ep(fmt, w_gate, w_up, w_down, x, expert_ids, expert_weights, *, hidden: int, inter: int,
               n_experts_local: int, expert_first: int, exchange_peers_dev, rank: int, world: int, max_tokens: int,
               y=None, y_dtype: int = BF16, workspace=None, accumulate: bool = False, ftz: bool = False,
               stream=None):
    """Expert-parallel MoE layer (one process per GPU): every rank passes the
    same x [T][hidden] / ids / weights and its expert range; y receives the
    whole layer (all ranks' experts), identical on every rank.  See
    spiral_b200.dist.MoeExchange for the exchange buffers."""
    import torch

    f = fmt_id(fmt)
    T, topk = int(expert_ids.shape[0]), int(expert_ids.shape[1])
    if y is None:
        y = torch.empty((T, hidden), dtype=torch.bfloat16 if y_dtype == BF16 else torch.float32, device=x.device)
    need = moe_workspace_bytes(n_experts_local, hidden, inter, T, topk)
    if workspace is None:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=x.device)
    flags = (FLAG_FTZ_SCALES if ftz else 0) | (FLAG_ACCUMULATE if accumulate else 0)
    _check(lib().spiral_moe_ffn_ep(f, _ptr(w_gate), _ptr(w_up), _ptr(w_down), n_experts_local, expert_first, hidden,
                                   inter, _ptr(x), int(x.stride(0)), T, max_tokens, _ptr(expert_ids),
                                   _ptr(expert_weights), topk, _ptr(y), y_dtype, int(y.stride(0)),
                                   _ptr(exchange_peers_dev), rank, world, _ptr(workspace), int(workspace.numel()),
                                   flags, _stream(stream)))
    return y


# ------------------------------------------------------------ ggml boundary


def ggml_tensor(type_id: int, ne, nb, data) -> GgmlTensor:
    """A spiral_ggml_tensor from ggml-style ne/nb (innermost first) and a
    device pointer (int or tensor)."""
    t = GgmlTensor()
    t.type = int(type_id)
    ne = list(ne) + [1] * (4 - len(ne))
    nb = list(nb) + [0] * (4 - len(nb))
    for i in range(4):
        t.ne[i] = int(ne[i])
        t.nb[i] = int(nb[i])
    t.data = _ptr(data)
    return t


def ggml_supports_mul_mat(src0: GgmlTensor, src1: GgmlTensor, dst: GgmlTensor) -> bool:
    return bool(lib().spiral_ggml_supports_mul_mat(ctypes.byref(src0), ctypes.byref(src1), ctypes.byref(dst)))


def ggml_mul_mat(src0: GgmlTensor, src1: GgmlTensor, dst: GgmlTensor, *, ftz: bool = False,
                 accumulate: bool = False, stream=None) -> None:
    flags = (FLAG_FTZ_SCALES if ftz else 0) | (FLAG_ACCUMULATE if accumulate else 0)
    _check(lib().spiral_ggml_mul_mat(ctypes.byref(src0), ctypes.byref(src1), ctypes.byref(dst), flags,
                                     _stream(stream)))
