"""Python host bindings for libipuc.so, the B200 operator-catalog backend.

The C ABI (include/ipuc.h) is the product boundary; this module is a thin
ctypes layer over it so Python callers (tests, bench.py, the graph runtime in
ipuc.graph) can pass device pointers.  Every function raises IpucError with
the library's status and message when the C call fails — there is no fallback
path: if libipuc.so is missing, import fails loudly.

Device memory, streams and torch.distributed come from PyTorch; PyTorch is
plumbing here, the arithmetic is in the CUDA kernels behind the ABI.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libipuc.so")

# ipuc_status
OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_ALIGNMENT, ERR_CUDA, ERR_NCCL, ERR_DEVICE_TIMEOUT = range(7)
# ipuc_precision
F16, F32 = 0, 1
# ipuc_order
(ROW_MAJOR, AMP_LEFT, AMP_TRANSPOSED_LEFT, AMP_TRANSPOSED_RIGHT, AMP_OUTPUT, AMP_TRANSPOSED_OUTPUT,
 BLOCK_MAJOR, BLOCK_MAJOR_TRANSPOSED) = range(8)
# gemm flags
GEMM_ACCUMULATE, GEMM_B_TRANSPOSED, GEMM_OUT_F32, GEMM_EPILOGUE_GELU = 1, 2, 4, 8

# Every exported entry point with its argument types (kept in sync with
# include/ipuc.h; tests check the library exports each one).
_i64, _u64, _u32, _i32, _f32, _vp = (ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int32,
                                     ctypes.c_float, ctypes.c_void_p)
SIGNATURES = {
    "ipuc_version": (ctypes.c_char_p, []),
    "ipuc_status_string": (ctypes.c_char_p, [_i32]),
    "ipuc_last_error_string": (ctypes.c_char_p, []),
    "ipuc_device_status": (_i32, [_vp]),
    "ipuc_fill_zero": (_i32, [_vp, _u64, _vp]),
    "ipuc_selftest_bounded_wait": (_i32, [_u64, _vp]),
    "ipuc_gemm_f16": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _u32, _vp]),
    "ipuc_gemm_f16_batched": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                     _u32, _vp]),
    "ipuc_gemm_f32_workspace_bytes": (_u64, [_i64, _i64, _i64]),
    "ipuc_gemm_f32": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _u32, _vp, _u64, _vp]),
    "ipuc_gemm_f32_noalloc": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _u32, _vp]),
    "ipuc_gelu_f16": (_i32, [_vp, _vp, _u64, _vp]),
    "ipuc_reduce_sum": (_i32, [_vp, _vp, _vp, _u32, _u64, _i32, _vp]),
    "ipuc_add_f16": (_i32, [_vp, _vp, _vp, _u64, _u64, _u64, _vp]),
    "ipuc_cast": (_i32, [_vp, _i32, _vp, _i32, _u64, _vp]),
    "ipuc_flash_attention_f16": (_i32, [_vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _vp]),
    "ipuc_attention_softmax_f16": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_attention_merge_f16": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp]),
    "ipuc_rearrange_f16": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_unpack_f16": (_i32, [_vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_convert_order_f16": (_i32, [_vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_split_heads_f16": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_merge_heads_f16": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp]),
}


class IpucError(RuntimeError):
    def __init__(self, fn: str, status: int, message: str):
        self.status = status
        self.message = message
        super().__init__(f"{fn} failed: {STATUS_NAMES.get(status, status)}: {message}")


STATUS_NAMES = {OK: "IPUC_OK", ERR_INVALID_ARGUMENT: "IPUC_ERR_INVALID_ARGUMENT", ERR_UNSUPPORTED: "IPUC_ERR_UNSUPPORTED",
                ERR_ALIGNMENT: "IPUC_ERR_ALIGNMENT", ERR_CUDA: "IPUC_ERR_CUDA", ERR_NCCL: "IPUC_ERR_NCCL",
                ERR_DEVICE_TIMEOUT: "IPUC_ERR_DEVICE_TIMEOUT"}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libipuc.so (raises OSError if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"libipuc.so not built at {LIB_PATH}; run `make -C ipu-stack_b200`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _stream(stream) -> int | None:
    if stream is None:
        try:
            import torch
            if torch.cuda.is_available():
                return torch.cuda.current_stream().cuda_stream
        except Exception:  # pragma: no cover
            pass
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    return x.data_ptr()


def _check(fn: str, status: int):
    if status != OK:
        msg = lib().ipuc_last_error_string()
        raise IpucError(fn, status, msg.decode() if msg else "")


def call(name: str, *args):
    """Call an entry point by name with raw arguments; raises IpucError on failure."""
    st = getattr(lib(), name)(*args)
    _check(name, st)
    return st


def version() -> str:
    return lib().ipuc_version().decode()


def device_status(stream=None):
    _check("ipuc_device_status", lib().ipuc_device_status(_stream(stream)))


# ---- typed wrappers over torch tensors (device pointers) -------------------

def fill_zero(out, nbytes=None, stream=None):
    n = out.numel() * out.element_size() if nbytes is None else nbytes
    call("ipuc_fill_zero", _ptr(out), n, _stream(stream))


def gemm_f16(c, a, b, m, n, k, lda=None, ldb=None, ldc=None, flags=0, stream=None):
    bt = bool(flags & GEMM_B_TRANSPOSED)
    lda = k if lda is None else lda
    ldb = (k if bt else n) if ldb is None else ldb
    ldc = n if ldc is None else ldc
    call("ipuc_gemm_f16", _ptr(c), _ptr(a), _ptr(b), m, n, k, lda, ldb, ldc, flags, _stream(stream))


def gemm_f16_batched(c, a, b, batch, m, n, k, flags=0, stream=None):
    bt = bool(flags & GEMM_B_TRANSPOSED)
    ldb = k if bt else n
    call("ipuc_gemm_f16_batched", _ptr(c), _ptr(a), _ptr(b), batch, m, n, k, k, ldb, n, m * k, n * k, m * n, flags,
         _stream(stream))


def gemm_f32_workspace_bytes(m, n, k) -> int:
    return int(lib().ipuc_gemm_f32_workspace_bytes(m, n, k))


def gemm_f32(c, a, b, m, n, k, workspace, flags=0, lda=None, ldb=None, ldc=None, stream=None):
    bt = bool(flags & GEMM_B_TRANSPOSED)
    lda = k if lda is None else lda
    ldb = (k if bt else n) if ldb is None else ldb
    ldc = n if ldc is None else ldc
    ws = workspace.numel() * workspace.element_size() if workspace is not None else 0
    call("ipuc_gemm_f32", _ptr(c), _ptr(a), _ptr(b), m, n, k, lda, ldb, ldc, flags, _ptr(workspace), ws,
         _stream(stream))


def gelu_f16(out, inp, count=None, stream=None):
    call("ipuc_gelu_f16", _ptr(out), _ptr(inp), inp.numel() if count is None else count, _stream(stream))


def reduce_sum(out, initial, remote, num_partials, count, in_precision, stream=None):
    call("ipuc_reduce_sum", _ptr(out), _ptr(initial), _ptr(remote), num_partials, count, in_precision,
         _stream(stream))


def add_f16(out, left, right, count, left_period=0, right_period=0, stream=None):
    call("ipuc_add_f16", _ptr(out), _ptr(left), _ptr(right), count, left_period, right_period, _stream(stream))


def cast(out, to, inp, frm, count, stream=None):
    call("ipuc_cast", _ptr(out), to, _ptr(inp), frm, count, _stream(stream))


def flash_attention_f16(out, q, k, v, matrices, query_rows, key_rows, head_dim, out_precision=F16, scale=0.0,
                        stream=None):
    call("ipuc_flash_attention_f16", _ptr(out), out_precision, _ptr(q), _ptr(k), _ptr(v), matrices, query_rows,
         key_rows, head_dim, scale, _stream(stream))


def attention_softmax_f16(weights, scores, query_rows, key_rows, key_block_columns, head_dimension, stream=None):
    call("ipuc_attention_softmax_f16", _ptr(weights), _ptr(scores), query_rows, key_rows, key_block_columns,
         head_dimension, _stream(stream))


def attention_merge_f16(acc, block, state, query_rows, value_dimension, padded_value_dimension, initial, final,
                        stream=None):
    call("ipuc_attention_merge_f16", _ptr(acc), _ptr(block), _ptr(state), query_rows, value_dimension,
         padded_value_dimension, int(initial), int(final), _stream(stream))


def rearrange_f16(dst, src, matrices, logical_rows, physical_rows, target_order, logical_columns, physical_columns,
                  row_block=64, column_block=16, stream=None):
    call("ipuc_rearrange_f16", _ptr(dst), _ptr(src), matrices, logical_rows, physical_rows, target_order,
         logical_columns, physical_columns, row_block, column_block, _stream(stream))


def unpack_f16(dst, src, source_order, matrices, logical_rows, physical_rows, logical_columns, physical_columns,
               stream=None):
    call("ipuc_unpack_f16", _ptr(dst), _ptr(src), source_order, matrices, logical_rows, physical_rows,
         logical_columns, physical_columns, _stream(stream))


def convert_order_f16(dst, to, src, frm, matrices, rows, columns, row_block=64, column_block=16, stream=None):
    call("ipuc_convert_order_f16", _ptr(dst), to, _ptr(src), frm, matrices, rows, columns, row_block, column_block,
         _stream(stream))


def split_heads_f16(out, inp, batch, rows, heads, channels, stream=None):
    call("ipuc_split_heads_f16", _ptr(out), _ptr(inp), batch, rows, heads, channels, _stream(stream))


def merge_heads_f16(out, inp, batch, rows, heads, channels, stream=None):
    call("ipuc_merge_heads_f16", _ptr(out), _ptr(inp), batch, rows, heads, channels, _stream(stream))
