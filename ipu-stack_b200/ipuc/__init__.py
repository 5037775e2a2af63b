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
GEMM_F32_SPLIT_TF32 = 16  # ipuc_gemm_f32: the unscaled 3xTF32 split instead of the scaled f16 one
GEMM_A_TRANSPOSED = 32    # ipuc_gemm_f16: A stored [k x m] (GemmOptions::transpose_left)

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
    "ipuc_gemm_f16_addend": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _u32, _vp, _i64, _vp]),
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
    "ipuc_flash_attention_heads_f16": (_i32, [_vp, _i32, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _f32, _vp]),
    "ipuc_attention_softmax_f16": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_attention_merge_f16": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, _vp]),
    "ipuc_rearrange_f16": (_i32, [_vp, _vp, _i64, _i64, _i64, _i32, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_unpack_f16": (_i32, [_vp, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_convert_order_f16": (_i32, [_vp, _i32, _vp, _i32, _i64, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_split_heads_f16": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_merge_heads_f16": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp]),
    "ipuc_query_abi": (_i32, [_vp, _i32, _vp]),
    "ipuc_launch": (_i32, [_vp, _vp, _vp, _i32, _vp, _i32, _vp, _u64, _vp]),
    "ipuc_peer_signal_bytes": (_u64, []),
    "ipuc_ipc_handle": (_i32, [_vp, _vp, _u64, ctypes.POINTER(_u64)]),
    "ipuc_ipc_open": (_i32, [_vp, _u64, ctypes.POINTER(_vp)]),
    "ipuc_ipc_close": (_i32, [_vp]),
    "ipuc_peer_all_reduce_f16": (_i32, [_vp, _vp, _vp, _i32, _i32, _u64, _vp]),
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
    lda = (m if flags & GEMM_A_TRANSPOSED else k) if lda is None else lda
    ldb = (k if bt else n) if ldb is None else ldb
    ldc = n if ldc is None else ldc
    call("ipuc_gemm_f16", _ptr(c), _ptr(a), _ptr(b), m, n, k, lda, ldb, ldc, flags, _stream(stream))


def gemm_f16_addend(c, a, b, m, n, k, addend, ld_addend=None, lda=None, ldb=None, ldc=None, flags=0, stream=None):
    """C = epilogue(A.B + addend): the Gemm -> Add fusion with the addend read by the epilogue."""
    bt = bool(flags & GEMM_B_TRANSPOSED)
    lda = k if lda is None else lda
    ldb = (k if bt else n) if ldb is None else ldb
    ldc = n if ldc is None else ldc
    ld_addend = n if ld_addend is None else ld_addend
    call("ipuc_gemm_f16_addend", _ptr(c), _ptr(a), _ptr(b), m, n, k, lda, ldb, ldc, flags, _ptr(addend), ld_addend,
         _stream(stream))


def gemm_f16_batched(c, a, b, batch, m, n, k, flags=0, stream=None):
    bt = bool(flags & GEMM_B_TRANSPOSED)
    ldb = k if bt else n
    lda = m if flags & GEMM_A_TRANSPOSED else k
    call("ipuc_gemm_f16_batched", _ptr(c), _ptr(a), _ptr(b), batch, m, n, k, lda, ldb, n, m * k, n * k, m * n, flags,
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


def flash_attention_heads_f16(out, q, k, v, batch, heads, query_rows, key_rows, head_dim, out_precision=F16,
                              scale=0.0, stream=None):
    """Attention on [batch, rows, heads * head_dim] tensors (split/merge heads folded in)."""
    call("ipuc_flash_attention_heads_f16", _ptr(out), out_precision, _ptr(q), _ptr(k), _ptr(v), batch, heads,
         query_rows, key_rows, head_dim, scale, _stream(stream))


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


# ---- spec-driven dispatch (ipuc_query_abi / ipuc_launch) -------------------
# Mirrors TileKernelSpec (crates/ipu-codegen/src/operator.rs:57-96) and the
# KernelAbi that tile_kernel_abi derives from it (kernel.rs:1215-1382).

(KERNEL_FILL_ZERO, KERNEL_GEMM, KERNEL_GELU, KERNEL_REDUCTION_SUM, KERNEL_ADD, KERNEL_FLASH_ATTENTION,
 KERNEL_ATTENTION_SOFTMAX, KERNEL_ATTENTION_MERGE, KERNEL_CAST, KERNEL_REARRANGE) = range(10)
AVAILABILITY_IMPLEMENTED, AVAILABILITY_REQUIRED = 0, 1


class Layout(ctypes.Structure):
    _fields_ = [("order", ctypes.c_int32), ("row_block", ctypes.c_uint32), ("column_block", ctypes.c_uint32)]


class _Gemm(ctypes.Structure):
    _fields_ = [("multiply", ctypes.c_int32), ("accumulate", ctypes.c_int32), ("mode", ctypes.c_uint32),
                ("interleaved_weights", ctypes.c_uint32), ("inner_block", ctypes.c_uint32),
                ("output_columns", ctypes.c_uint32), ("b_transposed", ctypes.c_uint32),
                ("epilogue_gelu", ctypes.c_uint32)]


class _Reduction(ctypes.Structure):
    _fields_ = [("partials", ctypes.c_uint16)]


class _Attention(ctypes.Structure):
    _fields_ = [("causal", ctypes.c_uint32), ("scale", ctypes.c_float), ("accumulate", ctypes.c_int32)]


class _Softmax(ctypes.Structure):
    _fields_ = [("head_dimension", ctypes.c_uint32), ("key_columns", ctypes.c_uint32),
                ("padded_key_columns", ctypes.c_uint32)]


class _Merge(ctypes.Structure):
    _fields_ = [("value_dimension", ctypes.c_uint32), ("padded_value_dimension", ctypes.c_uint32),
                ("key_block_columns", ctypes.c_uint32), ("initial", ctypes.c_uint32), ("final_block", ctypes.c_uint32)]


class _Cast(ctypes.Structure):
    _fields_ = [("from_", ctypes.c_int32), ("to", ctypes.c_int32)]


class _Rearrange(ctypes.Structure):
    _fields_ = [("from_", Layout), ("to", Layout)]


class KernelSpec(ctypes.Structure):
    """ipuc_kernel_spec; build one with the TileKernelSpec-named helpers below."""
    _fields_ = [("kind", ctypes.c_int32), ("gemm", _Gemm), ("reduction_sum", _Reduction),
                ("flash_attention", _Attention), ("attention_softmax", _Softmax), ("attention_merge", _Merge),
                ("cast", _Cast), ("rearrange", _Rearrange)]


class Tensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("precision", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 4)]


class KernelAbi(ctypes.Structure):
    _fields_ = [("symbol", ctypes.c_char_p), ("reference_symbol", ctypes.c_char_p), ("availability", ctypes.c_int32),
                ("input_count", ctypes.c_int32), ("scalar_count", ctypes.c_int32),
                ("scalar_names", ctypes.c_char_p * 8)]


def _layout(order, row_block=0, column_block=0):
    if isinstance(order, Layout):
        return order
    return Layout(order, row_block, column_block)


class TileKernelSpec:
    """Constructors named after the reference enum's variants."""

    @staticmethod
    def fill_zero():
        return KernelSpec(kind=KERNEL_FILL_ZERO)

    @staticmethod
    def gemm(multiply=F16, accumulate=F32, mode="initialize", interleaved_weights=False, inner_block=64,
             output_columns=16, b_transposed=False, epilogue_gelu=False):
        s = KernelSpec(kind=KERNEL_GEMM)
        s.gemm = _Gemm(multiply, accumulate, 1 if mode == "accumulate" else 0, int(interleaved_weights),
                       inner_block, output_columns, int(b_transposed), int(epilogue_gelu))
        return s

    @staticmethod
    def gelu():
        return KernelSpec(kind=KERNEL_GELU)

    @staticmethod
    def reduction_sum(partials):
        s = KernelSpec(kind=KERNEL_REDUCTION_SUM)
        s.reduction_sum = _Reduction(partials)
        return s

    @staticmethod
    def add():
        return KernelSpec(kind=KERNEL_ADD)

    @staticmethod
    def flash_attention(causal=False, scale=0.0, accumulate=F32):
        s = KernelSpec(kind=KERNEL_FLASH_ATTENTION)
        s.flash_attention = _Attention(int(causal), scale, accumulate)
        return s

    @staticmethod
    def attention_softmax(head_dimension, key_columns, padded_key_columns):
        s = KernelSpec(kind=KERNEL_ATTENTION_SOFTMAX)
        s.attention_softmax = _Softmax(head_dimension, key_columns, padded_key_columns)
        return s

    @staticmethod
    def attention_merge(value_dimension, padded_value_dimension, key_block_columns, initial, final_block):
        s = KernelSpec(kind=KERNEL_ATTENTION_MERGE)
        s.attention_merge = _Merge(value_dimension, padded_value_dimension, key_block_columns, int(initial),
                                   int(final_block))
        return s

    @staticmethod
    def cast(frm, to):
        s = KernelSpec(kind=KERNEL_CAST)
        s.cast = _Cast(frm, to)
        return s

    @staticmethod
    def rearrange(frm, to):
        s = KernelSpec(kind=KERNEL_REARRANGE)
        s.rearrange = _Rearrange(_layout(*frm) if isinstance(frm, tuple) else _layout(frm),
                                 _layout(*to) if isinstance(to, tuple) else _layout(to))
        return s


def _precision_of(t):
    import torch
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.float32:
        return F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def tensor(t, shape=None, precision=None):
    """ipuc_tensor for a torch tensor (dense; `shape` overrides its shape)."""
    shape = tuple(t.shape) if shape is None else tuple(shape)
    if not 1 <= len(shape) <= 4:
        raise ValueError("rank 1..4")
    dims = (ctypes.c_int64 * 4)(*(list(shape) + [0] * (4 - len(shape))))
    out = Tensor(t.data_ptr(), _precision_of(t) if precision is None else precision, len(shape), dims)
    out._owner = t  # keep the device memory alive as long as the descriptor
    return out


def query_abi(spec, output_precision=F16):
    """tile_kernel_abi: dict(symbol, reference_symbol, availability, input_count, scalar_names)."""
    abi = KernelAbi()
    call("ipuc_query_abi", ctypes.byref(spec), output_precision, ctypes.byref(abi))
    return {
        "symbol": abi.symbol.decode(),
        "reference_symbol": abi.reference_symbol.decode(),
        "availability": abi.availability,
        "input_count": abi.input_count,
        "scalar_names": [abi.scalar_names[i].decode() for i in range(abi.scalar_count)],
    }


def launch(spec, out, inputs=(), scalars=(), workspace=None, stream=None):
    """validate_kernel_run + call: `out`/`inputs` are torch tensors or Tensor structs."""
    o = out if isinstance(out, Tensor) else tensor(out)
    ins = [x if isinstance(x, Tensor) else tensor(x) for x in inputs]
    arr = (Tensor * max(1, len(ins)))(*ins) if ins else None
    sc = (ctypes.c_uint32 * max(1, len(scalars)))(*scalars) if scalars else None
    ws = workspace.numel() * workspace.element_size() if workspace is not None else 0
    call("ipuc_launch", ctypes.byref(spec), ctypes.byref(o), arr, len(ins), sc, len(scalars), _ptr(workspace), ws,
         _stream(stream))


# ---- peer-memory all-reduce over NVLink (one process per GPU) -------------

class PeerAllReduce:
    """Sum of f16 tensors across the ranks of a torch.distributed group with
    this library's peer-memory kernel (ipuc_peer_all_reduce_f16).  `inputs`
    and `outputs` are lists of this rank's device tensors, the same shapes on
    every rank; the constructor is collective (CUDA IPC handles travel through
    torch.distributed.all_gather_object).  reduce(i) sums inputs[i] of all
    ranks into outputs[i] of every rank, stream-ordered."""

    def __init__(self, inputs, outputs, group=None):
        import torch
        import torch.distributed as dist
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.signal = torch.zeros(int(lib().ipuc_peer_signal_bytes()), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        self._keep = list(inputs) + list(outputs)
        mine = []
        for t in [self.signal] + list(inputs) + list(outputs):
            h = ctypes.create_string_buffer(64)
            off = _u64(0)
            call("ipuc_ipc_handle", _ptr(t), h, 64, ctypes.byref(off))
            mine.append((h.raw, off.value))
        every = [None] * self.world
        dist.all_gather_object(every, mine, group=group)
        self._opened = []
        table = []
        for q in range(self.world):
            row = []
            for e, (h, off) in enumerate(every[q]):
                if q == self.rank:
                    row.append(_ptr(([self.signal] + list(inputs) + list(outputs))[e]))
                    continue
                p = _vp()
                call("ipuc_ipc_open", h, off, ctypes.byref(p))
                self._opened.append(p.value)
                row.append(p.value)
            table.append(row)
        n = len(inputs)
        arr = _vp * self.world
        self._sig = arr(*[table[q][0] for q in range(self.world)])
        self._in = [arr(*[table[q][1 + i] for q in range(self.world)]) for i in range(n)]
        self._out = [arr(*[table[q][1 + n + i] for q in range(self.world)]) for i in range(n)]
        self._count = [t.numel() for t in inputs]
        dist.barrier(group=group)

    def reduce(self, i: int = 0, stream=None):
        call("ipuc_peer_all_reduce_f16", self._in[i], self._out[i], self._sig, self.rank, self.world,
             self._count[i], _stream(stream))

    def close(self):
        for p in self._opened:
            lib().ipuc_ipc_close(p)
        self._opened = []
