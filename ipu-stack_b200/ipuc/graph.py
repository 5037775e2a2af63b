"""ComputeGraph and Session: Python face of include/ipug.h.

Method names follow the reference's graph API
(crates/ipu-codegen/src/graph.rs:209-515): host_input, parameter, gemm,
gemm_with_options, gelu, add, split_heads, flash_attention,
flash_attention_with_options, set_outputs.  Building and lowering happen in
libipuc.so (C++); this module records the operations it adds (so a checker can
re-evaluate the same graph) and wraps the session calls.  Invalid graphs raise
GraphError, the counterpart of graph.rs's GraphResult errors.
"""

from __future__ import annotations

import ctypes
import json
from dataclasses import dataclass, field

import numpy as np

from . import IpucError, OK, lib as _lib, _stream

_u32p = ctypes.POINTER(ctypes.c_uint32)
_i32p = ctypes.POINTER(ctypes.c_int32)
_vp = ctypes.c_void_p

_G_SIGS = {
    "ipug_graph_create": (_vp, []),
    "ipug_graph_destroy": (None, [_vp]),
    "ipug_host_input": (ctypes.c_int32, [_vp, ctypes.c_char_p, _u32p, ctypes.c_int32]),
    "ipug_parameter": (ctypes.c_int32, [_vp, ctypes.c_char_p, _u32p, ctypes.c_int32]),
    "ipug_gemm": (ctypes.c_int32, [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32]),
    "ipug_gelu": (ctypes.c_int32, [_vp, ctypes.c_int32]),
    "ipug_add": (ctypes.c_int32, [_vp, ctypes.c_int32, ctypes.c_int32]),
    "ipug_split_heads": (ctypes.c_int32, [_vp, ctypes.c_int32, ctypes.c_uint32]),
    "ipug_merge_heads": (ctypes.c_int32, [_vp, ctypes.c_int32, ctypes.c_uint32]),
    "ipug_flash_attention": (ctypes.c_int32, [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                              ctypes.c_float]),
    "ipug_set_outputs": (ctypes.c_int32, [_vp, _i32p, ctypes.c_int32]),
    "ipug_value_shape": (ctypes.c_int32, [_vp, ctypes.c_int32, _u32p]),
    "ipug_session_open": (_vp, [_vp, ctypes.c_int32, _i32p]),
    "ipug_session_close": (None, [_vp]),
    "ipug_session_write": (ctypes.c_int32, [_vp, ctypes.c_int32, _vp, ctypes.c_uint64, _vp]),
    "ipug_session_read": (ctypes.c_int32, [_vp, ctypes.c_int32, _vp, ctypes.c_uint64, _vp]),
    "ipug_session_device_ptr": (_vp, [_vp, ctypes.c_int32]),
    "ipug_session_run": (ctypes.c_int32, [_vp, _vp]),
    "ipug_session_peer_reduce": (ctypes.c_int32, [_vp, ctypes.c_int32, _vp]),
    "ipug_session_profile": (ctypes.c_int32, [_vp, _vp, ctypes.c_char_p, ctypes.c_uint64,
                                              ctypes.POINTER(ctypes.c_uint64)]),
    "ipug_session_profile_capnp": (ctypes.c_int32, [_vp, _vp, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64,
                                                    ctypes.POINTER(ctypes.c_uint64)]),
    "ipug_session_plan": (ctypes.c_char_p, [_vp]),
    "ipug_graph_plan": (ctypes.c_int32, [_vp, ctypes.c_char_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    "ipug_value_sequence": (ctypes.c_int32, [_vp, ctypes.c_char_p, _i32p, ctypes.c_int32]),
    "ipug_repeat_begin": (ctypes.c_int32, [_vp, ctypes.c_uint32, _i32p, ctypes.c_int32, _i32p, ctypes.c_int32, _i32p,
                                           ctypes.c_int32, _i32p]),
    "ipug_repeat_end": (ctypes.c_int32, [_vp, _i32p, ctypes.c_int32, _i32p]),
    "ipug_session_open_ex": (_vp, [_vp, _vp, _i32p]),
    "ipug_nccl_unique_id": (ctypes.c_int32, [_vp, ctypes.c_uint64]),
    "ipug_graph_plan_ex": (ctypes.c_int32, [_vp, _vp, ctypes.c_char_p, ctypes.c_uint64,
                                            ctypes.POINTER(ctypes.c_uint64)]),
    "ipug_graph_shard_json": (ctypes.c_int32, [_vp, ctypes.c_int32, ctypes.c_int32, ctypes.c_char_p, ctypes.c_uint64,
                                               ctypes.POINTER(ctypes.c_uint64)]),
    "ipug_session_diagnose": (ctypes.c_int32, [_vp, _i32p, _vp, ctypes.c_int32, _vp, _vp]),
}


class SessionOptions(ctypes.Structure):
    """ipug_session_options."""
    _fields_ = [("device", ctypes.c_int32), ("rank", ctypes.c_int32), ("world", ctypes.c_int32),
                ("nccl_id", ctypes.c_void_p), ("fuse", ctypes.c_int32)]


class ValueReport(ctypes.Structure):
    """ipug_value_report."""
    _fields_ = [("value", ctypes.c_int32), ("producer", ctypes.c_int32), ("available", ctypes.c_int32),
                ("elements", ctypes.c_uint64), ("nonfinite", ctypes.c_uint64), ("max_abs_err", ctypes.c_double),
                ("max_abs_ref", ctypes.c_double), ("rel_l2", ctypes.c_double)]


def _arr(values):
    values = [int(v) for v in values]
    return (ctypes.c_int32 * max(1, len(values)))(*values), len(values)


def nccl_unique_id() -> bytes:
    """A new 128-byte NCCL unique id (one rank makes it, every rank opens its
    sharded Session with it)."""
    buf = ctypes.create_string_buffer(128)
    st = glib().ipug_nccl_unique_id(buf, 128)
    if st != OK:
        raise IpucError("ipug_nccl_unique_id", st, _lib().ipuc_last_error_string().decode())
    return buf.raw


def _options(device=0, rank=0, world=1, nccl_id=None, fuse=True):
    o = SessionOptions(device, rank, world, None, 1 if fuse else 0)
    keep = None
    if nccl_id is not None:
        keep = ctypes.create_string_buffer(bytes(nccl_id), 128)
        o.nccl_id = ctypes.cast(keep, ctypes.c_void_p)
    return o, keep


@dataclass
class RepeatArguments:
    """The body's arguments (graph.rs:197-202): carried, invariants, iterated."""
    carried: list
    invariants: list
    iterated: list
_bound = False


def glib():
    global _bound
    L = _lib()
    if not _bound:
        for name, (res, args) in _G_SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _bound = True
    return L


class GraphError(ValueError):
    pass


@dataclass
class OpRecord:
    kind: str
    inputs: list
    result: int
    options: dict = field(default_factory=dict)


@dataclass
class InputRecord:
    name: str
    value: int
    shape: tuple
    kind: str  # "host" or "parameter"


class ComputeGraph:
    def __init__(self):
        self._g = glib().ipug_graph_create()
        self.inputs: list[InputRecord] = []
        self.operations: list[OpRecord] = []
        self.outputs: list[int] = []
        self.sequences: list[list] = []   # value ids per value sequence
        self._ops = self.operations       # where new operations are recorded (a Repeat body while one is open)

    def __del__(self):
        if getattr(self, "_g", None):
            glib().ipug_graph_destroy(self._g)
            self._g = None

    def _check(self, v: int) -> int:
        if v < 0:
            raise GraphError(_lib().ipuc_last_error_string().decode())
        return v

    def _input(self, fn, name, shape, kind):
        dims = (ctypes.c_uint32 * len(shape))(*shape)
        v = self._check(fn(self._g, name.encode(), dims, len(shape)))
        self.inputs.append(InputRecord(name, v, tuple(shape), kind))
        return v

    def host_input(self, name: str, shape) -> int:
        return self._input(glib().ipug_host_input, name, shape, "host")

    def parameter(self, name: str, shape) -> int:
        return self._input(glib().ipug_parameter, name, shape, "parameter")

    def gemm(self, left: int, right: int) -> int:
        return self.gemm_with_options(left, right)

    def gemm_with_options(self, left: int, right: int, transpose_left=False, transpose_right=False) -> int:
        v = self._check(glib().ipug_gemm(self._g, left, right, int(transpose_left), int(transpose_right)))
        self._ops.append(OpRecord("gemm", [left, right], v, dict(transpose_left=transpose_left,
                                                                       transpose_right=transpose_right)))
        return v

    def gelu(self, x: int) -> int:
        v = self._check(glib().ipug_gelu(self._g, x))
        self._ops.append(OpRecord("gelu", [x], v))
        return v

    def add(self, left: int, right: int) -> int:
        v = self._check(glib().ipug_add(self._g, left, right))
        self._ops.append(OpRecord("add", [left, right], v))
        return v

    def split_heads(self, x: int, heads: int) -> int:
        v = self._check(glib().ipug_split_heads(self._g, x, heads))
        self._ops.append(OpRecord("split_heads", [x], v, dict(heads=heads)))
        return v

    def merge_heads(self, x: int, heads: int) -> int:
        """Inverse of split_heads (an extension of the reference's graph API)."""
        v = self._check(glib().ipug_merge_heads(self._g, x, heads))
        self._ops.append(OpRecord("merge_heads", [x], v, dict(heads=heads)))
        return v

    def flash_attention(self, q: int, k: int, v: int) -> int:
        return self.flash_attention_with_options(q, k, v)

    def flash_attention_with_options(self, q: int, k: int, v: int, causal=False, scale=None) -> int:
        r = self._check(glib().ipug_flash_attention(self._g, q, k, v, int(causal), 0.0 if scale is None else scale))
        self._ops.append(OpRecord("flash_attention", [q, k, v], r, dict(causal=causal, scale=scale)))
        return r

    def value_sequence(self, name: str, values) -> int:
        """graph.rs:294-313: a named list of same-shaped values, iterated by Repeat."""
        arr, n = _arr(values)
        sid = self._check(glib().ipug_value_sequence(self._g, name.encode(), arr, n))
        self.sequences.append([int(v) for v in values])
        return sid

    def repeat(self, count: int, carried, invariants, iterated, build) -> list:
        """graph.rs:382-473: run `build(body, args)` once to record the body;
        it returns one yield per carried value.  `body` is this graph (its
        builder methods add to the body while it is open) and `args` the
        RepeatArguments.  Returns the Repeat's results (one per carried value)."""
        carried, invariants, iterated = list(carried), list(invariants), list(iterated)
        ca, nc = _arr(carried)
        ia, ni = _arr(invariants)
        sa, ns = _arr(iterated)
        args = (ctypes.c_int32 * max(1, nc + ni + ns))()
        st = glib().ipug_repeat_begin(self._g, count, ca, nc, ia, ni, sa, ns, args)
        if st != OK:
            raise GraphError(_lib().ipuc_last_error_string().decode())
        arguments = [args[i] for i in range(nc + ni + ns)]
        ra = RepeatArguments(arguments[:nc], arguments[nc:nc + ni], arguments[nc + ni:])
        body: list[OpRecord] = []
        outer = self._ops
        self._ops = body
        try:
            yields = list(build(self, ra))
        except BaseException:
            self._ops = outer
            glib().ipug_repeat_end(self._g, None, -1, None)  # discard the open body
            raise
        self._ops = outer
        ya, ny = _arr(yields)
        res = (ctypes.c_int32 * max(1, nc))()
        n = glib().ipug_repeat_end(self._g, ya, ny, res)
        if n < 0:
            raise GraphError(_lib().ipuc_last_error_string().decode())
        results = [res[i] for i in range(n)]
        self._ops.append(OpRecord("repeat", carried + invariants, results[0] if results else -1,
                                  dict(count=count, carried=nc, invariants=ni,
                                       sequences=[self.sequences[q] for q in iterated], arguments=arguments,
                                       body=body, yields=yields, results=results)))
        return results

    def set_outputs(self, outputs) -> None:
        outs = list(outputs)
        arr = (ctypes.c_int32 * len(outs))(*outs)
        st = glib().ipug_set_outputs(self._g, arr, len(outs))
        if st != OK:
            raise GraphError(_lib().ipuc_last_error_string().decode())
        self.outputs = outs

    def plan(self, rank: int = 0, world: int = 1, fuse: bool = True) -> str:
        """The per-GPU lowering (one line per step), computed on the host
        without a device: the plan a Session of this graph (rank `rank` of a
        sharded session over `world` GPUs) would run."""
        o, _ = _options(0, rank, world, None, fuse)
        need = ctypes.c_uint64(0)
        glib().ipug_graph_plan_ex(self._g, ctypes.byref(o), None, 0, ctypes.byref(need))
        if need.value == 0:
            raise GraphError(_lib().ipuc_last_error_string().decode())
        buf = ctypes.create_string_buffer(need.value)
        st = glib().ipug_graph_plan_ex(self._g, ctypes.byref(o), buf, need.value, ctypes.byref(need))
        if st != OK:
            raise IpucError("ipug_graph_plan", st, _lib().ipuc_last_error_string().decode())
        return buf.value.decode()

    def shard(self, rank: int, world: int) -> dict:
        """Rank `rank`'s shard of the graph over `world` GPUs (ipug_graph_shard_json)."""
        need = ctypes.c_uint64(0)
        glib().ipug_graph_shard_json(self._g, rank, world, None, 0, ctypes.byref(need))
        if need.value == 0:
            raise GraphError(_lib().ipuc_last_error_string().decode())
        buf = ctypes.create_string_buffer(need.value)
        st = glib().ipug_graph_shard_json(self._g, rank, world, buf, need.value, ctypes.byref(need))
        if st != OK:
            raise IpucError("ipug_graph_shard_json", st, _lib().ipuc_last_error_string().decode())
        return json.loads(buf.value.decode())

    def value_shape(self, v: int) -> tuple:
        dims = (ctypes.c_uint32 * 8)()
        r = glib().ipug_value_shape(self._g, v, dims)
        if r < 0:
            raise GraphError(f"unknown value {v}")
        return tuple(dims[:r])


class _DeviceBuffer:
    """__cuda_array_interface__ view of a session buffer (f16, row-major)."""

    def __init__(self, ptr: int, shape: tuple):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<f2", "data": (ptr, False), "version": 2,
                                         "strides": None}


class Session:
    """Lowered graph on one GPU (ipu-runtime's open/load/run/read back), or one
    rank of a session sharded over `world` GPUs (every rank opens the same
    graph with the same `nccl_id`)."""

    def __init__(self, graph: ComputeGraph, device: int = 0, rank: int = 0, world: int = 1, nccl_id=None,
                 fuse: bool = True):
        self.graph = graph
        self.rank, self.world = rank, world
        o, keep = _options(device, rank, world, nccl_id, fuse)
        st = ctypes.c_int32(0)
        self._s = glib().ipug_session_open_ex(graph._g, ctypes.byref(o), ctypes.byref(st))
        del keep
        if not self._s:
            raise IpucError("ipug_session_open", st.value, _lib().ipuc_last_error_string().decode())

    def close(self):
        if getattr(self, "_s", None):
            glib().ipug_session_close(self._s)
            self._s = None

    __del__ = close

    def _call(self, name, *args):
        st = getattr(glib(), name)(*args)
        if st != OK:
            raise IpucError(name, st, _lib().ipuc_last_error_string().decode())

    def write(self, value: int, data: np.ndarray, stream=None):
        a = np.ascontiguousarray(np.asarray(data).astype(np.float16))
        self._call("ipug_session_write", self._s, value, a.ctypes.data, a.nbytes, _stream(stream))
        import torch
        torch.cuda.synchronize()

    def write_device(self, value: int, tensor, stream=None):
        """Copy a device (or host) f16 torch tensor into a value without a
        host round trip; a sharded parameter takes the whole tensor."""
        self._call("ipug_session_write", self._s, value, tensor.data_ptr(), tensor.numel() * tensor.element_size(),
                   _stream(stream))

    def read(self, value: int, stream=None, shape=None) -> np.ndarray:
        shape = self.graph.value_shape(value) if shape is None else shape
        out = np.empty(shape, dtype=np.float16)
        self._call("ipug_session_read", self._s, value, out.ctypes.data, out.nbytes, _stream(stream))
        return out

    def diagnose(self, references: dict, stream=None) -> list:
        """Per-value comparison of the session's buffers (after a run) with
        f32 reference values {value id: array} (ipug_session_diagnose)."""
        ids = list(references)
        refs = [np.ascontiguousarray(np.asarray(references[v], dtype=np.float32)) for v in ids]
        ptrs = (ctypes.c_void_p * max(1, len(ids)))(*[r.ctypes.data for r in refs])
        arr, n = _arr(ids)
        out = (ValueReport * max(1, n))()
        self._call("ipug_session_diagnose", self._s, arr, ptrs, n, out, _stream(stream))
        return [{"value": r.value, "producer": r.producer, "available": bool(r.available), "elements": r.elements,
                 "nonfinite": r.nonfinite, "max_abs_err": r.max_abs_err, "max_abs_ref": r.max_abs_ref,
                 "rel_l2": r.rel_l2} for r in out[:n]]

    def device_ptr(self, value: int) -> int:
        return glib().ipug_session_device_ptr(self._s, value)

    def tensor(self, value: int, shape=None):
        """A torch f16 tensor aliasing the value's device buffer (no copy); it
        is valid while the session is open."""
        import torch
        ptr = self.device_ptr(value)
        if not ptr:
            raise IpucError("ipug_session_device_ptr", 1, _lib().ipuc_last_error_string().decode())
        shape = tuple(self.graph.value_shape(value) if shape is None else shape)
        return torch.as_tensor(_DeviceBuffer(ptr, shape), device="cuda")

    def run(self, stream=None):
        self._call("ipug_session_run", self._s, _stream(stream))

    def peer_reduce(self, enable: bool = True, stream=None):
        """Collective: run the all-reduce steps with the library's peer-memory
        kernel (True) or with NCCL (False)."""
        self._call("ipug_session_peer_reduce", self._s, int(bool(enable)), _stream(stream))

    def profile(self, stream=None) -> dict:
        need = ctypes.c_uint64(0)
        glib().ipug_session_profile(self._s, _stream(stream), None, 0, ctypes.byref(need))
        buf = ctypes.create_string_buffer(int(need.value) + 64)
        self._call("ipug_session_profile", self._s, _stream(stream), buf, len(buf), ctypes.byref(need))
        return json.loads(buf.value.decode())

    def profile_capnp(self, physical_tile: int = 0, stream=None) -> bytes:
        """Run once with event timing and return the reference's Cap'n Proto
        Profile message (decode with ipuc.profile.read)."""
        need = ctypes.c_uint64(0)
        glib().ipug_session_profile_capnp(self._s, _stream(stream), physical_tile, None, 0, ctypes.byref(need))
        buf = ctypes.create_string_buffer(int(need.value) + 4096)  # labels may not change, timings can
        self._call("ipug_session_profile_capnp", self._s, _stream(stream), physical_tile, buf, len(buf),
                   ctypes.byref(need))
        return buf.raw[:need.value]

    @property
    def plan(self) -> str:
        return glib().ipug_session_plan(self._s).decode()
