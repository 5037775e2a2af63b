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
    "ipug_session_profile": (ctypes.c_int32, [_vp, _vp, ctypes.c_char_p, ctypes.c_uint64,
                                              ctypes.POINTER(ctypes.c_uint64)]),
    "ipug_session_profile_capnp": (ctypes.c_int32, [_vp, _vp, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64,
                                                    ctypes.POINTER(ctypes.c_uint64)]),
    "ipug_session_plan": (ctypes.c_char_p, [_vp]),
    "ipug_graph_plan": (ctypes.c_int32, [_vp, ctypes.c_char_p, ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
}
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
        self.operations.append(OpRecord("gemm", [left, right], v, dict(transpose_left=transpose_left,
                                                                       transpose_right=transpose_right)))
        return v

    def gelu(self, x: int) -> int:
        v = self._check(glib().ipug_gelu(self._g, x))
        self.operations.append(OpRecord("gelu", [x], v))
        return v

    def add(self, left: int, right: int) -> int:
        v = self._check(glib().ipug_add(self._g, left, right))
        self.operations.append(OpRecord("add", [left, right], v))
        return v

    def split_heads(self, x: int, heads: int) -> int:
        v = self._check(glib().ipug_split_heads(self._g, x, heads))
        self.operations.append(OpRecord("split_heads", [x], v, dict(heads=heads)))
        return v

    def merge_heads(self, x: int, heads: int) -> int:
        """Inverse of split_heads (an extension of the reference's graph API)."""
        v = self._check(glib().ipug_merge_heads(self._g, x, heads))
        self.operations.append(OpRecord("merge_heads", [x], v, dict(heads=heads)))
        return v

    def flash_attention(self, q: int, k: int, v: int) -> int:
        return self.flash_attention_with_options(q, k, v)

    def flash_attention_with_options(self, q: int, k: int, v: int, causal=False, scale=None) -> int:
        r = self._check(glib().ipug_flash_attention(self._g, q, k, v, int(causal), 0.0 if scale is None else scale))
        self.operations.append(OpRecord("flash_attention", [q, k, v], r, dict(causal=causal, scale=scale)))
        return r

    def set_outputs(self, outputs) -> None:
        outs = list(outputs)
        arr = (ctypes.c_int32 * len(outs))(*outs)
        st = glib().ipug_set_outputs(self._g, arr, len(outs))
        if st != OK:
            raise GraphError(_lib().ipuc_last_error_string().decode())
        self.outputs = outs

    def plan(self) -> str:
        """The per-GPU lowering (one line per step), computed on the host
        without a device: the plan a Session of this graph would run."""
        need = ctypes.c_uint64(0)
        glib().ipug_graph_plan(self._g, None, 0, ctypes.byref(need))
        if need.value == 0:
            raise GraphError(_lib().ipuc_last_error_string().decode())
        buf = ctypes.create_string_buffer(need.value)
        st = glib().ipug_graph_plan(self._g, buf, need.value, ctypes.byref(need))
        if st != OK:
            raise IpucError("ipug_graph_plan", st, _lib().ipuc_last_error_string().decode())
        return buf.value.decode()

    def value_shape(self, v: int) -> tuple:
        dims = (ctypes.c_uint32 * 8)()
        r = glib().ipug_value_shape(self._g, v, dims)
        if r < 0:
            raise GraphError(f"unknown value {v}")
        return tuple(dims[:r])


class Session:
    """Lowered graph on one GPU (ipu-runtime's open/load/run/read back)."""

    def __init__(self, graph: ComputeGraph, device: int = 0):
        self.graph = graph
        st = ctypes.c_int32(0)
        self._s = glib().ipug_session_open(graph._g, device, ctypes.byref(st))
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

    def read(self, value: int, stream=None) -> np.ndarray:
        shape = self.graph.value_shape(value)
        out = np.empty(shape, dtype=np.float16)
        self._call("ipug_session_read", self._s, value, out.ctypes.data, out.nbytes, _stream(stream))
        return out

    def device_ptr(self, value: int) -> int:
        return glib().ipug_session_device_ptr(self._s, value)

    def run(self, stream=None):
        self._call("ipug_session_run", self._s, _stream(stream))

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
