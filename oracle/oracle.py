"""CPU oracle for the ipu-stack operator-catalog hot path.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, always as the checker, never
as the thing measured or shipped.  The product library (libipuc.so) neither
links nor calls anything here.

It restates the reference's host-side evaluator,
crates/ipu-tests/src/diagnostic.rs:411-847 (``evaluate``):

* every op result is quantised to its storage precision (diagnostic.rs:454-460);
* GEMM is ``cblas_sgemm`` row-major, alpha 1, beta 0 (diagnostic.rs:581-654).
  Here that is numpy's matmul on float32, which dispatches to the OpenBLAS
  0.3.30 numpy bundles (the same library family the reference links with
  ``#[link(name = "openblas")]``);
* GELU is ``gelu_reference`` (crates/ipu-tests/src/main.rs:1985-1987);
* attention, split_heads, add and the layout maps are in oracle.c (scalar C),
  each citing the reference function it follows.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

# Element orders, numbered as in include/ipuc.h (ipuc_order).
ROW_MAJOR, AMP_LEFT, AMP_TRANSPOSED_LEFT, AMP_TRANSPOSED_RIGHT = 0, 1, 2, 3
AMP_OUTPUT, AMP_TRANSPOSED_OUTPUT, BLOCK_MAJOR, BLOCK_MAJOR_TRANSPOSED = 4, 5, 6, 7


def build() -> str:
    path = os.path.join(_HERE, "liboracle.so")
    src = os.path.join(_HERE, "oracle.c")
    if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return path


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        L = ctypes.CDLL(build())
        i64, i32, f32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p
        L.oracle_layout_index.restype = i64
        L.oracle_layout_index.argtypes = [i32, i64, i64, i64, i64, i64, i64]
        L.oracle_layout_coordinates.restype = i32
        L.oracle_layout_coordinates.argtypes = [i32, i64, i64, i64, i64, i64,
                                                ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.oracle_rearrange_f16.restype = i32
        L.oracle_rearrange_f16.argtypes = [vp, vp, i64, i64, i64, i32, i64, i64, i64, i64]
        L.oracle_unpack_f16.restype = i32
        L.oracle_unpack_f16.argtypes = [vp, vp, i32, i64, i64, i64, i64, i64]
        L.oracle_gelu.restype = f32
        L.oracle_gelu.argtypes = [f32]
        L.oracle_gelu_f16.argtypes = [vp, vp, i64]
        L.oracle_reduce_sum.argtypes = [vp, vp, vp, i64, i64, i32]
        L.oracle_sgemm_scalar.argtypes = [vp, vp, vp, i64, i64, i64, i32, i32]
        L.oracle_attention.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, i32, i32]
        L.oracle_flash_attention_online.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, f32, i64]
        L.oracle_attention_softmax.argtypes = [vp, vp, vp, i64, i64, i64, i64]
        L.oracle_attention_merge.argtypes = [vp, vp, vp, i64, i64, i64, i32, i32]
        L.oracle_split_heads.argtypes = [vp, vp, i64, i64, i64, i64]
        L.oracle_add_f16.argtypes = [vp, vp, vp, i64, i64, i64]
        L.oracle_f32_to_half.restype = ctypes.c_uint16
        L.oracle_f32_to_half.argtypes = [f32]
        L.oracle_half_to_f32.restype = f32
        L.oracle_half_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f32_to_half_array.argtypes = [vp, vp, i64]
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# --------------------------------------------------------------------------
# Precision helpers (diagnostic.rs:841-847 quantize; main.rs:2040-2046)
# --------------------------------------------------------------------------

def f16_bits(x: np.ndarray) -> np.ndarray:
    """f32 -> IEEE binary16 bits, round to nearest even (the `half` crate)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_half_array(_p(x), _p(out), x.size)
    return out


def quantize_f16(x: np.ndarray) -> np.ndarray:
    return f16_bits(x).view(np.float16).astype(np.float32)


# --------------------------------------------------------------------------
# Evaluator ops (diagnostic.rs:411-847)
# --------------------------------------------------------------------------

def gemm(left: np.ndarray, right: np.ndarray, transpose_left=False, transpose_right=False) -> np.ndarray:
    """diagnostic.rs:533-654: f32 SGEMM on (already quantised) f32 operands."""
    a = np.asarray(left, dtype=np.float32)
    b = np.asarray(right, dtype=np.float32)
    if transpose_left:
        a = np.swapaxes(a, -1, -2)
    if transpose_right:
        b = np.swapaxes(b, -1, -2)
    return np.matmul(a, b).astype(np.float32)


def gemm_scalar(a: np.ndarray, b: np.ndarray, ta=False, tb=False) -> np.ndarray:
    """Scalar f32 loop used to pin the BLAS path (diagnostic.rs:855-907)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    M = a.shape[1] if ta else a.shape[0]
    K = a.shape[0] if ta else a.shape[1]
    N = b.shape[0] if tb else b.shape[1]
    out = np.empty((M, N), dtype=np.float32)
    lib().oracle_sgemm_scalar(_p(out), _p(a), _p(b), M, N, K, int(ta), int(tb))
    return out


def gelu(x: np.ndarray) -> np.ndarray:
    """gelu_reference (main.rs:1985-1987) elementwise in f32."""
    x = np.asarray(x, dtype=np.float32)
    return (0.5 * x * (1.0 + np.tanh(np.float32(0.7978846) * (x + np.float32(0.044715) * (x * x * x))))).astype(np.float32)


def gelu_f16_bits(x_bits: np.ndarray) -> np.ndarray:
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    out = np.empty_like(x_bits)
    lib().oracle_gelu_f16(_p(out), _p(x_bits), x_bits.size)
    return out


def reduce_sum(initial: np.ndarray, remote: np.ndarray) -> np.ndarray:
    """out = p0 + sum(remote partials) -> f16 bits.  remote: [P, n]."""
    initial = np.ascontiguousarray(initial)
    remote = np.ascontiguousarray(remote)
    in_f32 = initial.dtype == np.float32
    if not in_f32:
        initial = initial.view(np.uint16) if initial.dtype == np.float16 else initial
        remote = remote.view(np.uint16) if remote.dtype == np.float16 else remote
    n = initial.size
    P = remote.size // max(n, 1)
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_reduce_sum(_p(out), _p(initial), _p(remote), P, n, int(in_f32))
    return out


def attention(q, k, v, scale=None, causal=False, threads=1) -> np.ndarray:
    """diagnostic.rs:711-780 scalar attention.  q:[S,Sq,D] k:[S,Sk,D] v:[S,Sk,Dv] f32."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    S, Sq, D = q.shape
    Sk, Dv = k.shape[1], v.shape[2]
    if scale is None:
        scale = 1.0 / float(np.sqrt(np.float32(D)))
    out = np.empty((S, Sq, Dv), dtype=np.float32)
    lib().oracle_attention(_p(out), _p(q), _p(k), _p(v), S, Sq, Sk, D, Dv, float(scale), int(causal), int(threads))
    return out


def flash_attention_online(q_bits, k_bits, v_bits, scale=None, key_block=32) -> np.ndarray:
    """device/flash_attention_online_f16.cpp:61-143 (f16 in, f32 out)."""
    q_bits = np.ascontiguousarray(q_bits, dtype=np.uint16)
    k_bits = np.ascontiguousarray(k_bits, dtype=np.uint16)
    v_bits = np.ascontiguousarray(v_bits, dtype=np.uint16)
    M, Sq, D = q_bits.shape
    Sk, Dv = k_bits.shape[1], v_bits.shape[2]
    if scale is None:
        scale = 1.0 / float(np.sqrt(np.float32(D)))
    out = np.empty((M, Sq, Dv), dtype=np.float32)
    lib().oracle_flash_attention_online(_p(out), _p(q_bits), _p(k_bits), _p(v_bits), M, Sq, Sk, D, Dv,
                                        float(scale), key_block)
    return out


def attention_softmax(scores_bits, query_rows, key_rows, key_block_columns, head_dim):
    scores_bits = np.ascontiguousarray(scores_bits, dtype=np.uint16)
    w = np.empty(query_rows * key_block_columns, dtype=np.uint16)
    state = np.empty(2 * query_rows, dtype=np.float32)
    lib().oracle_attention_softmax(_p(w), _p(state), _p(scores_bits), query_rows, key_rows,
                                   key_block_columns, head_dim)
    return w, state


def attention_merge(acc, block_bits, state, query_rows, V, Vp, initial, final):
    acc = np.ascontiguousarray(acc, dtype=np.float32).copy()
    block_bits = np.ascontiguousarray(block_bits, dtype=np.uint16)
    state = np.ascontiguousarray(state, dtype=np.float32)
    lib().oracle_attention_merge(_p(acc), _p(block_bits), _p(state), query_rows, V, Vp, int(initial), int(final))
    return acc


def split_heads(x_bits: np.ndarray, heads: int) -> np.ndarray:
    x_bits = np.ascontiguousarray(x_bits, dtype=np.uint16)
    b, r, w = x_bits.shape
    out = np.empty((b * heads, r, w // heads), dtype=np.uint16)
    lib().oracle_split_heads(_p(out), _p(x_bits), b, r, heads, w // heads)
    return out


def add_f16(left_bits, right_bits, n, left_period=0, right_period=0):
    left_bits = np.ascontiguousarray(left_bits, dtype=np.uint16)
    right_bits = np.ascontiguousarray(right_bits, dtype=np.uint16)
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_add_f16(_p(out), _p(left_bits), _p(right_bits), n, left_period, right_period)
    return out


# --------------------------------------------------------------------------
# Layouts (crates/ipu-codegen/src/storage.rs) and rearranges (device/*.cpp)
# --------------------------------------------------------------------------

def layout_index(order, rows, cols, r, c, row_block=64, column_block=16) -> int:
    return lib().oracle_layout_index(order, row_block, column_block, rows, cols, r, c)


def layout_coordinates(order, rows, cols, linear, row_block=64, column_block=16):
    r, c = ctypes.c_int64(), ctypes.c_int64()
    rc = lib().oracle_layout_coordinates(order, row_block, column_block, rows, cols, linear,
                                         ctypes.byref(r), ctypes.byref(c))
    if rc != 0:
        raise ValueError("invalid view")
    return r.value, c.value


def rearrange_f16(src_bits, matrices, R, Rp, target, C, Cp, row_block=64, column_block=16):
    src_bits = np.ascontiguousarray(src_bits, dtype=np.uint16)
    dst = np.empty(matrices * Rp * Cp, dtype=np.uint16)
    rc = lib().oracle_rearrange_f16(_p(dst), _p(src_bits), matrices, R, Rp, target, C, Cp, row_block, column_block)
    if rc != 0:
        raise ValueError("unsupported rearrange geometry")
    return dst


def unpack_f16(src_bits, source_order, matrices, R, Rp, C, Cp):
    src_bits = np.ascontiguousarray(src_bits, dtype=np.uint16)
    dst = np.empty(matrices * Rp * Cp, dtype=np.uint16)
    rc = lib().oracle_unpack_f16(_p(dst), _p(src_bits), source_order, matrices, R, Rp, C, Cp)
    if rc != 0:
        raise ValueError("unsupported unpack geometry")
    return dst


# --------------------------------------------------------------------------
# Whole-graph evaluation: evaluate_operations (diagnostic.rs:420-464)
# --------------------------------------------------------------------------

def _attention_batched(q, k, v, scale, threads):
    lead = q.shape[:-2]
    s = int(np.prod(lead)) if lead else 1
    out = attention(q.reshape(s, *q.shape[-2:]), k.reshape(s, *k.shape[-2:]), v.reshape(s, *v.shape[-2:]),
                    scale=scale, threads=threads)
    return out.reshape(*lead, q.shape[-2], v.shape[-1])


def evaluate(graph, inputs: dict, threads: int = 8) -> dict:
    """Evaluate a recorded ComputeGraph (ipuc.graph.ComputeGraph) on f32 host
    values.  `inputs` maps input value ids to arrays; every input is first
    quantised to f16 (prepare_inputs, diagnostic.rs:324-341) and every op
    result is quantised to f16 (diagnostic.rs:454-460).  Returns a dict of
    value id -> f32 array."""
    vals = {v: quantize_f16(np.asarray(a, dtype=np.float32)) for v, a in inputs.items()}
    _evaluate_ops(graph.operations, vals, threads)
    return vals


def _repeat(op, vals, threads):
    """repeat_values (diagnostic.rs:467-520): the body runs `count` times on a
    copy of the values, carried arguments bound to the previous iteration's
    yields, invariants to the Repeat's invariant operands and iterated
    arguments to entry `iteration` of each sequence."""
    o = op.options
    nc, ni = o["carried"], o["invariants"]
    carried = [vals[v] for v in op.inputs[:nc]]
    invariants = [vals[v] for v in op.inputs[nc:nc + ni]]
    args = o["arguments"]
    for it in range(o["count"]):
        local = dict(vals)
        for a, x in zip(args[:nc], carried):
            local[a] = x
        for a, x in zip(args[nc:nc + ni], invariants):
            local[a] = x
        for a, seq in zip(args[nc + ni:], o["sequences"]):
            local[a] = vals[seq[it]]
        _evaluate_ops(o["body"], local, threads)
        carried = [local[y] for y in o["yields"]]
    for r, x in zip(o["results"], carried):
        vals[r] = x


def _evaluate_ops(operations, vals, threads):
    for op in operations:
        if op.kind == "repeat":
            _repeat(op, vals, threads)
            continue
        ins = [vals[i] for i in op.inputs]
        if op.kind == "gemm":
            r = gemm(ins[0], ins[1], op.options["transpose_left"], op.options["transpose_right"])
        elif op.kind == "gelu":
            r = gelu(ins[0])
        elif op.kind == "add":
            r = (ins[0] + ins[1]).astype(np.float32)
        elif op.kind == "split_heads":
            b, rows, w = ins[0].shape
            h = op.options["heads"]
            r = ins[0].reshape(b, rows, h, w // h).transpose(0, 2, 1, 3).reshape(b * h, rows, w // h)
        elif op.kind == "merge_heads":
            bh, rows, c = ins[0].shape
            h = op.options["heads"]
            r = ins[0].reshape(bh // h, h, rows, c).transpose(0, 2, 1, 3).reshape(bh // h, rows, h * c)
        elif op.kind == "flash_attention":
            if op.options.get("causal"):
                raise NotImplementedError("causal attention")
            r = _attention_batched(ins[0], ins[1], ins[2], op.options.get("scale"), threads)
        else:
            raise ValueError(op.kind)
        vals[op.result] = quantize_f16(np.ascontiguousarray(r, dtype=np.float32))


# --------------------------------------------------------------------------
# Sampled checks of full-size workloads: the evaluator restricted to a few
# output rows, so that a GPU result at BASELINE size can be compared in seconds
# --------------------------------------------------------------------------

F16_MAX_REL, F16_REL_L2 = 2e-2, 5e-3   # BASELINE FP16 tolerance


def compare_f16(actual, ref, max_rel=F16_MAX_REL, rel_l2=F16_REL_L2) -> dict:
    """max|err| / max|ref| and rel-L2 of `actual` against `ref`, with pass/fail
    against the FP16 tolerance (max|err| <= 2e-2 max|ref|, rel-L2 <= 5e-3)."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    err = np.abs(a - r)
    mr = float(err.max() / max(np.abs(r).max(), 1e-30)) if err.size else 0.0
    l2 = float(np.linalg.norm(a - r) / max(np.linalg.norm(r), 1e-30)) if err.size else 0.0
    finite = bool(np.isfinite(a).all())
    return {"max_err_over_max_ref": mr, "rel_l2": l2, "elements": int(err.size),
            "pass": bool(finite and mr <= max_rel and l2 <= rel_l2)}


def mlp_rows(x_rows, w) -> np.ndarray:
    """Rows of the MLP up-projection graph GELU(X W) (config 3, GELU fused or
    not): evaluate() quantises the GEMM result and the GELU result to f16."""
    return quantize_f16(gelu(quantize_f16(gemm(quantize_f16(x_rows), quantize_f16(w)))))


def block_rows(x_b, w: dict, heads: int, rows, threads: int = 8) -> np.ndarray:
    """evaluate() of the transformer-block graph
        h = Wo-proj(merge_heads(attention(split_heads(x Wq), split_heads(x Wk), split_heads(x Wv)))) + x
        y = GELU(h W1) W2 + h
    restricted to token rows `rows` of one batch element x_b [S, d].  A row's
    attention reads K and V of every row of its batch element, so those two
    projections are evaluated in full; everything else only for `rows`.
    Every op result is quantised to f16 (diagnostic.rs:454-460)."""
    q16 = quantize_f16
    x_b = q16(x_b)
    W = {n: q16(a) for n, a in w.items()}
    rows = np.asarray(rows)
    S, d = x_b.shape
    dh = d // heads
    xr = x_b[rows]
    q = q16(gemm(xr, W["wq"]))
    k = q16(gemm(x_b, W["wk"]))
    v = q16(gemm(x_b, W["wv"]))
    qh = np.ascontiguousarray(q.reshape(len(rows), heads, dh).transpose(1, 0, 2))
    kh = np.ascontiguousarray(k.reshape(S, heads, dh).transpose(1, 0, 2))
    vh = np.ascontiguousarray(v.reshape(S, heads, dh).transpose(1, 0, 2))
    a = q16(attention(qh, kh, vh, threads=threads))
    a = np.ascontiguousarray(a.transpose(1, 0, 2).reshape(len(rows), d))
    h = q16(q16(gemm(a, W["wo"])) + xr)
    u = q16(gelu(q16(gemm(h, W["w1"]))))
    return q16(q16(gemm(u, W["w2"])) + h)
