"""The sampled checkers that the BASELINE-size GPU tests and bench.py use
(oracle.mlp_rows, oracle.block_rows, oracle.compare_f16) agree with the full
evaluator (oracle.evaluate) on the rows they cover."""
import numpy as np

import oracle
from ipuc.graph import ComputeGraph


def test_block_rows_match_evaluate():
    B, S, d, H, ff = 2, 64, 64, 4, 128
    g = ComputeGraph()
    x = g.host_input("x", [B, S, d])
    w = {n: g.parameter(n, shp) for n, shp in [("wq", [d, d]), ("wk", [d, d]), ("wv", [d, d]), ("wo", [d, d]),
                                               ("w1", [d, ff]), ("w2", [ff, d])]}
    q = g.split_heads(g.gemm(x, w["wq"]), H)
    k = g.split_heads(g.gemm(x, w["wk"]), H)
    v = g.split_heads(g.gemm(x, w["wv"]), H)
    a = g.merge_heads(g.flash_attention(q, k, v), H)
    h = g.add(g.gemm(a, w["wo"]), x)
    y = g.add(g.gemm(g.gelu(g.gemm(h, w["w1"])), w["w2"]), h)
    g.set_outputs([y])
    rng = np.random.default_rng(3)
    xin = rng.standard_normal((B, S, d)).astype(np.float32)
    wv = {n: (rng.standard_normal(g.value_shape(val)) * 0.1).astype(np.float32) for n, val in w.items()}
    inputs = {x: xin, **{w[n]: wv[n] for n in w}}
    full = oracle.evaluate(g, inputs, threads=2)[y]
    rows = np.array([0, 5, 33, S - 1])
    for b in range(B):
        part = oracle.block_rows(xin[b], wv, H, rows, threads=2)
        assert np.array_equal(part, full[b, rows])


def test_mlp_rows_match_evaluate():
    rng = np.random.default_rng(4)
    xin = rng.standard_normal((32, 48)).astype(np.float32)
    win = (rng.standard_normal((48, 40)) / 7).astype(np.float32)
    g = ComputeGraph()
    x = g.host_input("x", [32, 48])
    w = g.parameter("w", [48, 40])
    y = g.gelu(g.gemm(x, w))
    g.set_outputs([y])
    full = oracle.evaluate(g, {x: xin, w: win})[y]
    rows = np.array([1, 7, 31])
    assert np.array_equal(oracle.mlp_rows(xin[rows], win), full[rows])


def test_compare_f16_limits():
    ref = np.linspace(-1, 1, 1000).astype(np.float32)
    assert oracle.compare_f16(ref, ref)["pass"]
    bad = ref.copy()
    bad[10] += 0.05          # one element 2.5e-2 of max|ref| off
    r = oracle.compare_f16(bad, ref)
    assert not r["pass"] and abs(r["max_err_over_max_ref"] - 0.05) < 1e-6
    nan = ref.copy()
    nan[3] = np.nan
    assert not oracle.compare_f16(nan, ref)["pass"]
