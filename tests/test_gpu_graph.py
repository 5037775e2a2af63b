"""ComputeGraph -> per-GPU lowering -> session, checked end to end against the
oracle's restatement of the host evaluator (diagnostic.rs:411-847), with the
FP16 tolerance max|err| <= 2e-2*max|ref|, rel-L2 <= 5e-3."""
import numpy as np
import pytest

import ipuc
import oracle
from conftest import f16_close, seeded_normal
from ipuc.graph import ComputeGraph, Session

pytestmark = pytest.mark.gpu


def run_graph(g, inputs):
    s = Session(g)
    for v, a in inputs.items():
        s.write(v, a)
    s.run()
    return s


def test_mlp_chain_fuses_gelu():
    """mlp-smoke structure (main.rs:1996-2033): GEMM-GELU-GEMM-GELU, 64 wide."""
    g = ComputeGraph()
    x = g.host_input("input", [16, 64])
    w0 = g.parameter("w0", [64, 64])
    w1 = g.parameter("w1", [64, 64])
    y = g.gelu(g.gemm(g.gelu(g.gemm(x, w0)), w1))
    g.set_outputs([y])
    inputs = {x: seeded_normal(1, (16, 64), 0.5), w0: seeded_normal(2, (64, 64), 0.125),
              w1: seeded_normal(3, (64, 64), 0.125)}
    s = run_graph(g, inputs)
    assert s.plan.count("gemm_f16+gelu") == 2
    ref = oracle.evaluate(g, inputs)[y]
    ok, msg = f16_close(s.read(y).astype(np.float32), ref)
    assert ok, msg


def build_block(B, S, d, H, ff):
    g = ComputeGraph()
    x = g.host_input("x", [B, S, d])
    ws = {n: g.parameter(n, shp) for n, shp in [("wq", [d, d]), ("wk", [d, d]), ("wv", [d, d]), ("wo", [d, d]),
                                                ("w1", [d, ff]), ("w2", [ff, d])]}
    q = g.split_heads(g.gemm(x, ws["wq"]), H)
    k = g.split_heads(g.gemm(x, ws["wk"]), H)
    v = g.split_heads(g.gemm(x, ws["wv"]), H)
    a = g.merge_heads(g.flash_attention(q, k, v), H)
    h = g.add(g.gemm(a, ws["wo"]), x)                  # residual add fused into the GEMM
    out = g.add(g.gemm(g.gelu(g.gemm(h, ws["w1"])), ws["w2"]), h)
    g.set_outputs([out])
    return g, x, ws, out


def test_transformer_block_small():
    """Config-5 structure at small size: QKV projections, per-head attention,
    output projection + residual, MLP with GELU + residual."""
    B, S, d, H, ff = 2, 256, 256, 4, 1024
    g, x, ws, out = build_block(B, S, d, H, ff)
    rng = np.random.default_rng(7)
    inputs = {x: rng.standard_normal((B, S, d)).astype(np.float32)}
    for n, v in ws.items():
        inputs[v] = (rng.standard_normal(g.value_shape(v)) * 0.02).astype(np.float32)
    s = run_graph(g, inputs)
    plan = s.plan
    assert plan.count("gemm_f16+add") == 2 and plan.count("gemm_f16+gelu") == 1
    # split-heads -> attention -> merge-heads lowers to one attention call on the
    # unsplit projections (no split or merge copies)
    assert "flash_attention_heads_f16" in plan and "split_heads_f16" not in plan and "merge_heads_f16" not in plan
    ref = oracle.evaluate(g, inputs)[out]
    ok, msg = f16_close(s.read(out).astype(np.float32), ref)
    assert ok, msg
    prof = s.profile()
    assert len(prof["steps"]) == plan.count("\n") and prof["total_ms"] > 0
    assert any("tflops" in st for st in prof["steps"])
    # the same timings as the reference's Cap'n Proto Profile (one tile = this GPU)
    from ipuc import profile as P
    rep = P.read(s.profile_capnp(physical_tile=5))
    assert rep.clock_hz == 1_000_000_000 and [t.physical_tile for t in rep.tiles] == [5]
    samples = rep.tiles[0].samples
    assert [smp.step.kernel for smp in samples] == [st["kernel"] for st in prof["steps"]]
    assert all(smp.step.kind == "compute" and smp.step.operation.startswith("operation.") for smp in samples)
    assert samples[0].start_cycle == 0
    assert all(a.end_cycle <= b.start_cycle + 1 and a.start_cycle <= a.end_cycle for a, b in zip(samples, samples[1:]))
    assert samples[-1].end_cycle > 0
    top = P.query(rep, "kernel")["groups"][0]
    assert top["sampleCount"] >= 1 and top["phaseMs"] > 0


def test_attention_without_merge_keeps_split_heads():
    """An attention result that is itself a graph output is not fused with its
    SplitHeads producers: the plan keeps the split copies and plain attention."""
    B, S, d, H = 2, 192, 256, 2
    g = ComputeGraph()
    x = g.host_input("x", [B, S, d])
    ws = {n: g.parameter(n, [d, d]) for n in ("wq", "wk", "wv")}
    q, k, v = (g.split_heads(g.gemm(x, ws[n]), H) for n in ("wq", "wk", "wv"))
    a = g.flash_attention(q, k, v)
    g.set_outputs([a])
    rng = np.random.default_rng(9)
    inputs = {x: rng.standard_normal((B, S, d)).astype(np.float32)}
    for n, val in ws.items():
        inputs[val] = (rng.standard_normal((d, d)) * 0.05).astype(np.float32)
    s = run_graph(g, inputs)
    assert s.plan.count("split_heads_f16") == 3 and "flash_attention_f16" in s.plan
    ok, msg = f16_close(s.read(a).astype(np.float32), oracle.evaluate(g, inputs)[a])
    assert ok, msg


def test_bias_broadcast_add_and_unfused_gemm():
    g = ComputeGraph()
    x = g.host_input("x", [64, 128])
    w = g.parameter("w", [128, 256])
    b = g.parameter("b", [256])
    y = g.gemm(x, w)
    z = g.add(y, b)          # bias: broadcast add, not fused
    r = g.gelu(y)            # second consumer keeps the GEMM unfused
    g.set_outputs([z, r])
    inputs = {x: seeded_normal(4, (64, 128)), w: seeded_normal(5, (128, 256), 0.1), b: seeded_normal(6, (256,))}
    s = run_graph(g, inputs)
    assert "gemm_f16 " in s.plan and "add_f16" in s.plan and "gelu_f16" in s.plan
    ref = oracle.evaluate(g, inputs)
    for v in (z, r):
        ok, msg = f16_close(s.read(v).astype(np.float32), ref[v])
        assert ok, msg


def test_unsupported_features_fail_loudly():
    g = ComputeGraph()
    q = g.host_input("q", [2, 64, 64])
    g.flash_attention_with_options(q, q, q, causal=True)
    with pytest.raises(ipuc.IpucError) as e:
        Session(g)
    assert e.value.status == ipuc.ERR_UNSUPPORTED


def test_add_of_two_gemms():
    """Add(Gemm(x, W1), Gemm(y, W2)): one GEMM fused with the Add, the other kept."""
    g = ComputeGraph()
    x = g.host_input("x", [192, 128])
    y = g.host_input("y", [192, 96])
    w1 = g.parameter("w1", [128, 256])
    w2 = g.parameter("w2", [96, 256])
    s = g.add(g.gemm(x, w1), g.gemm(y, w2))
    g.set_outputs([s])
    inputs = {x: seeded_normal(11, (192, 128)), y: seeded_normal(12, (192, 96)),
              w1: seeded_normal(13, (128, 256), 0.1), w2: seeded_normal(14, (96, 256), 0.1)}
    sess = run_graph(g, inputs)
    assert sess.plan.count("gemm_f16+add") == 1
    ok, msg = f16_close(sess.read(s).astype(np.float32), oracle.evaluate(g, inputs)[s])
    assert ok, msg
