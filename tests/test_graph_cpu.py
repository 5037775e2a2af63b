"""Graph construction and shape inference on CPU (no device calls): the
checks of crates/ipu-codegen/src/graph.rs:836-966 restated."""
import pytest

from ipuc.graph import ComputeGraph, GraphError


def test_gemm_shape_with_batch_broadcast():
    g = ComputeGraph()
    a = g.host_input("a", [4, 1, 16, 32])
    b = g.parameter("b", [3, 32, 8])
    c = g.gemm(a, b)
    assert g.value_shape(c) == (4, 3, 16, 8)
    d = g.gemm_with_options(a, g.parameter("bt", [8, 32]), transpose_right=True)
    assert g.value_shape(d) == (4, 1, 16, 8)


def test_invalid_shapes_raise():
    g = ComputeGraph()
    a = g.host_input("a", [16, 32])
    with pytest.raises(GraphError, match="inner dimensions"):
        g.gemm(a, g.parameter("b", [31, 8]))
    with pytest.raises(GraphError, match="rank at least two"):
        g.gemm(a, g.parameter("v", [32]))
    with pytest.raises(GraphError, match="divisible"):
        g.split_heads(g.host_input("x", [2, 4, 30]), 4)
    with pytest.raises(GraphError, match="head or sequence"):
        g.flash_attention(g.host_input("q", [2, 4, 8]), g.host_input("k", [2, 5, 9]), g.host_input("v", [2, 5, 8]))
    with pytest.raises(GraphError, match="broadcast"):
        g.add(a, g.host_input("z", [3, 32]))
    with pytest.raises(GraphError):
        g.host_input("", [1])
    with pytest.raises(GraphError):
        g.gelu(999)


def test_split_heads_and_attention_shapes():
    g = ComputeGraph()
    x = g.host_input("x", [2, 17, 64])
    h = g.split_heads(x, 4)
    assert g.value_shape(h) == (8, 17, 16)
    o = g.flash_attention(h, h, h)
    assert g.value_shape(o) == (8, 17, 16)
    s = g.add(x, g.parameter("bias", [64]))
    assert g.value_shape(s) == (2, 17, 64)
    g.set_outputs([o, s])
    assert g.outputs == [o, s]


# ---- lowering decisions (ipug_graph_plan: the per-GPU plan, computed on the host) ----

def block(B, S, d, H, ff, merge=True):
    g = ComputeGraph()
    x = g.host_input("x", [B, S, d])
    w = {n: g.parameter(n, s) for n, s in [("wq", [d, d]), ("wk", [d, d]), ("wv", [d, d]), ("wo", [d, d]),
                                           ("w1", [d, ff]), ("w2", [ff, d])]}
    q, k, v = (g.split_heads(g.gemm(x, w[n]), H) for n in ("wq", "wk", "wv"))
    a = g.flash_attention(q, k, v)
    if not merge:
        g.set_outputs([a])
        return g
    h = g.add(g.gemm(g.merge_heads(a, H), w["wo"]), x)
    y = g.add(g.gemm(g.gelu(g.gemm(h, w["w1"])), w["w2"]), h)
    g.set_outputs([y])
    return g


def labels(plan):
    return [line.split()[0] for line in plan.strip().splitlines()]


def test_transformer_block_lowering():
    """Config 5: QKV GEMMs, one strided-heads attention (split x3 -> attention ->
    merge fused), output projection with the residual added by the GEMM
    epilogue, MLP up with fused GELU, MLP down + residual."""
    plan = block(4, 2048, 4096, 32, 16384).plan()
    assert labels(plan) == ["gemm_f16"] * 3 + ["flash_attention_heads_f16", "gemm_f16+add", "gemm_f16+gelu",
                                                "gemm_f16+add"]
    assert "split_heads" not in plan and "merge_heads" not in plan


def test_attention_output_keeps_split_heads():
    """An attention result that is itself an output is not fused with its splits."""
    assert labels(block(2, 64, 256, 2, 512, merge=False).plan()) == \
        ["gemm_f16", "split_heads_f16"] * 3 + ["flash_attention_f16"]


def test_shared_split_is_not_fused():
    """A split value used twice (here as both key and value) stays a copy."""
    g = ComputeGraph()
    x = g.host_input("x", [2, 64, 256])
    q = g.split_heads(g.gemm(x, g.parameter("wq", [256, 256])), 2)
    kv = g.split_heads(g.gemm(x, g.parameter("wk", [256, 256])), 2)
    g.set_outputs([g.merge_heads(g.flash_attention(q, kv, kv), 2)])
    got = labels(g.plan())
    assert "flash_attention_f16" in got and "flash_attention_heads_f16" not in got
    assert got.count("split_heads_f16") == 2 and got.count("merge_heads_f16") == 1


def test_plan_reports_unsupported_features():
    g = ComputeGraph()
    q = g.host_input("q", [2, 64, 64])
    g.set_outputs([g.flash_attention_with_options(q, q, q, causal=True)])
    with pytest.raises(Exception, match="causal"):
        g.plan()


def test_add_of_two_gemms_fuses_one():
    """x W1 + y W2 with both products used once: the first GEMM's epilogue adds
    the second GEMM's result, which keeps its own step and buffer."""
    g = ComputeGraph()
    x = g.host_input("x", [64, 128])
    y = g.host_input("y", [64, 96])
    s = g.add(g.gemm(x, g.parameter("w1", [128, 256])), g.gemm(y, g.parameter("w2", [96, 256])))
    g.set_outputs([s])
    assert labels(g.plan()) == ["gemm_f16", "gemm_f16+add"]


# ---- Repeat regions and value sequences (graph.rs:294-313, 382-473) ----

def mlp_repeat(blocks=3, d=64, hidden=256):
    """The SiglipMlpBenchmark graph shape (main.rs:707-756): GEMM-GELU-GEMM
    blocks in a Repeat over sequences of up and down weights."""
    g = ComputeGraph()
    x = g.host_input("left", [2, 16, d])
    ups = [g.parameter(f"up{i}", [1, d, hidden]) for i in range(blocks)]
    downs = [g.parameter(f"down{i}", [1, hidden, d]) for i in range(blocks)]
    su = g.value_sequence("MLP up weights", ups)
    sd = g.value_sequence("MLP down weights", downs)
    y = g.repeat(blocks, [x], [], [su, sd],
                 lambda b, a: [b.gemm(b.gelu(b.gemm(a.carried[0], a.iterated[0])), a.iterated[1])])[0]
    g.set_outputs([y])
    return g, x, ups, downs, y


def test_repeat_unrolls_per_iteration():
    g, x, ups, downs, y = mlp_repeat()
    assert g.value_shape(y) == (2, 16, 64)
    plan = g.plan().strip().splitlines()
    assert [l.split()[0] for l in plan] == ["gemm_f16+gelu", "gemm_f16"] * 3
    assert [l.split()[-1] for l in plan] == ["iter=0", "iter=0", "iter=1", "iter=1", "iter=2", "iter=2"]
    rep = g.operations[-1]
    assert rep.kind == "repeat" and rep.options["count"] == 3 and len(rep.options["body"]) == 3


def test_repeat_errors_follow_graph_error():
    g = ComputeGraph()
    x = g.host_input("x", [4, 8])
    w = g.parameter("w", [8, 8])
    other = g.parameter("o", [8, 4])
    seq = g.value_sequence("ws", [w, w])
    with pytest.raises(GraphError, match="nonzero"):
        g.repeat(0, [x], [], [], lambda b, a: [a.carried[0]])
    with pytest.raises(GraphError, match="2 entries for 3 iterations"):
        g.repeat(3, [x], [], [seq], lambda b, a: [a.carried[0]])
    with pytest.raises(GraphError, match="yielded 0 values for 1 carried"):
        g.repeat(2, [x], [], [seq], lambda b, a: [])
    with pytest.raises(GraphError, match="does not have the shape of carried value 0"):
        g.repeat(2, [x], [other], [], lambda b, a: [b.gemm(a.carried[0], a.invariants[0])])  # [4, 4] for [4, 8]
    with pytest.raises(GraphError, match="not available"):
        g.repeat(2, [x], [], [seq], lambda b, a: [b.gemm(a.carried[0], w)])  # outer value used inside the body
    with pytest.raises(GraphError, match="different shape"):
        g.value_sequence("bad", [w, other])
    # the graph is still usable after the failed bodies
    y = g.repeat(2, [x], [w], [seq], lambda b, a: [b.add(b.gemm(a.carried[0], a.iterated[0]), a.carried[0])])[0]
    g.set_outputs([y])
    assert g.value_shape(y) == (4, 8)
    assert len(g.plan().strip().splitlines()) == 2


def test_repeat_matches_unrolled_evaluation():
    """oracle.evaluate's Repeat (repeat_values, diagnostic.rs:467-520) equals the
    same graph written out iteration by iteration."""
    import numpy as np
    import oracle
    g, x, ups, downs, y = mlp_repeat(blocks=2, d=32, hidden=64)
    rng = np.random.default_rng(2)
    inputs = {x: rng.standard_normal((2, 16, 32)).astype(np.float32)}
    for v in ups + downs:
        inputs[v] = (rng.standard_normal(g.value_shape(v)) * 0.2).astype(np.float32)
    g2 = ComputeGraph()
    x2 = g2.host_input("left", [2, 16, 32])
    u2 = [g2.parameter(f"up{i}", [1, 32, 64]) for i in range(2)]
    d2 = [g2.parameter(f"down{i}", [1, 64, 32]) for i in range(2)]
    h = x2
    for i in range(2):
        h = g2.gemm(g2.gelu(g2.gemm(h, u2[i])), d2[i])
    g2.set_outputs([h])
    in2 = {x2: inputs[x], **{u2[i]: inputs[ups[i]] for i in range(2)}, **{d2[i]: inputs[downs[i]] for i in range(2)}}
    assert np.array_equal(oracle.evaluate(g, inputs)[y], oracle.evaluate(g2, in2)[h])


def test_transpose_left_lowers_to_m_major_gemm():
    g = ComputeGraph()
    a = g.host_input("a", [64, 128])        # [k, m]
    b = g.parameter("b", [64, 32])
    c = g.gemm_with_options(a, b, transpose_left=True)
    g.set_outputs([c])
    assert g.value_shape(c) == (128, 32)
    assert labels(g.plan()) == ["gemm_f16"]
