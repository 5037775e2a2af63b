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
