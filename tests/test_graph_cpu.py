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
