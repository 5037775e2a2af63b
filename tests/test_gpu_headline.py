"""Parity at the BASELINE sizes the bench times, by row sampling: the GPU runs
the full workload, the oracle evaluates a sample of output rows (each row of
these workloads depends on whole inputs, so a row sample is an exact check of
those rows).  FP16 tolerance max|err| <= 2e-2*max|ref|, rel-L2 <= 5e-3.

* config 3: X[8192x4096] W[4096x16384], GELU fused, 128 rows x all columns;
  and the 8-GPU column shard (8192x2048x4096);
* config 4: 256 streams x 4096 x 128 flash attention, 4 streams x 128 query
  rows over all keys; and the 8-GPU shard (32 streams, split-cluster tail);
* config 5: the transformer block (B=4, S=2048, d=4096, 32 heads, ff=16384)
  through the graph session, 8 token rows against the evaluator restricted to
  those rows (oracle.block_rows).
"""
import os

import numpy as np
import pytest
import torch

import ipuc
import oracle

pytestmark = pytest.mark.gpu
THREADS = os.cpu_count() or 8


def _check(got, ref):
    r = oracle.compare_f16(got, ref)
    assert r["pass"], r


@pytest.mark.parametrize("n", [16384, 2048])
def test_config3_mlp_up_projection_sampled(n):
    m, k = 8192, 4096
    g = torch.Generator(device="cuda")
    g.manual_seed(31 + n)
    x = torch.randn((m, k), generator=g, device="cuda").half()
    w = (torch.randn((k, n), generator=g, device="cuda") / 64).half()
    y = torch.full((m, n), float("nan"), dtype=torch.float16, device="cuda")
    ipuc.gemm_f16(y, x, w, m, n, k, flags=ipuc.GEMM_EPILOGUE_GELU)
    torch.cuda.synchronize()
    rows = np.sort(np.random.default_rng(n).choice(m, 128, replace=False))
    # the first and last row tiles of the persistent schedule are in the sample too
    rows = np.unique(np.concatenate([rows, [0, 255, m - 256, m - 1]]))
    ri = torch.from_numpy(rows).cuda()
    got = y.index_select(0, ri).float().cpu().numpy()
    ref = oracle.mlp_rows(x.index_select(0, ri).float().cpu().numpy(), w.float().cpu().numpy())
    _check(got, ref)
    assert not torch.isnan(y).any().item(), "unwritten output elements"


@pytest.mark.parametrize("streams", [256, 32])
def test_config4_attention_sampled(streams):
    S, D = 4096, 128
    g = torch.Generator(device="cuda")
    g.manual_seed(41 + streams)
    q, k, v = (torch.randn((streams, S, D), generator=g, device="cuda").half() for _ in range(3))
    o = torch.full((streams, S, D), float("nan"), dtype=torch.float16, device="cuda")
    ipuc.flash_attention_f16(o, q, k, v, streams, S, S, D)
    torch.cuda.synchronize()
    rng = np.random.default_rng(streams)
    # first, last and two random streams: the last stream's units run in the tail
    st = np.unique(np.concatenate([[0, streams - 1], rng.choice(streams, 2, replace=False)]))
    qr = np.unique(np.concatenate([[0, S - 1], rng.choice(S, 126, replace=False)]))
    si, qi = torch.from_numpy(st).cuda(), torch.from_numpy(qr).cuda()
    got = o.index_select(0, si).index_select(1, qi).float().cpu().numpy()
    ref = oracle.attention(q.index_select(0, si).index_select(1, qi).float().cpu().numpy(),
                           k.index_select(0, si).float().cpu().numpy(), v.index_select(0, si).float().cpu().numpy(),
                           threads=THREADS)
    _check(got, oracle.quantize_f16(ref))
    assert not torch.isnan(o).any().item(), "unwritten output elements"


def test_config5_transformer_block_sampled():
    from ipuc.graph import ComputeGraph, Session
    B, S, d, H, ff = 4, 2048, 4096, 32, 16384
    gr = ComputeGraph()
    x = gr.host_input("x", [B, S, d])
    w = {n: gr.parameter(n, shp) for n, shp in [("wq", [d, d]), ("wk", [d, d]), ("wv", [d, d]), ("wo", [d, d]),
                                                ("w1", [d, ff]), ("w2", [ff, d])]}
    q = gr.split_heads(gr.gemm(x, w["wq"]), H)
    k = gr.split_heads(gr.gemm(x, w["wk"]), H)
    v = gr.split_heads(gr.gemm(x, w["wv"]), H)
    a = gr.merge_heads(gr.flash_attention(q, k, v), H)
    h = gr.add(gr.gemm(a, w["wo"]), x)
    y = gr.add(gr.gemm(gr.gelu(gr.gemm(h, w["w1"])), w["w2"]), h)
    gr.set_outputs([y])
    rng = np.random.default_rng(5)
    xin = rng.standard_normal((B, S, d), dtype=np.float32)
    wv = {n: rng.standard_normal(gr.value_shape(val), dtype=np.float32) * np.float32(0.02) for n, val in w.items()}
    sess = Session(gr)
    sess.write(x, xin)
    for n, val in w.items():
        sess.write(val, wv[n])
    sess.run()
    got = sess.read(y).astype(np.float32)
    sess.close()
    pick = np.random.default_rng(6)
    gots, refs = [], []
    for b in (0, B - 1):
        rows = np.sort(np.concatenate([[0, S - 1], pick.choice(np.arange(1, S - 1), 2, replace=False)]))
        refs.append(oracle.block_rows(xin[b], wv, H, rows, threads=THREADS))
        gots.append(got[b, rows])
    _check(np.concatenate(gots), np.concatenate(refs))
    assert np.isfinite(got).all()
