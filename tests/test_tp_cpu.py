"""Host logic of the tensor-parallel transformer block on CPU: the Megatron
shard plan (ipuc.tp.plan) and, on two gloo ranks, that summing the per-rank
partial products with the residual folded into rank 0 reproduces the
unsharded block (numpy arithmetic in f32, in this test only)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ipuc.tp import plan


def test_plan_tiles_heads_and_ff():
    d, H, ff, world = 4096, 32, 16384, 8
    shards = [plan(d, H, ff, r, world) for r in range(world)]
    assert [s.heads for s in shards] == [(4 * r, 4 * r + 4) for r in range(world)]
    assert [s.qkv_cols for s in shards] == [(512 * r, 512 * r + 512) for r in range(world)]
    assert [s.ff_cols for s in shards] == [(2048 * r, 2048 * r + 2048) for r in range(world)]
    assert [s.adds_residual for s in shards] == [True] + [False] * 7


def test_plan_rejects_uneven_split():
    with pytest.raises(ValueError):
        plan(4096, 32, 16384, 0, 3)
    with pytest.raises(ValueError):
        plan(4096, 32, 16384, 2, 2)


def gelu(x):
    return 0.5 * x * (1.0 + np.tanh(0.7978846 * (x + 0.044715 * x ** 3)))


def attention(q, k, v):
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(q.shape[-1])
    s = np.exp(s - s.max(axis=-1, keepdims=True))
    return (s / s.sum(axis=-1, keepdims=True)) @ v


def heads_attention(x, wq, wk, wv, heads, dh):
    T = x.shape[0]
    split = lambda m: (x @ m).reshape(T, heads, dh).transpose(1, 0, 2)
    a = attention(split(wq), split(wk), split(wv))
    return a.transpose(1, 0, 2).reshape(T, heads * dh)


def full_block(x, w, H):
    dh = x.shape[1] // H
    h = x + heads_attention(x, w["wq"], w["wk"], w["wv"], H, dh) @ w["wo"]
    return h + gelu(h @ w["w1"]) @ w["w2"]


def _worker(rank, world, port, out, d, H, ff):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        T = 24
        x = rng.standard_normal((T, d)).astype(np.float32)
        w = {n: (rng.standard_normal(s) * 0.1).astype(np.float32)
             for n, s in [("wq", (d, d)), ("wk", (d, d)), ("wv", (d, d)), ("wo", (d, d)), ("w1", (d, ff)),
                          ("w2", (ff, d))]}
        sh = plan(d, H, ff, rank, world)
        c0, c1 = sh.qkv_cols
        f0, f1 = sh.ff_cols
        hl, dh = sh.heads[1] - sh.heads[0], d // H
        a = heads_attention(x, w["wq"][:, c0:c1], w["wk"][:, c0:c1], w["wv"][:, c0:c1], hl, dh)
        h = torch.from_numpy(a @ w["wo"][c0:c1, :] + (x if sh.adds_residual else 0))
        dist.all_reduce(h)
        h = h.numpy()
        y = torch.from_numpy(gelu(h @ w["w1"][:, f0:f1]) @ w["w2"][f0:f1, :] + (h if sh.adds_residual else 0))
        dist.all_reduce(y)
        ref = full_block(x, w, H)
        out.put((rank, float(np.abs(y.numpy() - ref).max()), float(np.abs(ref).max())))
    finally:
        dist.destroy_process_group()


def test_sharded_block_sums_to_unsharded_block_gloo():
    world, d, H, ff = 2, 64, 4, 128
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, d, H, ff)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, err, scale in res:
        assert err <= 1e-5 * scale


def test_graph_shard_matches_closed_form_plan():
    """The sharded session's split, derived from the block's graph, is the
    closed-form Megatron plan (ipuc.tp.plan) at every rank."""
    from ipuc.tp import block_graph
    d, H, ff = 1024, 16, 4096
    g, x, w, y = block_graph(2, 128, d, H, ff)
    for world in (2, 4, 8):
        for rank in range(world):
            sh = plan(d, H, ff, rank, world)
            sl = {v["graph_value"]: v for v in g.shard(rank, world)["values"] if v["kind"] == 1}
            for n in ("wq", "wk", "wv"):
                assert (sl[w[n]]["slice"], tuple(sl[w[n]]["range"])) == ("columns", sh.qkv_cols)
            assert (sl[w["wo"]]["slice"], tuple(sl[w["wo"]]["range"])) == ("rows", sh.qkv_cols)
            assert (sl[w["w1"]]["slice"], tuple(sl[w["w1"]]["range"])) == ("columns", sh.ff_cols)
            assert (sl[w["w2"]]["slice"], tuple(sl[w["w2"]]["range"])) == ("rows", sh.ff_cols)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_all_reduce_steps_line_up_across_ranks(world):
    """The peer-memory all-reduce pairs every rank's buffers by the position of
    the all-reduce steps in each rank's plan (local value ids differ between
    ranks), so every rank's plan must hold the same all-reduces, in the same
    order, over the same shapes, with element counts the kernel accepts."""
    import re
    from ipuc.tp import block_graph
    g, _, _, _ = block_graph(4, 2048, 4096, 32, 16384)
    seqs = []
    for rank in range(world):
        steps = [ln for ln in g.plan(rank=rank, world=world).splitlines() if "all_reduce" in ln]
        seqs.append([re.sub(r"out=[lv]\d+", "out=", ln) for ln in steps])
    assert len(seqs[0]) == 2
    assert all(s == seqs[0] for s in seqs)
    for ln in seqs[0]:
        dims = [int(d) for d in re.search(r"\[([\d,]+)\]", ln).group(1).split(",")]
        assert int(np.prod(dims)) % (8 * world) == 0
