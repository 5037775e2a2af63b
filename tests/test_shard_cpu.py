"""Per-GPU shard derivation from the graph (ipug_graph_plan_ex /
ipug_graph_shard_json), on the host: the Megatron split of the config-5 block
read off the graph (column-split QKV and MLP-up weights, head-local attention,
row-split output and MLP-down weights, one NCCL all-reduce per half), and on
gloo ranks that the per-rank shards evaluated with the oracle's ops and summed
by the collectives reproduce the unsharded evaluation."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from conftest import f16_close
from ipuc.graph import ComputeGraph


def block(B, S, d, H, ff):
    g = ComputeGraph()
    x = g.host_input("x", [B, S, d])
    w = {n: g.parameter(n, s) for n, s in [("wq", [d, d]), ("wk", [d, d]), ("wv", [d, d]), ("wo", [d, d]),
                                           ("w1", [d, ff]), ("w2", [ff, d])]}
    q, k, v = (g.split_heads(g.gemm(x, w[n]), H) for n in ("wq", "wk", "wv"))
    a = g.merge_heads(g.flash_attention(q, k, v), H)
    h = g.add(g.gemm(a, w["wo"]), x)
    y = g.add(g.gemm(g.gelu(g.gemm(h, w["w1"])), w["w2"]), h)
    g.set_outputs([y])
    return g, x, w, y


def labels(plan):
    return [line.split()[0] for line in plan.strip().splitlines() if not line.startswith("#")]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_block_shard_plan(world):
    g, x, w, y = block(4, 2048, 4096, 32, 16384)
    for rank in range(world):
        plan = g.plan(rank, world)
        assert plan.startswith(f"# rank {rank} of {world}")
        want = ["gemm_f16"] * 3 + ["flash_attention_heads_f16"]
        # rank 0's output projection epilogue adds the residual x (the other
        # ranks' GEMMs yield plain partial sums); the MLP-down epilogue adds
        # every rank's partial sum of h, so the all-reduce yields h + MLP(h)
        want += ["gemm_f16+add" if rank == 0 else "gemm_f16", "nccl_all_reduce", "gemm_f16+gelu",
                 "gemm_f16+add", "nccl_all_reduce"]
        assert labels(plan) == want, plan
        desc = g.shard(rank, world)
        sl = {v["graph_value"]: v for v in desc["values"] if v["kind"] == 1}
        d, ff = 4096, 16384
        for n in ("wq", "wk", "wv"):
            assert sl[w[n]]["slice"] == "columns" and sl[w[n]]["range"] == [rank * d // world, (rank + 1) * d // world]
        assert sl[w["w1"]]["slice"] == "columns" and sl[w["w1"]]["shape"] == [d, ff // world]
        assert sl[w["wo"]]["slice"] == "rows" and sl[w["wo"]]["shape"] == [d // world, d]
        assert sl[w["w2"]]["slice"] == "rows" and sl[w["w2"]]["range"] == [rank * ff // world, (rank + 1) * ff // world]
        states = [desc["values"][op["result"]]["state"] for op in desc["ops"]]
        assert states.count("partial") >= 2 and [o["kind"] for o in desc["ops"]].count("all_reduce") == 2


def test_world_one_is_the_single_gpu_plan():
    g, *_ = block(2, 64, 256, 4, 512)
    assert g.plan(0, 1) == g.plan()


def test_heads_that_do_not_divide_keep_attention_replicated():
    """3 heads over 2 GPUs: the attention half runs replicated (whole QKV and
    output weights, no collective); the MLP half still splits (one all-reduce)."""
    g, x, w, y = block(2, 64, 192, 3, 512)
    plan = g.plan(1, 2)
    assert labels(plan).count("nccl_all_reduce") == 1
    desc = g.shard(1, 2)
    sl = {v["graph_value"]: v for v in desc["values"] if v["kind"] == 1}
    for n in ("wq", "wk", "wv", "wo"):
        assert "slice" not in sl[w[n]]
    assert sl[w["w1"]]["slice"] == "columns" and sl[w["w2"]]["slice"] == "rows"
    # with no split at all (odd feed-forward width too) nothing is exchanged
    g2, *_ = block(2, 64, 192, 3, 501)
    assert "nccl" not in g2.plan(1, 2) and labels(g2.plan(1, 2)) == labels(g2.plan())


def test_column_split_output_is_gathered():
    """A column-split GEMM whose result is a graph output needs the whole value:
    it is computed replicated (no split is chosen for an output)."""
    g = ComputeGraph()
    x = g.host_input("x", [32, 64])
    y = g.gelu(g.gemm(x, g.parameter("w", [64, 128])))
    g.set_outputs([y])
    assert "nccl" not in g.plan(0, 2)
    # an MLP (up, GELU, down) splits and ends in one all-reduce
    g2 = ComputeGraph()
    x2 = g2.host_input("x", [32, 64])
    h = g2.gelu(g2.gemm(x2, g2.parameter("w1", [64, 128])))
    g2.set_outputs([g2.gemm(h, g2.parameter("w2", [128, 64]))])
    assert labels(g2.plan(1, 2)) == ["gemm_f16+gelu", "gemm_f16", "nccl_all_reduce"]


def _gloo_worker(rank, world, port, out, case):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from shard_eval import evaluate_shard
        rng = np.random.default_rng(17)
        if case == "block":
            B, S, d, H, ff = 2, 32, 64, 4, 128
            g, x, w, y = block(B, S, d, H, ff)
            inputs = {x: rng.standard_normal((B, S, d)).astype(np.float32)}
            for v in w.values():
                inputs[v] = (rng.standard_normal(g.value_shape(v)) * 0.1).astype(np.float32)
        else:  # MLP blocks in a Repeat over sequences of [1, k, n] weights (SiglipMlpBenchmark structure)
            from test_graph_cpu import mlp_repeat
            g, x, ups, downs, y = mlp_repeat(blocks=3, d=64, hidden=256)
            inputs = {x: rng.standard_normal(g.value_shape(x)).astype(np.float32)}
            for v in ups + downs:
                inputs[v] = (rng.standard_normal(g.value_shape(v)) * 0.1).astype(np.float32)

        def all_reduce(a):
            t = torch.from_numpy(np.array(a, dtype=np.float32))  # a copy: the input stays the partial sum
            dist.all_reduce(t)
            return t.numpy()

        def all_gather(a):
            t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32))
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            return [p.numpy() for p in parts]

        desc = g.shard(rank, world)
        got = evaluate_shard(desc, inputs, all_reduce, all_gather)[y]
        ref = oracle.evaluate(g, inputs, threads=2)[y]
        ok, msg = f16_close(got, ref)
        kinds = [o["kind"] for o in desc["ops"]]
        out.put((rank, ok, msg, kinds.count("all_reduce")))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case,world,reduces", [("block", 2, 2), ("block", 4, 2), ("mlp_repeat", 2, 3)])
def test_shards_reproduce_unsharded_evaluation_gloo(case, world, reduces):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q, case)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok, msg, n in res:
        assert ok, f"rank {rank}: {msg}"
        assert n == reduces


def test_sharded_session_arguments_checked_before_any_device_work():
    import ipuc
    from ipuc.graph import Session
    g, *_ = block(2, 64, 256, 4, 512)
    with pytest.raises(ipuc.IpucError) as e:
        Session(g, rank=0, world=2)            # no NCCL unique id
    assert e.value.status == ipuc.ERR_INVALID_ARGUMENT and "unique id" in str(e.value)
    with pytest.raises(ValueError, match="rank must lie"):
        g.plan(2, 2)                            # rank outside [0, world)
    with pytest.raises(ValueError, match="rank must lie"):
        g.shard(0, 0)
