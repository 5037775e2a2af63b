"""Tensor-parallel transformer block (ipuc.tp, a client of the sharded graph
session) against the oracle's evaluation of the same ComputeGraph: one rank on
one GPU, and two ranks over NCCL when the box has two GPUs; plus a sharded
session of a Repeat graph opened directly through ipug_session_open_ex."""
import os
import socket

import numpy as np
import pytest
import torch

import oracle
from conftest import f16_close
from test_gpu_graph import build_block

pytestmark = pytest.mark.gpu

B, S, d, H, ff = 2, 256, 512, 4, 1024


def block_inputs():
    g, x, ws, out = build_block(B, S, d, H, ff)
    rng = np.random.default_rng(21)
    inputs = {x: oracle.quantize_f16(rng.standard_normal((B, S, d)).astype(np.float32))}
    for n, v in ws.items():
        inputs[v] = oracle.quantize_f16((rng.standard_normal(g.value_shape(v)) * 0.02).astype(np.float32))
    ref = oracle.evaluate(g, inputs)[out].reshape(B * S, d)
    names = {v: n for n, v in ws.items()}
    weights = {names[v]: a for v, a in inputs.items() if v in names}
    return inputs[x].reshape(B * S, d), weights, ref


def run_rank(rank, world, x, weights, all_reduce="nccl"):
    from ipuc.tp import TensorParallelBlock
    blk = TensorParallelBlock(B, S, d, H, ff, rank, world, all_reduce=all_reduce)
    blk.load({n: torch.from_numpy(a).half() for n, a in weights.items()})
    y = blk.forward(torch.from_numpy(x).half().cuda())
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def test_tp_block_one_rank_matches_graph_oracle():
    x, weights, ref = block_inputs()
    got = run_rank(0, 1, x, weights)
    ok, msg = f16_close(got, ref)
    assert ok, msg


def _nccl_worker(rank, world, port, q, all_reduce="nccl"):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        x, weights, ref = block_inputs()
        got = run_rank(rank, world, x, weights, all_reduce)
        q.put((rank,) + f16_close(got, ref))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("all_reduce", ["nccl", "peer"])
def test_tp_block_two_ranks_nccl(all_reduce):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q, all_reduce)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok, msg in res:
        assert ok, f"rank {rank}: {msg}"


def _repeat_worker(rank, world, nccl_id, q):
    """One rank of a sharded session of the MLP-blocks Repeat graph, opened
    with the NCCL unique id the parent made (no torch.distributed at all)."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from ipuc.graph import Session
    from test_graph_cpu import mlp_repeat
    g, x, ups, downs, y = mlp_repeat(blocks=3, d=256, hidden=1024)
    rng = np.random.default_rng(3)
    inputs = {x: rng.standard_normal(g.value_shape(x)).astype(np.float32)}
    for v in ups + downs:
        inputs[v] = (rng.standard_normal(g.value_shape(v)) * 0.06).astype(np.float32)
    sess = Session(g, device=rank, rank=rank, world=world, nccl_id=nccl_id)
    for v, a in inputs.items():
        sess.write(v, a)
    sess.run()
    got = sess.read(y).astype(np.float32)
    plan = sess.plan
    sess.close()
    q.put((rank, plan.count("nccl_all_reduce")) + f16_close(got, oracle.evaluate(g, inputs)[y]))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_repeat_session_two_ranks():
    import torch.multiprocessing as mp
    from ipuc.graph import nccl_unique_id
    nccl_id = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_repeat_worker, args=(r, 2, nccl_id, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, reduces, ok, msg in res:
        assert reduces == 3, f"rank {rank}: {reduces} all-reduces"
        assert ok, f"rank {rank}: {msg}"
