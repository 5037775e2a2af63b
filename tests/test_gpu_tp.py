"""Tensor-parallel transformer block (ipuc.tp) against the oracle's evaluation
of the same ComputeGraph: one rank on one GPU, and two ranks over NCCL when
the box has two GPUs."""
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


def run_rank(rank, world, x, weights, chunks=1):
    from ipuc.tp import TensorParallelBlock
    blk = TensorParallelBlock(B, S, d, H, ff, rank, world)
    blk.load({n: torch.from_numpy(a).half() for n, a in weights.items()})
    y = blk.forward(torch.from_numpy(x).half().cuda(), chunks=chunks)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def test_tp_block_one_rank_matches_graph_oracle():
    x, weights, ref = block_inputs()
    got = run_rank(0, 1, x, weights)
    ok, msg = f16_close(got, ref)
    assert ok, msg


def _nccl_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        x, weights, ref = block_inputs()
        got = run_rank(rank, world, x, weights)
        # the row-chunked pipeline (all-reduce of each block overlapping the
        # next block's GEMMs) computes the same sums
        piped = run_rank(rank, world, x, weights, chunks=4)
        q.put((rank,) + f16_close(got, ref) + f16_close(piped, ref))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_tp_block_two_ranks_nccl():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok, msg, ok_piped, msg_piped in res:
        assert ok, f"rank {rank}: {msg}"
        assert ok_piped, f"rank {rank}, chunks=4: {msg_piped}"
