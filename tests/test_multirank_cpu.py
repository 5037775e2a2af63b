"""World-size-2 gloo checks of bench.py's multi-rank host logic (shard ranges,
max-over-ranks timing) on CPU."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n0, nw = bench.shard(bench.MLP_N, world, rank)
        s0, ns = bench.shard(bench.ATT_B * bench.ATT_H, world, rank)
        t = bench.max_over_ranks(float(rank + 1) * 1.5, world)
        out.put((rank, n0, nw, s0, ns, t))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_shards_cover_and_max_over_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # column shards tile [0, N) and stream shards tile [0, B*H) exactly
    assert sum(r[2] for r in res) == bench.MLP_N and sum(r[4] for r in res) == bench.ATT_B * bench.ATT_H
    for a, b in zip(res, res[1:]):
        assert a[1] + a[2] == b[1] and a[3] + a[4] == b[3]
    assert all(r[5] == 1.5 * world for r in res)
