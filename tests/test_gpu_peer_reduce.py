"""Peer-memory all-reduce (ipuc_peer_all_reduce_f16) on two GPUs, one process
each: the kernel's f16 sum against the exactly rounded sum of the two ranks'
values and against NCCL's all_reduce, over several calls in a row (the
per-call counters of the signal area), in place and out of place, back to
back on the stream with the data changing between calls, and the
device error word clear afterwards.  The stand-in for ncclAllReduce in the
sharded session's row-split GEMMs; its sum is the reference's partial sum
(device/reduce_add_f16.S:31-72) over GPUs instead of tiles."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import ipuc
        msgs = []
        sizes = [16 * 1024 + 32, 3 * 1024 * 1024]  # a ragged per-CTA chunk; 6 MiB
        xs = [torch.empty(n, dtype=torch.half, device="cuda") for n in sizes]
        ys = [torch.empty_like(x) for x in xs]
        inplace = torch.empty(sizes[1], dtype=torch.half, device="cuda")
        ar = ipuc.PeerAllReduce(xs + [inplace], ys + [inplace])
        stream = torch.cuda.current_stream().cuda_stream
        for call in range(3):
            for i, n in enumerate(sizes):
                g = torch.Generator(device="cuda")
                g.manual_seed(1000 * call + 10 * i + rank)
                xs[i].copy_(torch.randn(n, generator=g, device="cuda").half() * (4.0 if call == 1 else 1.0))
                inplace.copy_(xs[1])
                ref = xs[i].clone()
                dist.all_reduce(ref)
                # the exact sum of every rank's values, rounded once
                parts = [torch.empty_like(xs[i]) for _ in range(world)]
                dist.all_gather(parts, xs[i])
                exact = torch.stack([p.double() for p in parts]).sum(0).half()
                dist.barrier()
                ar.reduce(i, stream)
                if i == 1:
                    ar.reduce(2, stream)
                torch.cuda.synchronize()
                if not torch.equal(ys[i], exact):
                    msgs.append(f"call {call} size {n}: not the rounded exact sum "
                                f"({int((ys[i] != exact).sum())} elements)")
                if world == 2 and not torch.equal(ys[i], ref):
                    msgs.append(f"call {call} size {n}: differs from NCCL")
                if i == 1 and not torch.equal(inplace, ys[1]):
                    msgs.append(f"call {call}: in-place result differs")
        # back to back on the stream with no host synchronisation, the data
        # changing between calls: a missing ordering between one call's stores
        # and the next call's reads shows up as the previous call's values
        seq = []
        for call in range(8):
            i = call % 2
            g = torch.Generator(device="cuda")
            g.manual_seed(7000 + 10 * call + rank)
            xs[i].copy_(torch.randn(sizes[i], generator=g, device="cuda").half())
            ar.reduce(i, stream)
            seq.append(ys[i].clone())
        torch.cuda.synchronize()
        for call in range(8):
            i = call % 2
            parts = []
            for r in range(world):
                g = torch.Generator(device="cuda")
                g.manual_seed(7000 + 10 * call + r)
                parts.append(torch.randn(sizes[i], generator=g, device="cuda").half())
            exact = torch.stack([p.double() for p in parts]).sum(0).half()
            if not torch.equal(seq[call], exact):
                msgs.append(f"back-to-back call {call}: {int((seq[call] != exact).sum())} elements differ")
        ipuc.device_status(stream)
        ar.close()
        q.put((rank, not msgs, "; ".join(msgs)))
    except Exception as e:  # reported through the queue
        q.put((rank, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_all_reduce_two_ranks():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, ok, msg in res:
        assert ok, f"rank {rank}: {msg}"
