"""Tensor-parallel transformer block over the GPUs of one box (config 5), as a
client of the sharded graph session.

The block is written once as a ComputeGraph (QKV projections, SplitHeads ->
FlashAttention -> MergeHeads, output projection + residual, MLP up + GELU,
MLP down + residual) and every rank opens its shard of it
(ipug_session_open_ex with world > 1): the session derives the Megatron split
from the graph -- the QKV and MLP-up weights by columns (whole heads per
rank), attention head-local, the output and MLP-down weights by rows -- and
ends each half of the block with one NCCL all-reduce over the communicator it
owns.  `plan` states the same split in closed form (it is what the session
derives; the CPU tests check the two agree).
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    """One rank's slice of the block's weights (half-open column/row ranges)."""
    heads: tuple          # local heads [h0, h1)
    qkv_cols: tuple       # columns of Wq/Wk/Wv, rows of Wo: [h0 * dh, h1 * dh)
    ff_cols: tuple        # columns of W1, rows of W2
    adds_residual: bool   # rank 0 adds the residual x into its partial sum


def plan(d: int, heads: int, ff: int, rank: int, world: int) -> Shard:
    """Megatron split of a block with `heads` heads of d/heads channels."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank out of range")
    if heads % world or ff % world or d % heads:
        raise ValueError(f"heads ({heads}) and ff ({ff}) must divide by the world size ({world}); d by heads")
    dh = d // heads
    hl, fl = heads // world, ff // world
    h0 = rank * hl
    return Shard(heads=(h0, h0 + hl), qkv_cols=(h0 * dh, (h0 + hl) * dh), ff_cols=(rank * fl, (rank + 1) * fl),
                 adds_residual=rank == 0)


def block_graph(batch: int, seq: int, d: int, heads: int, ff: int):
    """The config-5 transformer block graph; returns (graph, x, weights, y)."""
    from .graph import ComputeGraph
    g = ComputeGraph()
    x = g.host_input("x", [batch, seq, d])
    w = {n: g.parameter(n, s) for n, s in [("wq", [d, d]), ("wk", [d, d]), ("wv", [d, d]), ("wo", [d, d]),
                                           ("w1", [d, ff]), ("w2", [ff, d])]}
    q, k, v = (g.split_heads(g.gemm(x, w[n]), heads) for n in ("wq", "wk", "wv"))
    a = g.merge_heads(g.flash_attention(q, k, v), heads)
    h = g.add(g.gemm(a, w["wo"]), x)
    y = g.add(g.gemm(g.gelu(g.gemm(h, w["w1"])), w["w2"]), h)
    g.set_outputs([y])
    return g, x, w, y


class TensorParallelBlock:
    """y = h + W2^T GELU(W1^T h), h = x + Wo^T attn(x Wq, x Wk, x Wv), one rank
    of a sharded graph session (this rank's weight slices resident on its GPU,
    f16, row-major [in, out]).  With world > 1, torch.distributed must be
    initialised: rank 0's NCCL unique id reaches the others through it.
    all_reduce "peer" runs the two all-reduces with the library's
    peer-memory kernel over NVLink instead of ncclAllReduce."""

    def __init__(self, batch: int, seq: int, d: int, heads: int, ff: int, rank: int, world: int, group=None,
                 all_reduce: str = "nccl"):
        import torch
        from .graph import Session, nccl_unique_id
        self.torch = torch
        self.B, self.S, self.d, self.H, self.ff = batch, seq, d, heads, ff
        self.rank, self.world = rank, world
        self.shard = plan(d, heads, ff, rank, world)
        self.dh = d // heads
        self.graph, self.x, self.w, self.y = block_graph(batch, seq, d, heads, ff)
        nccl_id = None
        if world > 1:
            import torch.distributed as dist
            box = [nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(box, src=0, group=group)
            nccl_id = box[0]
        self.session = Session(self.graph, device=torch.cuda.current_device(), rank=rank, world=world,
                               nccl_id=nccl_id)
        self.out = self.session.tensor(self.y, (batch * seq, d))
        if all_reduce not in ("nccl", "peer"):
            raise ValueError("all_reduce must be 'nccl' or 'peer'")
        if world > 1 and all_reduce == "peer":
            self.session.peer_reduce(True, torch.cuda.current_stream().cuda_stream)

    def load(self, weights: dict) -> None:
        """Copy this rank's slices out of full f16 torch tensors wq, wk, wv, wo
        ([d, d]), w1 ([d, ff]) and w2 ([ff, d]) on any device."""
        stream = self.torch.cuda.current_stream().cuda_stream
        for n, v in self.w.items():
            self.session.write_device(v, weights[n].contiguous(), stream)
        self.torch.cuda.current_stream().synchronize()

    def forward(self, x, chunks: int = 1):
        """x: [B*S, d] f16 on this GPU (the same on every rank); returns y
        ([B*S, d], complete on every rank; a view of the session's output
        buffer, rewritten by the next forward).  `chunks` is accepted for
        call compatibility; the session runs the block whole."""
        stream = self.torch.cuda.current_stream().cuda_stream
        self.session.write_device(self.x, x.contiguous(), stream)
        self.session.run(stream)
        return self.out

    @property
    def flop(self) -> float:
        """Algorithmic FLOP of the whole block (all ranks together)."""
        T, d, ff = self.B * self.S, self.d, self.ff
        return 2.0 * T * d * d * 4 + 4.0 * self.B * self.H * self.S * self.S * self.dh + 2 * 2.0 * T * d * ff
