"""Tensor-parallel transformer block over the GPUs of one box (config 5).

The reference runs its transformer-block graph on one IPU device; scaling it
over GPUs is Megatron-style tensor parallelism: the QKV projections are split
by columns (whole heads per rank), attention is head-local, the output
projection is split by rows, the MLP up-projection by columns and the
down-projection by rows, so each rank ends each half of the block with a
partial sum of the full activation and one all-reduce per half combines them.
The residual adds are folded into rank 0's partial sum (its GEMM epilogue adds
the residual), so each all-reduce yields the residual sum directly.

Compute is the library's kernels (ipuc_gemm_f16 with the fused GELU/accumulate
epilogues, and ipuc_flash_attention_heads_f16 reading the local heads straight
out of the QKV projections); the all-reduce is NCCL through torch.distributed.
The shard planning (`plan`) is plain host logic, tested on CPU.
"""

from __future__ import annotations

from dataclasses import dataclass

from . import GEMM_EPILOGUE_GELU, F16, call


@dataclass(frozen=True)
class Shard:
    """One rank's slice of the block's weights (half-open column/row ranges)."""
    heads: tuple          # local heads [h0, h1)
    qkv_cols: tuple       # columns of Wq/Wk/Wv, rows of Wo: [h0 * dh, h1 * dh)
    ff_cols: tuple        # columns of W1, rows of W2
    adds_residual: bool   # rank 0 adds the residual into its partial sums


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


class TensorParallelBlock:
    """y = h + W2^T GELU(W1^T h), h = x + Wo^T attn(x Wq, x Wk, x Wv), with this
    rank's shard of every weight resident on its GPU (f16, row-major [in, out])."""

    def __init__(self, batch: int, seq: int, d: int, heads: int, ff: int, rank: int, world: int, group=None):
        import torch
        self.torch = torch
        self.B, self.S, self.d, self.H, self.ff = batch, seq, d, heads, ff
        self.rank, self.world, self.group = rank, world, group
        self.shard = plan(d, heads, ff, rank, world)
        self.dh = d // heads
        self.hl = self.shard.heads[1] - self.shard.heads[0]
        self.dl = self.hl * self.dh
        self.fl = self.shard.ff_cols[1] - self.shard.ff_cols[0]
        dev = torch.device("cuda", torch.cuda.current_device())
        f16 = torch.float16
        T = batch * seq
        e = lambda *shape: torch.empty(shape, dtype=f16, device=dev)
        self.wq, self.wk, self.wv = e(d, self.dl), e(d, self.dl), e(d, self.dl)
        self.wo, self.w1, self.w2 = e(self.dl, d), e(d, self.fl), e(self.fl, d)
        self.qf, self.kf, self.vf = e(T, self.dl), e(T, self.dl), e(T, self.dl)
        self.a = e(T, self.dl)
        self.h, self.u, self.y = e(T, d), e(T, self.fl), e(T, d)

    def load(self, weights: dict) -> None:
        """Copy this rank's shard out of full f16 torch tensors wq, wk, wv, wo
        ([d, d]), w1 ([d, ff]) and w2 ([ff, d]) on any device."""
        c0, c1 = self.shard.qkv_cols
        f0, f1 = self.shard.ff_cols
        self.wq.copy_(weights["wq"][:, c0:c1])
        self.wk.copy_(weights["wk"][:, c0:c1])
        self.wv.copy_(weights["wv"][:, c0:c1])
        self.wo.copy_(weights["wo"][c0:c1, :])
        self.w1.copy_(weights["w1"][:, f0:f1])
        self.w2.copy_(weights["w2"][f0:f1, :])

    def _gemm(self, c, a, b, m, n, k, flags, s, addend=None):
        if addend is None:
            call("ipuc_gemm_f16", c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k, n, n, flags, s)
        else:  # the epilogue adds `addend` (the residual): no copy
            call("ipuc_gemm_f16_addend", c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k, n, n, flags,
                 addend.data_ptr(), n, s)

    def _all_reduce(self, t):
        import torch.distributed as dist
        if self.world > 1:
            dist.all_reduce(t, group=self.group)

    def forward(self, x, chunks: int = 1):
        """x: [B*S, d] f16 on this GPU (the same on every rank); returns y
        ([B*S, d], complete on every rank).

        chunks > 1 (N > 1 only) pipelines the two row-split projections with
        their all-reduces: the output projection and the MLP run in `chunks`
        row blocks, each block's all-reduce is issued on a side stream as
        soon as its GEMM is done, and the next block's GEMMs run meanwhile;
        the MLP of a block waits only for that block's reduced rows."""
        torch = self.torch
        cur = torch.cuda.current_stream()
        s = cur.cuda_stream
        T, d = self.B * self.S, self.d
        for w, out in ((self.wq, self.qf), (self.wk, self.kf), (self.wv, self.vf)):
            self._gemm(out, x, w, T, self.dl, d, 0, s)
        # Local heads read in place from [B, S, hl * dh] and written merged.
        call("ipuc_flash_attention_heads_f16", self.a.data_ptr(), F16, self.qf.data_ptr(), self.kf.data_ptr(),
             self.vf.data_ptr(), self.B, self.hl, self.S, self.S, self.dh, 0.0, s)
        res = self.shard.adds_residual
        if chunks <= 1 or self.world == 1 or T % chunks:
            # h = x + sum over ranks of a_r Wo_r (rank 0's epilogue adds x).
            self._gemm(self.h, self.a, self.wo, T, d, self.dl, 0, s, x if res else None)
            self._all_reduce(self.h)
            # y = h + sum over ranks of GELU(h W1_r) W2_r.
            self._gemm(self.u, self.h, self.w1, T, self.fl, d, GEMM_EPILOGUE_GELU, s)
            self._gemm(self.y, self.u, self.w2, T, d, self.fl, 0, s, self.h if res else None)
            self._all_reduce(self.y)
            return self.y
        import torch.distributed as dist
        if getattr(self, "_comm", None) is None:
            self._comm = torch.cuda.Stream()
        comm = self._comm
        rows = T // chunks
        blocks = [slice(i * rows, (i + 1) * rows) for i in range(chunks)]

        def reduce_async(t):
            ev = torch.cuda.Event()
            ev.record(cur)
            comm.wait_event(ev)
            with torch.cuda.stream(comm):
                return dist.all_reduce(t, group=self.group, async_op=True)

        reduced_h = []
        for r in blocks:
            self._gemm(self.h[r], self.a[r], self.wo, rows, d, self.dl, 0, s, x[r] if res else None)
            reduced_h.append(reduce_async(self.h[r]))
        reduced_y = []
        for r, work in zip(blocks, reduced_h):
            work.wait()   # the compute stream waits for this block's reduced h
            self._gemm(self.u[r], self.h[r], self.w1, rows, self.fl, d, GEMM_EPILOGUE_GELU, s)
            self._gemm(self.y[r], self.u[r], self.w2, rows, d, self.fl, 0, s, self.h[r] if res else None)
            reduced_y.append(reduce_async(self.y[r]))
        for work in reduced_y:
            work.wait()
        return self.y

    @property
    def flop(self) -> float:
        """Algorithmic FLOP of the whole block (all ranks together)."""
        T, d, ff = self.B * self.S, self.d, self.ff
        return 2.0 * T * d * d * 4 + 4.0 * self.B * self.H * self.S * self.S * self.dh + 2 * 2.0 * T * d * ff
