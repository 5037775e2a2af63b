"""Benchmark of the B200 operator-catalog hot path (one JSON line on rank 0).

Headline step (BASELINE.json metric "FP16 GEMM & flash-attn TFLOP/s"):
  * config 3  MLP up-projection: X[8192x4096] f16 ~N(0,1) times
    W[4096x16384] f16 ~N(0,1/4096), tanh-GELU fused into the GEMM epilogue,
    f16 out (ipuc_gemm_f16 with IPUC_GEMM_EPILOGUE_GELU);
  * config 4  flash attention: 8 x 32 streams, S=4096, D=128, Q/K/V ~N(0,1)
    f16, scale 1/sqrt(128), f16 out (ipuc_flash_attention_f16).
With N GPUs the GEMM is sharded along N (columns of W) and attention along
batch x heads (strong scaling: the total work is fixed); outputs stay sharded,
so no collective sits in the step.  value = algorithmic FLOP of the whole
step (1.0995e12 + 2.1990e12) / max-over-ranks device time.

Timing: W warm-up steps, then K timed steps bracketed by barrier +
synchronize, CUDA events on the launching stream.  Inputs (0.45 GB GEMM,
1 GB attention per step) exceed the 126 MB L2, so no flush is needed.

--impl reference times the reference's CPU evaluation of the same step on the
host cores (the oracle restatement of crates/ipu-tests/src/diagnostic.rs:
OpenBLAS SGEMM + scalar GELU, scalar attention loop) on a bounded sample.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "ipu-stack_b200"))

# ---- workload constants (BASELINE.json configs 3 and 4) ---------------------
MLP_M, MLP_K, MLP_N = 8192, 4096, 16384
ATT_B, ATT_H, ATT_S, ATT_D = 8, 32, 4096, 128
GEMM_FLOP = 2.0 * MLP_M * MLP_N * MLP_K                      # 1.0995e12
ATT_FLOP = 4.0 * ATT_B * ATT_H * ATT_S * ATT_S * ATT_D        # 2.1990e12
STEP_FLOP = GEMM_FLOP + ATT_FLOP
REARRANGE_ROWS, REARRANGE_COLS = 4096, 49152                  # 201M elements: config-5 weight tiles


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p.get("bf16_tflops", 1590.0), p.get("bf16_tflops_sustained", 1400.0), p.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML every 10 ms during the
    timed region (read-only queries; no GPU setting is changed).  The physical
    GPU index is taken from CUDA_VISIBLE_DEVICES when set."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"),
               ("hw_power_brake", "nvmlClocksEventReasonHwPowerBrakeSlowdown"))

    def __init__(self, device_index: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            try:
                device_index = int(vis.split(",")[device_index])
            except (ValueError, IndexError):
                pass
        self.device_index = device_index
        self.samples, self.reasons, self.sm_max = [], set(), None
        self._stop = threading.Event()
        self.error = None

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.device_index)
            self.sm_max = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        except Exception as e:  # pragma: no cover - reported in the JSON line
            self.error = f"nvml unavailable: {e}"
            return

        def loop():
            while not self._stop.is_set():
                try:
                    self.samples.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                    mask = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for name, attr in self.REASONS:
                        if mask & getattr(pynvml, attr):
                            self.reasons.add(name)
                except Exception as e:  # pragma: no cover
                    self.error = str(e)
                self._stop.wait(0.01)

        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()

    def stop(self):
        self._stop.set()
        if getattr(self, "thread", None):
            self.thread.join(timeout=2)
        out = {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.sm_max,
               "reasons": sorted(self.reasons), "samples": len(self.samples), "source": "nvml, 10 ms"}
        if self.error:
            out["error"] = self.error
        return out


def setup_dist(want_gpus: int):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def shard(total: int, world: int, rank: int):
    base = total // world
    return rank * base, base if rank < world - 1 else total - base * (world - 1)


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

def run_ours(args):
    import torch
    import ipuc

    rank, world, local = setup_dist(args.gpus)
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream()
    s = stream.cuda_stream
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)

    n0, nw = shard(MLP_N, world, rank)
    s0, ns = shard(ATT_B * ATT_H, world, rank)
    gx = torch.Generator(device=dev)
    gx.manual_seed(1234)  # X is one tensor for the whole job: the same on every rank
    x = torch.randn((MLP_M, MLP_K), generator=gx, device=dev, dtype=torch.float32).half()
    w = (torch.randn((MLP_K, nw), generator=g, device=dev, dtype=torch.float32) * (1.0 / 64.0)).half()
    y = torch.empty((MLP_M, nw), device=dev, dtype=torch.float16)
    q = torch.randn((ns, ATT_S, ATT_D), generator=g, device=dev, dtype=torch.float32).half()
    k = torch.randn((ns, ATT_S, ATT_D), generator=g, device=dev, dtype=torch.float32).half()
    v = torch.randn((ns, ATT_S, ATT_D), generator=g, device=dev, dtype=torch.float32).half()
    o = torch.empty((ns, ATT_S, ATT_D), device=dev, dtype=torch.float16)

    def gemm():
        ipuc.call("ipuc_gemm_f16", y.data_ptr(), x.data_ptr(), w.data_ptr(), MLP_M, nw, MLP_K, MLP_K, nw, nw,
                  ipuc.GEMM_EPILOGUE_GELU, s)

    def attn():
        ipuc.call("ipuc_flash_attention_f16", o.data_ptr(), ipuc.F16, q.data_ptr(), k.data_ptr(), v.data_ptr(), ns,
                  ATT_S, ATT_S, ATT_D, 0.0, s)

    def step():
        gemm()
        attn()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- headline timed region ----
    clocks = ClockSampler(local)
    clocks.start()
    barrier(world)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps + 1)]
    ev[0].record(stream)
    for i in range(args.steps):
        gemm()
        ev[2 * i + 1].record(stream)
        attn()
        ev[2 * i + 2].record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clock_info = clocks.stop()
    total_ms = ev[0].elapsed_time(ev[-1])
    gemm_ms = sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)) / args.steps
    attn_ms = sum(ev[2 * i + 1].elapsed_time(ev[2 * i + 2]) for i in range(args.steps)) / args.steps
    ipuc.device_status(stream)
    total_ms = max_over_ranks(total_ms, world)
    gemm_ms = max_over_ranks(gemm_ms, world)
    attn_ms = max_over_ranks(attn_ms, world)
    ms_per_step = total_ms / args.steps
    value = STEP_FLOP / (ms_per_step * 1e-3) / 1e12

    # ---- end to end through the C ABI with host buffers ----
    pin = lambda t: torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
    hx, hw, hq, hk, hv = pin(x), pin(w), pin(q), pin(k), pin(v)
    hy, ho = pin(y), pin(o)
    for h, d in ((hx, x), (hw, w), (hq, q), (hk, k), (hv, v)):
        h.copy_(d)
    torch.cuda.synchronize()

    # The step is pipelined over three streams: host->device copies (s_in),
    # the kernels (the bench stream) and device->host copies (s_out), chunked
    # so that each chunk's kernel starts when its inputs have landed and its
    # result leaves while later chunks are still arriving (PCIe is full duplex).
    # W goes first (every GEMM chunk reads all of it), then X in row chunks,
    # then Q/K/V in stream chunks.  One device buffer set serves every step:
    # a chunk's upload waits for the previous step's kernel on that chunk, and
    # a kernel waits for the previous step's read-back of its output chunk.
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    g_chunks = [(r, min(MLP_M, r + MLP_M // 4)) for r in range(0, MLP_M, MLP_M // 4)]
    a_step = max(1, ns // 8)
    a_chunks = [(c, min(ns, c + a_step)) for c in range(0, ns, a_step)]
    n_ch = len(g_chunks) + len(a_chunks)
    in_ev = [torch.cuda.Event() for _ in range(n_ch)]
    comp_ev = [torch.cuda.Event() for _ in range(n_ch)]
    out_ev = [torch.cuda.Event() for _ in range(n_ch)]
    w_ev = torch.cuda.Event()
    # X is replicated (every rank's GEMM shard reads all of it): at N>1 each rank
    # uploads a 1/N row slice of every chunk and an NCCL all-gather over NVLink
    # assembles the chunk, so each byte of X crosses PCIe once per step for the
    # whole job instead of once per rank.
    gather_x = world > 1 and not args.e2e_replicated_x and all((r1 - r0) % world == 0 for r0, r1 in g_chunks)
    if gather_x:
        import torch.distributed as dist

    def e2e_step():
        with torch.cuda.stream(s_in):
            s_in.wait_event(comp_ev[len(g_chunks) - 1])  # previous step's GEMMs are done with W
            w.copy_(hw, non_blocking=True)
            w_ev.record(s_in)
            for i, (r0, r1) in enumerate(g_chunks):
                s_in.wait_event(comp_ev[i])
                if gather_x:
                    # this rank uploads its 1/N of the chunk's rows; NVLink brings the rest
                    p = (r1 - r0) // world
                    a0 = r0 + rank * p
                    x[a0:a0 + p].copy_(hx[a0:a0 + p], non_blocking=True)
                    dist.all_gather_into_tensor(x[r0:r1], x[a0:a0 + p])
                else:
                    x[r0:r1].copy_(hx[r0:r1], non_blocking=True)
                in_ev[i].record(s_in)
            for j, (c0, c1) in enumerate(a_chunks):
                i = len(g_chunks) + j
                s_in.wait_event(comp_ev[i])
                q[c0:c1].copy_(hq[c0:c1], non_blocking=True)
                k[c0:c1].copy_(hk[c0:c1], non_blocking=True)
                v[c0:c1].copy_(hv[c0:c1], non_blocking=True)
                in_ev[i].record(s_in)
        stream.wait_event(w_ev)
        for i, (r0, r1) in enumerate(g_chunks):
            stream.wait_event(in_ev[i])
            stream.wait_event(out_ev[i])
            ipuc.call("ipuc_gemm_f16", y[r0].data_ptr(), x[r0].data_ptr(), w.data_ptr(), r1 - r0, nw, MLP_K, MLP_K,
                      nw, nw, ipuc.GEMM_EPILOGUE_GELU, s)
            comp_ev[i].record(stream)
        for j, (c0, c1) in enumerate(a_chunks):
            i = len(g_chunks) + j
            stream.wait_event(in_ev[i])
            stream.wait_event(out_ev[i])
            ipuc.call("ipuc_flash_attention_f16", o[c0].data_ptr(), ipuc.F16, q[c0].data_ptr(), k[c0].data_ptr(),
                      v[c0].data_ptr(), c1 - c0, ATT_S, ATT_S, ATT_D, 0.0, s)
            comp_ev[i].record(stream)
        with torch.cuda.stream(s_out):
            for i, (r0, r1) in enumerate(g_chunks):
                s_out.wait_event(comp_ev[i])
                hy[r0:r1].copy_(y[r0:r1], non_blocking=True)
                out_ev[i].record(s_out)
            for j, (c0, c1) in enumerate(a_chunks):
                i = len(g_chunks) + j
                s_out.wait_event(comp_ev[i])
                ho[c0:c1].copy_(o[c0:c1], non_blocking=True)
                out_ev[i].record(s_out)

    e2e_steps = max(1, min(args.steps, 5))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    s_out.wait_event(e0)
    for _ in range(e2e_steps):
        e2e_step()
    stream.wait_event(out_ev[-1])
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world)
    h2d = sum(t.numel() * t.element_size() for t in (hw, hq, hk, hv))
    h2d += hx.numel() * hx.element_size() // (world if gather_x else 1)
    d2h = sum(t.numel() * t.element_size() for t in (hy, ho))

    # ---- parity of the headline outputs against the oracle (outside the timing) ----
    parity = headline_parity(torch, rank, world, x, w, y, q, k, v, o, hy, ho)

    # ---- supplementary components (not in value) ----
    comps = {}
    peak_burst, peak_sus, hbm, peak_kind = load_peaks()
    if rank == 0:
        comps = measure_components(ipuc, torch, stream, hbm)
        parity["config5"] = comps["transformer_block"].pop("parity")
    if world == 1:
        parity["pass"] = parity_pass(parity)
    if world > 1:
        barrier(world)
        gather = gather_outputs(torch, world, y, o)
        tp = transformer_block_tp(torch, rank, world)
        tp_peer = ar = peer_error = None
        if world <= 8:
            # supplementary: a failure here (e.g. CUDA IPC refused) is reported, not fatal
            try:
                ar = all_reduce_compare(ipuc, torch, rank, world)
                tp_peer = transformer_block_tp(torch, rank, world, all_reduce="peer")
            except Exception as e:  # noqa: BLE001
                peer_error = repr(e)[:300]
                tp_peer = None
        if rank == 0:
            comps["gather_outputs"] = gather
            comps["transformer_block_tp"] = tp
            parity["config5_tp"] = tp.pop("parity")
            if peer_error is not None:
                comps["peer_all_reduce_error"] = peer_error
            if tp_peer is not None:
                comps["all_reduce_64MiB"] = ar
                comps["transformer_block_tp_peer"] = tp_peer
                parity["config5_tp_peer"] = tp_peer.pop("parity")
        parity["pass"] = all_ranks_true(parity_pass(parity), world)

    # ---- CPU baseline (oracle, bounded sample, rank 0 at N=1) ----
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_baseline(args.cpu_seconds)

    if rank == 0:
        dom = "flash_attention" if attn_ms >= gemm_ms else "gemm_f16_gelu"
        dom_ms = attn_ms if dom == "flash_attention" else gemm_ms
        dom_flop = (ATT_FLOP * ns / (ATT_B * ATT_H)) if dom == "flash_attention" else (GEMM_FLOP * nw / MLP_N)
        achieved = dom_flop / (dom_ms * 1e-3) / 1e12
        gemm_tf = GEMM_FLOP * nw / MLP_N / (gemm_ms * 1e-3) / 1e12
        attn_tf = ATT_FLOP * ns / (ATT_B * ATT_H) / (attn_ms * 1e-3) / 1e12
        if "shard8" in comps and world == 1:
            # the N=8 shards' per-GPU rate as a fraction of the full-size kernels' rate
            comps["shard8"]["gemm_f16_gelu"]["of_full"] = round(comps["shard8"]["gemm_f16_gelu"]["tflops"] / gemm_tf, 3)
            comps["shard8"]["flash_attention"]["of_full"] = round(comps["shard8"]["flash_attention"]["tflops"] / attn_tf,
                                                                  3)
        # The burst peak applies to a timed region shorter than the seconds-long
        # loop the sustained figure was measured with; 2 s or more of timed
        # work is held against the sustained (power-capped) peak.
        if total_ms >= 2000.0:
            peak, which, why = peak_sus, "sustained", f"timed region {total_ms / 1e3:.1f} s >= 2 s"
        else:
            peak, which, why = peak_burst, "burst", f"timed region {total_ms / 1e3:.2f} s < 2 s"
        line = {
            "metric": "FP16 GEMM (MLP up-proj, fused GELU) + flash-attention TFLOP/s",
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic (seeded N(0,1) / N(0,1/4096) f16, BASELINE shapes)",
            "config": step_config(world),
            "gpu_launches": (1 + attention_launches(torch, ns)) * args.steps,
            "clocks": clock_info,
            "e2e": {"value": round(STEP_FLOP / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "tensor", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_kind": f"{peak_kind} cuBLAS bf16 {which} ({why})",
                         "frac_of_burst": round(achieved / peak_burst, 4),
                         "frac_of_sustained": round(achieved / peak_sus, 4),
                         "traffic": profiled_traffic(dom, ns / (ATT_B * ATT_H) if dom == "flash_attention"
                                                     else nw / MLP_N)},
            "kernels": {"gemm_f16_gelu": {"ms": round(gemm_ms, 4), "tflops": round(gemm_tf, 1),
                                          "frac": round(gemm_tf / peak, 4)},
                        "flash_attention": {"ms": round(attn_ms, 4), "tflops": round(attn_tf, 1),
                                            "frac": round(attn_tf / peak, 4)},
                        "peak": f"{peak} TFLOP/s ({which})"},
            "components": comps,
            "parity": parity,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def all_ranks_true(ok: bool, world: int) -> bool:
    if world == 1:
        return bool(ok)
    return max_over_ranks(0.0 if ok else 1.0, world) == 0.0


def parity_pass(parity: dict) -> bool:
    return all(v.get("pass", False) for k, v in parity.items() if isinstance(v, dict))


def headline_parity(torch, rank, world, x, w, y, q, k, v, o, hy, ho):
    """Sampled check of the headline outputs against the oracle (the checker
    only; run after the timed regions).  Config 3: 128 rows of this rank's Y
    shard across all its columns against GELU(X W) evaluated on the host.
    Config 4: 4 of this rank's streams x 128 query rows against the scalar
    attention over all 4096 keys.  The same rows of the end-to-end outputs
    (host buffers) must equal the device outputs bit for bit.  Every rank checks
    its own shard; `pass` is true only if every rank passed."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    threads = max(1, (os.cpu_count() or 1) // world)
    rng = np.random.default_rng(99 + rank)
    t0 = time.perf_counter()
    rows = np.sort(rng.choice(y.shape[0], 128, replace=False))
    ri = torch.from_numpy(rows).to(y.device)
    got = y.index_select(0, ri).float().cpu().numpy()
    ref = oracle.mlp_rows(x.index_select(0, ri).float().cpu().numpy(), w.float().cpu().numpy())
    c3 = oracle.compare_f16(got, ref)
    c3.update(rows=128, columns=int(y.shape[1]), e2e_bitwise=bool(torch.equal(hy[torch.from_numpy(rows)],
                                                                               y.index_select(0, ri).cpu())))
    c3["pass"] = c3["pass"] and c3["e2e_bitwise"]
    streams = np.sort(rng.choice(o.shape[0], min(4, o.shape[0]), replace=False))
    qrows = np.sort(rng.choice(o.shape[1], 128, replace=False))
    si, qi = torch.from_numpy(streams).to(o.device), torch.from_numpy(qrows).to(o.device)
    got = o.index_select(0, si).index_select(1, qi).float().cpu().numpy()
    ref = oracle.attention(q.index_select(0, si).index_select(1, qi).float().cpu().numpy(),
                           k.index_select(0, si).float().cpu().numpy(), v.index_select(0, si).float().cpu().numpy(),
                           threads=threads)
    c4 = oracle.compare_f16(got, oracle.quantize_f16(ref))
    e2e_same = torch.equal(ho[torch.from_numpy(streams)][:, torch.from_numpy(qrows)],
                           o.index_select(0, si).index_select(1, qi).cpu())
    c4.update(streams=len(streams), query_rows=128, keys=int(k.shape[1]), e2e_bitwise=bool(e2e_same))
    c4["pass"] = c4["pass"] and c4["e2e_bitwise"]
    return {"config3": c3, "config4": c4, "checked_on": f"rank {rank} of {world} (each rank checks its shard)",
            "tolerance": "max|err| <= 2e-2 max|ref|, rel-L2 <= 5e-3 (f16); e2e outputs bitwise equal to device",
            "seconds": round(time.perf_counter() - t0, 1)}


def attention_launches(torch, streams: int) -> int:
    """Kernels one ipuc_flash_attention_f16 call launches at the bench shape:
    CTA-pair units of 512 query rows fill whole waves of sm/2 pair slots, and a
    tail of at most half a wave runs as a second (split-cluster) launch."""
    slots = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count // 2
    units = streams * ((ATT_S + 511) // 512)
    tail = units % slots
    split = tail > 0 and 4 * tail <= 2 * slots and (ATT_S + 127) // 128 >= 2
    return 2 if split and units > tail else 1


def profiled_traffic(kernel: str, share: float = 1.0):
    """DRAM bytes per launch from the committed ncu summary (captured on the
    full single-GPU launch), scaled to this rank's shard of the work, which
    traffic grows in proportion to; None without a summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            v = json.load(f).get(kernel)
        return None if v is None else int(round(v * share))
    return None


def measure_components(ipuc, torch, stream, hbm_gbs):
    """Layout-kernel GB/s (config-5 weight tiles), FP32 GEMM TFLOP/s (config 2) and
    the config-5 block, reported beside the headline, not folded into it."""
    s = stream.cuda_stream
    out = {}
    # Layout kernels on 201M f16 elements (4096 x 49152, the config-5 weight-tile
    # volume): row-major -> AMP-Left / AMP-TransposedRight / BlockMajor{64,16}
    # (rearrange_* codelets) and AMP-Output / AMP-TransposedLeft -> row-major
    # (unpack_amp_f16).  GB/s counts one read and one write of every element.
    n = REARRANGE_ROWS * REARRANGE_COLS
    R, C = REARRANGE_ROWS, REARRANGE_COLS
    src = torch.empty(n, dtype=torch.int16, device="cuda").random_(-30000, 30000)
    dst = torch.empty(n, dtype=torch.int16, device="cuda")
    layouts = [
        ("rearrange_amp_left", "ipuc_rearrange_f16", (dst.data_ptr(), src.data_ptr(), 1, R, R, 0, C, C, 64, 16, s)),
        ("rearrange_amp_transposed_right", "ipuc_rearrange_f16",
         (dst.data_ptr(), src.data_ptr(), 1, R, R, 1, C, C, 64, 16, s)),
        ("rearrange_block_major", "ipuc_rearrange_f16", (dst.data_ptr(), src.data_ptr(), 1, R, R, 2, C, C, 64, 16, s)),
        ("unpack_amp_output", "ipuc_unpack_f16", (dst.data_ptr(), src.data_ptr(), 0, 1, R, R, C, C, s)),
        ("unpack_amp_transposed_left", "ipuc_unpack_f16", (dst.data_ptr(), src.data_ptr(), 1, 1, R, R, C, C, s)),
    ]
    for name, fn, args in layouts:
        for _ in range(3):
            ipuc.call(fn, *args)
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record(stream)
        for _ in range(10):
            ipuc.call(fn, *args)
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / 10
        gbs = 2 * n * 2 / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm_gbs, 3)}
    del src, dst
    torch.cuda.empty_cache()
    # Config 3's unfused stages: split-K reduce of 4 fp32 partials -> f16
    # (4 x 512 MiB read + 256 MiB written) and standalone GELU (256 MiB each way).
    cnt = MLP_M * MLP_N
    parts = torch.randn((4, cnt), device="cuda", dtype=torch.float32)
    y16 = torch.empty(cnt, device="cuda", dtype=torch.float16)
    g16 = torch.empty(cnt, device="cuda", dtype=torch.float16)
    stages = [
        ("reduce_add_splitk4", 4 * cnt * 4 + cnt * 2,
         ("ipuc_reduce_sum", y16.data_ptr(), parts[0].data_ptr(), parts[1].data_ptr(), 3, cnt, ipuc.F32, s)),
        ("gelu_f16", 2 * cnt * 2, ("ipuc_gelu_f16", g16.data_ptr(), y16.data_ptr(), cnt, s)),
    ]
    for name, nbytes, args in stages:
        for _ in range(3):
            ipuc.call(*args)
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record(stream)
        for _ in range(10):
            ipuc.call(*args)
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / 10
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm_gbs, 3),
                     "bytes": nbytes}
    del parts, y16, g16
    # Config 5's residual Add (8192 x 4096 f16: two reads, one write) and a
    # Cast of the same activation f16 -> f32 (2 bytes read, 4 written).
    na = 8192 * 4096
    l16, r16 = (torch.randn(na, device="cuda").half() for _ in range(2))
    o16 = torch.empty(na, device="cuda", dtype=torch.float16)
    o32 = torch.empty(na, device="cuda", dtype=torch.float32)
    for name, nbytes, args in [
        ("add_f16", 3 * na * 2, ("ipuc_add_f16", o16.data_ptr(), l16.data_ptr(), r16.data_ptr(), na, 0, 0, s)),
        ("cast_f16_to_f32", na * 6, ("ipuc_cast", o32.data_ptr(), ipuc.F32, l16.data_ptr(), ipuc.F16, na, s)),
    ]:
        for _ in range(3):
            ipuc.call(*args)
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record(stream)
        for _ in range(10):
            ipuc.call(*args)
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / 10
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "frac_hbm": round(gbs / hbm_gbs, 3),
                     "bytes": nbytes}
    del l16, r16, o16, o32
    torch.cuda.empty_cache()
    # FP32 GEMM 4096^3 (3xF16 split)
    try:
        m = n_ = k = 4096
        a32 = torch.rand((m, k), device="cuda") * 2 - 1
        b32 = torch.rand((k, n_), device="cuda") * 2 - 1
        c32 = torch.empty((m, n_), device="cuda")
        ws = torch.empty(max(1, ipuc.gemm_f32_workspace_bytes(m, n_, k)), dtype=torch.uint8, device="cuda")

        def time32(flags):
            def run32():
                ipuc.call("ipuc_gemm_f32", c32.data_ptr(), a32.data_ptr(), b32.data_ptr(), m, n_, k, k, n_, n_,
                          flags, ws.data_ptr(), ws.numel(), s)
            for _ in range(3):
                run32()
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record(stream)
            for _ in range(10):
                run32()
            b.record(stream)
            torch.cuda.synchronize()
            return a.elapsed_time(b) / 10
        ms = time32(0)                                   # default: scaled 3xF16 split
        ms_tf32 = time32(ipuc.GEMM_F32_SPLIT_TF32)        # the classic 3xTF32 split, for comparison
        flop32 = 2 * m * n_ * k
        out["gemm_f32_4096"] = {"ms": round(ms, 4), "tflops": round(flop32 / (ms * 1e-3) / 1e12, 1),
                                "split": "3xF16 scaled",
                                "tflops_3xtf32": round(flop32 / (ms_tf32 * 1e-3) / 1e12, 1)}
    except ipuc.IpucError as e:
        out["gemm_f32_4096"] = {"unavailable": str(e)}
    del a32, b32, c32, ws
    torch.cuda.empty_cache()
    out["shard8"] = shard8_kernels(ipuc, torch, stream)
    out["gemm_f16_256"] = gemm_f16_small(ipuc, torch, stream)
    out["transformer_block"] = transformer_block(ipuc, torch, stream)
    return out


def shard8_kernels(ipuc, torch, stream):
    """The per-GPU shards of the headline step at N=8, timed on this GPU: the
    GEMM column shard 8192x2048x4096 + GELU (256 pair tiles on 74 pair slots:
    3.46 waves, the last one run as K halves) and the attention shard of 32
    streams (its tail as split clusters).  TFLOP/s per GPU, to set beside the
    full-size kernels' rates (kernels.*.tflops) as the N=8 per-GPU efficiency."""
    s = stream.cuda_stream
    m, n, k = MLP_M, MLP_N // 8, MLP_K
    x = torch.randn((m, k), device="cuda").half()
    w = (torch.randn((k, n), device="cuda") / 64).half()
    y = torch.empty((m, n), device="cuda", dtype=torch.float16)
    M = ATT_B * ATT_H // 8
    q, kk, v = (torch.randn((M, ATT_S, ATT_D), device="cuda").half() for _ in range(3))
    o = torch.empty_like(q)
    cases = {
        "gemm_f16_gelu": (2.0 * m * n * k, lambda: ipuc.call("ipuc_gemm_f16", y.data_ptr(), x.data_ptr(), w.data_ptr(),
                                                               m, n, k, k, n, n, ipuc.GEMM_EPILOGUE_GELU, s)),
        "flash_attention": (ATT_FLOP / 8, lambda: ipuc.call("ipuc_flash_attention_f16", o.data_ptr(), ipuc.F16,
                                                             q.data_ptr(), kk.data_ptr(), v.data_ptr(), M, ATT_S,
                                                             ATT_S, ATT_D, 0.0, s)),
    }
    out = {}
    for name, (flop, fn) in cases.items():
        for _ in range(3):
            fn()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record(stream)
        for _ in range(20):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / 20
        out[name] = {"ms": round(ms, 4), "tflops": round(flop / (ms * 1e-3) / 1e12, 1)}
    del x, w, y, q, kk, v, o
    torch.cuda.empty_cache()
    return out


def gemm_f16_small(ipuc, torch, stream):
    """Config 1: the FP16 GEMM at 256^3 (3.36e7 FLOP), a latency case.  200
    back-to-back launches on one stream (host launch rate included), and the same
    200 launches captured in one CUDA graph (device time per GEMM)."""
    m = n = k = 256
    a = (torch.randn((m, k), device="cuda") * 0.1).half()
    b = (torch.randn((k, n), device="cuda") * 0.1).half()
    c = torch.empty((m, n), device="cuda", dtype=torch.float16)
    reps = 200

    def run(s):
        for _ in range(reps):
            ipuc.call("ipuc_gemm_f16", c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k, n, n, 0, s)

    def timed(fn):
        e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / reps

    run(stream.cuda_stream)
    torch.cuda.synchronize()
    us = timed(lambda: run(stream.cuda_stream))
    res = {"us_per_gemm_stream": round(us, 2), "tflops_stream": round(2 * m * n * k / (us * 1e-6) / 1e12, 2)}
    try:
        side = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            run(side.cuda_stream)
        graph.replay()
        torch.cuda.synchronize()
        us_g = timed(graph.replay)
        res.update({"us_per_gemm_graph": round(us_g, 2),
                    "tflops_graph": round(2 * m * n * k / (us_g * 1e-6) / 1e12, 2)})
    except Exception as e:  # capture unsupported on this stack: keep the stream figure
        res["graph"] = f"unavailable: {type(e).__name__}: {e}"[:200]
    return res


def transformer_block(ipuc, torch, stream):
    """Config 5 lowered end to end through the ComputeGraph session on one GPU:
    batch 4 x seq 2048 (8192 tokens), d=4096, 32 heads of 128, MLP 4096->16384
    ->4096 with GELU, two residual adds; weights N(0, 0.02), f16."""
    import numpy as np
    from ipuc.graph import ComputeGraph, Session
    B, S, d, H, ff = 4, 2048, 4096, 32, 16384
    g = ComputeGraph()
    x = g.host_input("x", [B, S, d])
    w = {n: g.parameter(n, shp) for n, shp in [("wq", [d, d]), ("wk", [d, d]), ("wv", [d, d]), ("wo", [d, d]),
                                               ("w1", [d, ff]), ("w2", [ff, d])]}
    q = g.split_heads(g.gemm(x, w["wq"]), H)
    k = g.split_heads(g.gemm(x, w["wk"]), H)
    v = g.split_heads(g.gemm(x, w["wv"]), H)
    a = g.merge_heads(g.flash_attention(q, k, v), H)
    h = g.add(g.gemm(a, w["wo"]), x)
    y = g.add(g.gemm(g.gelu(g.gemm(h, w["w1"])), w["w2"]), h)
    g.set_outputs([y])
    sess = Session(g)
    rng = np.random.default_rng(5)
    xin = rng.standard_normal((B, S, d), dtype=np.float32)
    sess.write(x, xin)
    wv = {}
    for name, val in w.items():
        wv[name] = rng.standard_normal(g.value_shape(val), dtype=np.float32) * np.float32(0.02)
        sess.write(val, wv[name])
    flop = 2.0 * B * S * d * d * 4 + 4.0 * B * H * S * S * (d // H) + 2 * 2.0 * B * S * d * ff
    for _ in range(2):
        sess.run(stream)
    e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
    e0.record(stream)
    for _ in range(5):
        sess.run(stream)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / 5
    out = {"ms": round(ms, 4), "tflops": round(flop / (ms * 1e-3) / 1e12, 1), "flop": flop,
           "steps": sess.plan.count("\n")}
    # parity: 4 token rows of each of 2 batch elements against the oracle's
    # evaluation of the same graph restricted to those rows
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    t0 = time.perf_counter()
    got = sess.read(y).astype(np.float32)
    sess.close()
    pick = np.random.default_rng(6)
    gots, refs = [], []
    for b in (0, B - 1):
        rows = np.sort(pick.choice(S, 4, replace=False))
        refs.append(oracle.block_rows(xin[b], wv, H, rows, threads=os.cpu_count() or 8))
        gots.append(got[b, rows])
    par = oracle.compare_f16(np.concatenate(gots), np.concatenate(refs))
    par.update(token_rows=8, batches=[0, B - 1], seconds=round(time.perf_counter() - t0, 1))
    out["parity"] = par
    return out


def gather_outputs(torch, world, y, o):
    """The optional final exchange of the sharded step: NCCL all-gather of every
    rank's GEMM output columns and attention streams onto every GPU (over NVLink
    on one box).  Not part of the headline (consumers that are themselves
    sharded need no gather).  Device time, max over ranks; bus bandwidth
    (N-1)/N x gathered bytes / time."""
    import torch.distributed as dist
    gy = torch.empty((world,) + tuple(y.shape), dtype=y.dtype, device=y.device)
    go = torch.empty((world,) + tuple(o.shape), dtype=o.dtype, device=o.device)
    stream = torch.cuda.current_stream()

    def run():
        dist.all_gather_into_tensor(gy, y.contiguous())
        dist.all_gather_into_tensor(go, o.contiguous())
    for _ in range(3):
        run()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(5):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / 5, world)
    total = (gy.numel() + go.numel()) * gy.element_size()
    del gy, go
    return {"ms": round(ms, 4), "gathered_bytes": total,
            "bus_GB/s": round((world - 1) / world * total / (ms * 1e-3) / 1e9, 1), "collective": "NCCL all_gather"}


def transformer_block_tp(torch, rank, world, all_reduce="nccl"):
    """Config 5 over all ranks through the sharded graph session (ipuc.tp):
    the session derives the Megatron split from the block's graph (QKV and
    MLP-up by columns, output and MLP-down projections by rows, one NCCL
    all-reduce after each half; NCCL's, or with all_reduce="peer" the
    library's peer-memory kernel).  Device time, max over ranks; TFLOP/s of the
    whole block."""
    from ipuc.tp import TensorParallelBlock
    B, S, d, H, ff = 4, 2048, 4096, 32, 16384
    blk = TensorParallelBlock(B, S, d, H, ff, rank, world, all_reduce=all_reduce)
    g = torch.Generator(device="cuda")
    g.manual_seed(77)  # the same full weights and input on every rank
    full = {n: (torch.randn(shp, generator=g, device="cuda") * 0.02).half()
            for n, shp in [("wq", (d, d)), ("wk", (d, d)), ("wv", (d, d)), ("wo", (d, d)), ("w1", (d, ff)),
                           ("w2", (ff, d))]}
    blk.load(full)
    host_w = {n: t.float().cpu().numpy() for n, t in full.items()} if rank == 0 else None
    del full
    x = torch.randn((B * S, d), generator=g, device="cuda").half()
    stream = torch.cuda.current_stream()

    def timed():
        for _ in range(3):
            blk.forward(x)
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            blk.forward(x)
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / 5, world)

    ms = timed()
    # parity (rank 0; the output is complete on every rank): 4 token rows of
    # the first and last batch element against the oracle's evaluation of the
    # unsharded block
    par = None
    if rank == 0:
        import numpy as np
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        t0 = time.perf_counter()
        pick = np.random.default_rng(8)
        sel = [(b, np.sort(pick.choice(S, 4, replace=False))) for b in (0, B - 1)]
        xh = x.float().cpu().numpy().reshape(B, S, d)
        refs = np.concatenate([oracle.block_rows(xh[b], host_w, H, r, threads=os.cpu_count() or 8) for b, r in sel])
    yv = blk.forward(x)
    torch.cuda.synchronize()
    if rank == 0:
        yh = yv.float().cpu().numpy().reshape(B, S, d)
        par = oracle.compare_f16(np.concatenate([yh[b, r] for b, r in sel]), refs)
        par.update(token_rows=8, seconds=round(time.perf_counter() - t0, 1))
    barrier(world)
    return {"parity": par, "ms": round(ms, 4), "tflops": round(blk.flop / (ms * 1e-3) / 1e12, 1), "flop": blk.flop,
            "parallelism": f"tp{world}", "steps": blk.session.plan.count("\n") - 1,
            "collective": {"nccl": "2 NCCL all-reduces",
                           "peer": "2 peer-memory all-reduces (ipuc_peer_all_reduce_f16)"}[all_reduce] +
                          " of 64 MiB (f16) per block, derived from the graph by the sharded session"}


def all_reduce_compare(ipuc, torch, rank, world):
    """The block's all-reduce alone (64 MiB of f16, [8192, 4096]): NCCL's
    all_reduce against the library's peer-memory kernel on the same data.
    Device time per call, max over ranks; algorithmic bandwidth = bytes / time.
    Rank 0 checks the kernel's sum against NCCL's (bitwise at world 2, where
    both round the exact sum once; within one f16 ulp of the f32 sum above)."""
    import torch.distributed as dist
    g = torch.Generator(device="cuda")
    g.manual_seed(100 + rank)
    x = torch.randn((8192, 4096), generator=g, device="cuda").half()
    ref = x.clone()
    y = torch.empty_like(x)
    peer = ipuc.PeerAllReduce([x], [y])
    stream = torch.cuda.current_stream()

    def timed(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(10):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return max_over_ranks(e0.elapsed_time(e1) / 10, world)

    t_peer = timed(lambda: peer.reduce(0, stream.cuda_stream))
    ipuc.device_status(stream.cuda_stream)
    work = ref.clone()
    t_nccl = timed(lambda: dist.all_reduce(work.copy_(ref)))
    dist.all_reduce(ref)
    torch.cuda.synchronize()
    diff = (y.float() - ref.float()).abs()
    ulp = ref.float().abs().clamp(min=2.0 ** -14) * 2.0 ** -10
    same = bool(torch.equal(y, ref))
    within = bool((diff <= ulp).all())
    peer.close()
    nbytes = x.numel() * 2
    return {"bytes": nbytes, "peer_ms": round(t_peer, 4), "nccl_ms_incl_copy": round(t_nccl, 4),
            "peer_algbw_GB/s": round(nbytes / (t_peer * 1e-3) / 1e9, 1),
            "nccl_algbw_GB/s": round(nbytes / (t_nccl * 1e-3) / 1e9, 1),
            "bitwise_equal_nccl": same, "within_1ulp_of_nccl": within,
            "note": "the NCCL leg includes a 64 MiB device copy that restores its in-place input"}


# ---------------------------------------------------------------------------
# CPU legs (oracle = restatement of the reference's host evaluator)
# ---------------------------------------------------------------------------

class CpuSample:
    """The reference CPU path on a bounded sample of the step, scaled to the
    full step: GEMM+GELU on R rows of X against all of W (f32 OpenBLAS SGEMM on
    f16-quantised values, f16 rounding of each op result), and the scalar
    attention loop on `streams` streams x SQ query rows against all 4096 keys.
    `leg(seconds)` repeats both parts until each has run for about half of
    `seconds` and returns the full-step time implied by the per-row rates."""

    def __init__(self, threads: int):
        import numpy as np
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle
        self.oracle = oracle
        self.threads = threads
        self.R = 1024 if threads > 1 else 64
        self.SQ = 64 if threads > 1 else 16
        rng = np.random.default_rng(0)
        self.xs = oracle.quantize_f16(rng.standard_normal((self.R, MLP_K), dtype=np.float32))
        self.ws = oracle.quantize_f16(rng.standard_normal((MLP_K, MLP_N), dtype=np.float32) / 64)
        self.streams = max(1, threads)
        shape_q, shape_kv = (self.streams, self.SQ, ATT_D), (self.streams, ATT_S, ATT_D)
        self.q = oracle.quantize_f16(rng.standard_normal(shape_q, dtype=np.float32))
        self.k = oracle.quantize_f16(rng.standard_normal(shape_kv, dtype=np.float32))
        self.v = oracle.quantize_f16(rng.standard_normal(shape_kv, dtype=np.float32))

    def _limits(self):
        try:
            from threadpoolctl import threadpool_limits
            return threadpool_limits(self.threads)
        except ImportError:  # pragma: no cover
            import contextlib
            return contextlib.nullcontext()

    def _gemm(self):
        o = self.oracle
        o.quantize_f16(o.gelu(o.quantize_f16(o.gemm(self.xs, self.ws))))

    def _attn(self):
        self.oracle.attention(self.q, self.k, self.v, threads=self.threads)

    def leg(self, seconds: float):
        def rate(fn, budget):
            t0 = time.perf_counter()
            n = 0
            while True:
                fn()
                n += 1
                el = time.perf_counter() - t0
                if el >= budget:
                    return el / n, n, el
        with self._limits():
            g_s, g_n, g_el = rate(self._gemm, seconds / 2)
            a_s, a_n, a_el = rate(self._attn, seconds / 2)
        gemm_full = g_s * (MLP_M / self.R)
        att_full = a_s * (ATT_B * ATT_H * ATT_S) / (self.streams * self.SQ)
        full = gemm_full + att_full
        sample = (f"GEMM+GELU on {self.R} of {MLP_M} rows x{g_n} ({g_el:.1f} s), attention {self.streams} streams x "
                  f"{self.SQ} of {ATT_S} query rows x{a_n} ({a_el:.1f} s); {self.threads} threads; per-row rates "
                  f"scaled to the full step ({full:.0f} s)")
        return {"tflops": STEP_FLOP / full / 1e12, "full_step_s": full, "measured_s": g_el + a_el,
                "sample": sample}


def cpu_baseline(seconds_budget: float):
    """All host threads: three legs of seconds_budget/3 each (default 10 s),
    median reported; plus one 1-thread leg of the same length on a smaller
    sample."""
    threads = os.cpu_count() or 1
    leg_s = max(2.0, seconds_budget / 3)
    cs = CpuSample(threads)
    cs.leg(1.0)  # warm the BLAS thread pool and the pages
    legs = [cs.leg(leg_s) for _ in range(3)]
    med = sorted(legs, key=lambda r: r["tflops"])[1]
    one = CpuSample(1).leg(leg_s)
    return {"value": round(med["tflops"], 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": med["sample"] + "; median of 3 legs",
            "legs_tflops": [round(r["tflops"], 6) for r in legs],
            "single_core": {"value": round(one["tflops"], 6), "cores": 1, "sample": one["sample"]}}


def step_config(world: int) -> dict:
    """The workload both arms report (config 3 + config 4 of BASELINE.json)."""
    return {"workload": "config3 MLP up-proj 8192x4096x16384 +GELU fused, N-sharded; config4 flash "
                        "attention B=8 H=32 S=4096 D=128, sharded over batch*heads",
            "global_batch": MLP_M, "seq_len": ATT_S, "parallelism": f"shard{world}",
            "l2": "inputs larger than L2 (no flush)"}


def run_reference(args):
    """The reference arm: the reference's host evaluator (restated by the
    oracle) on all host cores.  Each step is one bounded sample leg, sized so
    that all K steps take about two minutes; `ms_per_step` is the measured
    wall time of a leg and `value` the median full-step rate it implies."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    steps = max(1, args.steps)
    leg_s = min(10.0, max(2.0, 120.0 / steps))
    cs = CpuSample(threads)
    for _ in range(max(1, min(args.warmup, 2))):
        cs.leg(1.0)  # warm-up (BLAS thread pool, page faults)
    t0 = time.perf_counter()
    legs = [cs.leg(leg_s) for _ in range(steps)]
    wall = time.perf_counter() - t0
    value = statistics.median(r["tflops"] for r in legs)
    line = {
        "metric": "FP16 GEMM (MLP up-proj, fused GELU) + flash-attention TFLOP/s",
        "impl": "reference",
        "value": round(value, 6),
        "unit": "TFLOP/s",
        "n_gpus": args.gpus,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(wall / steps * 1e3, 1),
        "full_step_ms_extrapolated": round(statistics.median(r["full_step_s"] for r in legs) * 1e3, 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 (f16-quantised operands)",
        "data": "synthetic",
        "config": step_config(args.gpus),
        "evaluator": "the reference's host evaluator restated (oracle port), on the host cores; each step is a "
                     "bounded sample of the step, value = median of the full-step rates the samples imply",
        "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": legs[len(legs) // 2]["sample"]},
        "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def attention_vendor_compare():
    """Config 4 through this library's attention and through torch's SDPA on its
    cuDNN backend (the vendor's sm100 attention), alternating 10-launch batches
    timed by CUDA events: a measured reference point for what the hardware
    sustains on this shape, printed as TFLOP/s per batch."""
    import torch
    import ipuc
    from torch.nn.attention import SDPBackend, sdpa_kernel
    torch.cuda.set_device(0)
    s = torch.cuda.current_stream().cuda_stream
    B, H, S, D = ATT_B, ATT_H, ATT_S, ATT_D
    q, k, v = (torch.randn((B, H, S, D), device="cuda").half() for _ in range(3))
    o = torch.empty_like(q)
    flop = 4.0 * B * H * S * S * D
    ours = lambda: ipuc.call("ipuc_flash_attention_f16", o.data_ptr(), ipuc.F16, q.data_ptr(), k.data_ptr(),
                             v.data_ptr(), B * H, S, S, D, 0.0, s)

    def vendor():
        with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
            torch.nn.functional.scaled_dot_product_attention(q, k, v)

    rates = {"ipuc": [], "cudnn": []}
    for _ in range(3):
        ours(), vendor()
    for _ in range(4):
        for name, fn in (("ipuc", ours), ("cudnn", vendor)):
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            for _ in range(10):
                fn()
            b.record()
            torch.cuda.synchronize()
            rates[name].append(round(flop * 10 / (a.elapsed_time(b) * 1e-3) / 1e12, 1))
    print(json.dumps({"case": "attention_vendor", "tflops": rates}))


def gemm_vendor_compare():
    """Config 3's GEMM (8192x4096 . 4096x16384, f16) through this library (GELU
    fused, and without the epilogue) and through torch.matmul (cuBLAS, no GELU),
    alternating 10-launch batches timed by CUDA events, TFLOP/s per batch."""
    import torch
    import ipuc
    torch.cuda.set_device(0)
    s = torch.cuda.current_stream().cuda_stream
    m, n, k = MLP_M, MLP_N, MLP_K
    a = torch.randn((m, k), device="cuda").half()
    b = (torch.randn((k, n), device="cuda") / 64).half()
    c = torch.empty((m, n), device="cuda", dtype=torch.float16)
    flop = 2.0 * m * n * k
    fns = {
        "ipuc_gelu": lambda: ipuc.call("ipuc_gemm_f16", c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k, n, n,
                                       ipuc.GEMM_EPILOGUE_GELU, s),
        "ipuc": lambda: ipuc.call("ipuc_gemm_f16", c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k, n, n, 0, s),
        "cublas": lambda: torch.matmul(a, b, out=c),
    }
    rates = {name: [] for name in fns}
    for fn in fns.values():
        for _ in range(3):
            fn()
    for _ in range(4):
        for name, fn in fns.items():
            e0, e1 = torch.cuda.Event(True), torch.cuda.Event(True)
            e0.record()
            for _ in range(10):
                fn()
            e1.record()
            torch.cuda.synchronize()
            rates[name].append(round(flop * 10 / (e0.elapsed_time(e1) * 1e-3) / 1e12, 1))
    print(json.dumps({"case": "gemm_vendor", "tflops": rates}))


def profile_case(kernel: str):
    """One kernel at the exact shape the headline step launches it with (at most
    ~1.3 GB on the device), for ncu captures: 1 warm-up + 3 launches."""
    import torch
    import ipuc
    if kernel == "attention_vendor":
        attention_vendor_compare()
        return
    if kernel == "gemm_vendor":
        gemm_vendor_compare()
        return
    torch.cuda.set_device(0)
    s = torch.cuda.current_stream().cuda_stream
    if kernel == "gemm":
        m, n, k = MLP_M, MLP_N, MLP_K
        a = torch.randn((m, k), device="cuda").half()
        b = (torch.randn((k, n), device="cuda") / 64).half()
        c = torch.empty((m, n), device="cuda", dtype=torch.float16)
        run = lambda: ipuc.call("ipuc_gemm_f16", c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k, n, n,
                                ipuc.GEMM_EPILOGUE_GELU, s)
    elif kernel in ("attention", "attention8"):
        # attention8: the 8-GPU shard (32 streams), whose tail runs as split clusters.
        M = ATT_B * ATT_H if kernel == "attention" else ATT_B * ATT_H // 8
        q, kk, v = (torch.randn((M, ATT_S, ATT_D), device="cuda").half() for _ in range(3))
        o = torch.empty_like(q)
        run = lambda: ipuc.call("ipuc_flash_attention_f16", o.data_ptr(), ipuc.F16, q.data_ptr(), kk.data_ptr(),
                                v.data_ptr(), M, ATT_S, ATT_S, ATT_D, 0.0, s)
    elif kernel in ("rearrange", "rearrange_amp_left"):
        rows, cols = REARRANGE_ROWS, REARRANGE_COLS
        src = torch.empty(rows * cols, dtype=torch.int16, device="cuda").random_(-30000, 30000)
        dst = torch.empty_like(src)
        target = 2 if kernel == "rearrange" else 0
        run = lambda: ipuc.call("ipuc_rearrange_f16", dst.data_ptr(), src.data_ptr(), 1, rows, rows, target, cols,
                                cols, 64, 16, s)
    elif kernel in ("reduce", "gelu"):
        # config 3's unfused stages: split-K reduce of 4 fp32 partials (2.42 GB
        # on the device) and standalone GELU on the reduced 134M elements
        cnt = MLP_M * MLP_N
        parts = torch.randn((4, cnt), device="cuda")
        y16 = torch.empty(cnt, device="cuda", dtype=torch.float16)
        if kernel == "reduce":
            run = lambda: ipuc.call("ipuc_reduce_sum", y16.data_ptr(), parts[0].data_ptr(), parts[1].data_ptr(), 3,
                                    cnt, ipuc.F32, s)
        else:
            del parts
            y16.normal_()
            g16 = torch.empty_like(y16)
            run = lambda: ipuc.call("ipuc_gelu_f16", g16.data_ptr(), y16.data_ptr(), cnt, s)
    elif kernel == "cast":
        # config 5's activation (8192 x 4096) f16 -> f32
        na = 8192 * 4096
        x16 = torch.randn(na, device="cuda").half()
        x32 = torch.empty(na, device="cuda")
        run = lambda: ipuc.call("ipuc_cast", x32.data_ptr(), ipuc.F32, x16.data_ptr(), ipuc.F16, na, s)
    elif kernel == "gemm_small":
        # config 1: 256^3 FP16 GEMM (the latency kernel)
        m = n = k = 256
        a = (torch.randn((m, k), device="cuda") * 0.1).half()
        b = (torch.randn((k, n), device="cuda") * 0.1).half()
        c = torch.empty((m, n), device="cuda", dtype=torch.float16)
        run = lambda: ipuc.call("ipuc_gemm_f16", c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k, n, n, 0, s)
    else:
        m = n = k = 4096
        a = torch.rand((m, k), device="cuda")
        b = torch.rand((k, n), device="cuda")
        c = torch.empty((m, n), device="cuda")
        ws = torch.empty(max(1, ipuc.gemm_f32_workspace_bytes(m, n, k)), dtype=torch.uint8, device="cuda")
        run = lambda: ipuc.call("ipuc_gemm_f32", c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, k, n, n, 0,
                                ws.data_ptr(), ws.numel(), s)
    for _ in range(4):
        run()
    torch.cuda.synchronize()
    ipuc.device_status()
    print(f"profile case {kernel}: ok")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the cpu_baseline leg")
    ap.add_argument("--e2e-replicated-x", action="store_true",
                    help="at N>1 every rank uploads all of X in the e2e step (no NVLink all-gather)")
    ap.add_argument("--cpu-seconds", type=float, default=30.0,
                    help="CPU baseline budget: three all-core legs of a third each, plus a 1-core leg")
    ap.add_argument("--profile", choices=["gemm", "attention", "attention8", "rearrange", "rearrange_amp_left",
                                          "gemm_f32", "reduce", "gelu", "cast", "gemm_small", "attention_vendor",
                                          "gemm_vendor"],
                    help="run a few launches of one kernel on a small case (for ncu captures) and exit")
    args = ap.parse_args()
    if args.profile:
        profile_case(args.profile)
        return
    if args.warmup < 3 and args.impl == "ours":
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
