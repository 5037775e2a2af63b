"""Cap'n Proto profile reports (ipug_profile_encode / ipuc.profile): CPU tests.

The reference writes `Profile` messages with the capnp crate
(crates/ipu-package/src/lib.rs:198-222).  No Cap'n Proto implementation is
installed here, so the golden test spells out the expected words from the
published encoding and the schema's field layout, independently of the
encoder; the rest are round trips through the library's encoder and the
Python reader, and the reader's checks (schema versions 1-5 only,
lib.rs:229-234).
"""
import struct

import numpy as np
import pytest

import ipuc
from ipuc import profile as P


def _words(data: bytes):
    assert len(data) % 8 == 0
    return list(struct.unpack(f"<{len(data) // 8}Q", data))


def _struct_ptr(off, dw, pw):
    return ((off & 0x3FFFFFFF) << 2) | (dw << 32) | (pw << 48)


def _list_ptr(off, size_code, count):
    return 1 | ((off & 0x3FFFFFFF) << 2) | (size_code << 32) | (count << 35)


def _small_report():
    step = P.ProfileStep(local_index=1, phase=2, epoch=3, operation="op", kind="compute", kernel="k",
                         exchange_event_cycles=4)
    return P.ProfileReport(1_000_000_000, [P.TileProfile(7, [P.CycleSample(step, 10, 25)])])


def test_golden_layout():
    data = P.write(_small_report())
    head, body = data[:8], data[8:]
    words = _words(body)
    assert struct.unpack("<2I", head) == (0, len(words))      # one segment, its size in words
    want = [
        _struct_ptr(0, 2, 1),                  # root -> Profile (2 data words, 1 pointer)
        5,                                     # schemaVersion
        1_000_000_000,                         # clockHz
        _list_ptr(0, 7, 2),                    # tiles: composite, 1 element x 2 words
        (1 << 2) | (1 << 32) | (1 << 48),      # tag: 1 element, 1 data word, 1 pointer
        7,                                     # physicalTile
        _list_ptr(0, 7, 2),                    # samples
        (1 << 2) | (1 << 32) | (1 << 48),
        10 | (25 << 32),                       # startCycle, endCycle
        _struct_ptr(0, 3, 4),                  # step -> Step (3 data words, 4 pointers)
        1 | (2 << 32),                         # localIndex, phase
        3 | (1 << 32),                         # epoch, kind = compute (u16 at byte 12)
        4,                                     # exchangeEventCycles
        _list_ptr(3, 2, 3),                    # operation: "op\0"
        _list_ptr(3, 2, 2),                    # kernel: "k\0"
        _list_ptr(3, 7, 0),                    # metadata: empty composite list
        _list_ptr(3, 7, 0),                    # exchangeActivities: empty
        int.from_bytes(b"op\0".ljust(8, b"\0"), "little"),
        int.from_bytes(b"k\0".ljust(8, b"\0"), "little"),
        2 << 48,                               # metadata tag: 0 elements, 0 data, 2 pointers
        2 << 32,                               # activities tag: 0 elements, 2 data, 0 pointers
    ]
    assert words == want


def test_round_trip_full():
    acts = [P.ExchangeActivity("send", 1, 9), P.ExchangeActivity("partnerBusy", 3, 4),
            P.ExchangeActivity("receive", 0, 0xFFFFFFFF)]
    steps = [
        P.ProfileStep(0, 0, 0, "operation.0", "compute", "gemm_f16+gelu", [("flop", "1.0995e+12"), ("tflops", "1450")]),
        P.ProfileStep(1, 1, 0, "", "exchange", "", [], acts, 77),
        P.ProfileStep(2, 5, 1, "operation.12", "synchronization", "x" * 1000, [("ünïcode", "värde"), ("", "")]),
        P.ProfileStep(3, 6, 1, "operation.3", "idle", "k"),
    ]
    rep = P.ProfileReport(1_850_000_000, [
        P.TileProfile(0, [P.CycleSample(s, 100 * i, 100 * i + 50) for i, s in enumerate(steps)]),
        P.TileProfile(1471, []),
        P.TileProfile(3, [P.CycleSample(steps[0], 0, 0xFFFFFFFF)]),
    ])
    back = P.read(P.write(rep))
    assert back == rep


def test_empty_report():
    rep = P.ProfileReport(0, [])
    assert P.read(P.write(rep)) == rep


def test_reader_rejects_schema_versions():
    data = bytearray(P.write(_small_report()))
    for v, ok in ((1, True), (5, True), (0, False), (6, False)):
        struct.pack_into("<I", data, 16, v)       # framing 8 bytes + root pointer 8 bytes
        if ok:
            P.read(bytes(data))
        else:
            with pytest.raises(P.ProfileError, match=f"unsupported profile schema version {v}"):
                P.read(bytes(data))


def test_reader_rejects_truncation():
    data = P.write(_small_report())
    with pytest.raises(P.ProfileError):
        P.read(data[:-8])
    with pytest.raises(P.ProfileError):
        P.read(data[:4])


def _frame(segments):
    n = len(segments)
    head = struct.pack(f"<{n + 1}I", n - 1, *[len(s) for s in segments])
    if len(head) % 8:
        head += b"\0" * 4
    return head + b"".join(struct.pack(f"<{len(s)}Q", *s) for s in segments)


def test_reader_follows_far_pointers():
    words = _words(P.write(_small_report())[8:])
    want = P.read(P.write(_small_report()))
    # single far: segment 0 holds only a far pointer to the landing pad (the
    # original root pointer) at word 0 of segment 1
    single = _frame([[2 | (0 << 3) | (1 << 32)], words])
    assert P.read(single) == want
    # double far: segment 2 holds the landing pad (a far pointer to the struct
    # at segment 1 word 1) and the tag word (a struct pointer with offset 0)
    double = _frame([[2 | (1 << 2) | (0 << 3) | (2 << 32)], words,
                     [2 | (1 << 3) | (1 << 32), _struct_ptr(0, 2, 1)]])
    assert P.read(double) == want


def test_encoder_rejects_bad_kinds():
    rep = _small_report()
    rep.tiles[0].samples[0].step.kind = "compute"
    P.write(rep)
    with pytest.raises(ValueError):
        rep.tiles[0].samples[0].step.kind = "bogus"
        P.write(rep)


def test_encoder_reports_needed_size():
    import ctypes
    fn = P._encoder()
    need = ctypes.c_uint64(0)
    tiles = (P._Tile * 1)()
    st = fn(1, tiles, 0, None, 0, ctypes.byref(need))
    assert st == ipuc.ERR_INVALID_ARGUMENT and need.value == len(P.write(P.ProfileReport(1, [])))


def test_merge_and_query():
    def tile(t, spans):
        return P.TileProfile(t, [P.CycleSample(P.ProfileStep(i, i, 0, f"operation.{i}", "compute", k), a, b)
                                 for i, (k, a, b) in enumerate(spans)])
    r0 = P.ProfileReport(1_000_000_000, [tile(0, [("gemm", 0, 1000), ("attn", 1000, 4000)])])
    r1 = P.ProfileReport(1_000_000_000, [tile(1, [("gemm", 0, 2000), ("attn", 2000, 3000)])])
    m = P.merge([r0, r1])
    assert [t.physical_tile for t in m.tiles] == [0, 1]
    rep = P.query(m, "kernel", sort_by="work-cycles")
    assert [(g["name"], g["sampleCount"], g["workCycles"], g["tileCount"]) for g in rep["groups"]] == [
        ("attn", 2, 4000, 2), ("gemm", 2, 3000, 2)]
    assert rep["groups"][0]["phaseCycles"] == 3000 and rep["groups"][0]["phaseMs"] == pytest.approx(3e-3)
    assert rep["sampleCount"] == rep["matchedSampleCount"] == 4 and rep["profileSpanCycles"] == 4000
    assert [g["name"] for g in P.query(m, "tile", sort_by="name")["groups"]] == ["tile 0", "tile 1"]
    assert P.query(m, "kernel", kind="idle")["groups"] == []
    with pytest.raises(P.ProfileError):
        P.merge([r0, P.ProfileReport(2, [])])


# The query cases below restate the reference's own tests of `ipu-profile query`
# (crates/ipu-profile/src/lib.rs:792-1049) with their expected values.

def _smp(phase, kind, kernel, start, end):
    step = P.ProfileStep(phase, phase, 0, f"operation {phase}", kind, kernel, [("block", str(phase))])
    return P.CycleSample(step, start, end)


def test_query_groups_parallel_samples_by_kernel():
    rep = P.ProfileReport(1_000_000_000, [P.TileProfile(2, [_smp(0, "compute", "add", 100, 120)]),
                                          P.TileProfile(3, [_smp(1, "compute", "add", 100, 130)])])
    r = P.query(rep)
    (g,) = r["groups"]
    assert (g["phaseCycles"], g["workCycles"], g["averageActiveTiles"]) == (30, 50, 50 / 30)
    assert r["profileSpanCycles"] == 30


def test_query_crops_one_common_initial_entry_span():
    rng = np.random.default_rng(0x70726F6772616D)
    for case in range(64):
        starts = rng.integers(1000, 10001, rng.integers(2, 33))
        boundary = int(starts.max()) + int(rng.integers(1, 2001))
        work = int(rng.integers(1, 2001))
        rep = P.ProfileReport(1_000_000_000, [
            P.TileProfile(t, [_smp(0, "synchronization", "", int(st), boundary),
                              _smp(1, "compute", "work", boundary, boundary + work)])
            for t, st in enumerate(starts)])
        aligned = P.query(rep, group_by="kind")
        shared = P.query(rep, shared_clock=True)
        wait = boundary - int(starts.max())
        assert aligned["profileSpanCycles"] == wait + work, case
        assert shared["profileSpanCycles"] >= aligned["profileSpanCycles"], case
        groups = {g["name"]: g for g in aligned["groups"]}
        assert groups["synchronization"]["firstOffset"] == 0 and groups["synchronization"]["maximumCycles"] == wait
        assert groups["compute"]["firstOffset"] == wait


def test_query_phase_cycles_of_sequential_repeats():
    rep = P.ProfileReport(1_000_000_000, [
        P.TileProfile(2, [_smp(0, "compute", "gemm", 100, 110), _smp(0, "compute", "gemm", 110, 120)]),
        P.TileProfile(3, [_smp(0, "compute", "gemm", 100, 108), _smp(0, "compute", "gemm", 108, 116)])])
    g = P.query(rep)["groups"][0]
    assert (g["phaseCycles"], g["workCycles"], g["averageActiveTiles"]) == (20, 36, 1.8)


def test_query_common_origin_keeps_entry_skew_out_of_later_samples():
    rep = P.ProfileReport(1_000_000_000, [
        P.TileProfile(2, [_smp(0, "exchange", "", 100, 150), _smp(1, "compute", "gemm", 150, 160)]),
        P.TileProfile(3, [_smp(0, "exchange", "", 120, 150), _smp(1, "compute", "gemm", 150, 160)])])
    r = P.query(rep, kind="compute", sample_limit=2, shared_clock=True)
    assert len(r["samples"]) == 2 and all(x["offset"] == 50 for x in r["samples"])
    assert r["groups"][0]["phaseCycles"] == 10


def test_query_time_and_metadata_filters_across_counter_wrap():
    rep = P.ProfileReport(1_500_000_000, [P.TileProfile(9, [_smp(0, "exchange", "", 0xFFFFFFFF - 4, 5),
                                                            _smp(1, "compute", "add", 5, 15)])])
    r = P.query(rep, at_offset=12, metadata=[("block", "1")], sample_limit=1)
    assert r["matchedSampleCount"] == 1 and r["samples"][0]["phase"] == 1 and r["samples"][0]["offset"] == 10


def test_query_groups_by_metadata_value():
    rep = P.ProfileReport(1_000_000_000, [P.TileProfile(1, [_smp(0, "compute", "add", 0, 10),
                                                            _smp(1, "compute", "add", 10, 30)])])
    r = P.query(rep, group_by="metadata", metadata_key="block")
    assert [g["name"] for g in r["groups"]] == ["1", "0"]


def _gather_worker(rank, world, port, out):
    import os

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        step = P.ProfileStep(0, 0, 0, "operation.0", "compute", f"gemm_rank{rank}", [("device", str(rank))])
        mine = P.ProfileReport(1_000_000_000, [P.TileProfile(rank, [P.CycleSample(step, 0, 1000 * (rank + 1))])])
        merged = P.gather(P.write(mine))
        if rank == 0:
            out.put(P.write(merged))
        else:
            assert merged is None
    finally:
        dist.destroy_process_group()


def test_gather_across_gloo_ranks():
    import socket

    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    data = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rep = P.read(data)
    assert [t.physical_tile for t in rep.tiles] == [0, 1]
    assert [g["name"] for g in P.query(rep, "kernel")["groups"]] == ["gemm_rank1", "gemm_rank0"]
