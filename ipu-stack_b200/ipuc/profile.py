"""Profile reports in the reference's Cap'n Proto format.

The reference's profile is a `Profile` message (schemas/profile.capnp,
schemas/profile_common.capnp) written and read by ProfileReport
(crates/ipu-package/src/lib.rs:186-260) and queried by `ipu-profile query`
(crates/ipu-profile/src/lib.rs:450-585).  On this backend a Session produces
the same message from CUDA event timings (Session.profile_capnp, one tile per
GPU, clockHz 1e9 so a cycle is a nanosecond); `write` encodes any report
through the library's encoder (ipug_profile_encode) and `read` decodes one
(any segment count, far pointers included) following the published Cap'n
Proto encoding.  `merge` joins the one-tile reports of several GPUs (`gather`
across torch.distributed ranks), and `query` is ipu-profile's query: the same
filters, grouping, ordering and report fields.

Data classes mirror the reference's Rust types: ProfileReport{clock_hz, tiles},
TileProfile{physical_tile, samples}, CycleSample{step, start_cycle, end_cycle},
ProfileStep{local_index, phase, epoch, operation, kind, kernel, metadata,
exchange_activities, exchange_event_cycles}.
"""

from __future__ import annotations

import ctypes
import struct
from dataclasses import dataclass, field

from . import IpucError

SCHEMA_VERSION = 5                      # crates/ipu-package/src/lib.rs:262
STEP_KINDS = ("exchange", "compute", "synchronization", "idle")
ACTIVITY_KINDS = ("send", "receive", "partnerBusy")


class ProfileError(ValueError):
    """A malformed or unsupported profile message (PackageError::Invalid / Capnp)."""


@dataclass
class ExchangeActivity:
    kind: str
    start_cycle: int
    end_cycle: int


@dataclass
class ProfileStep:
    local_index: int = 0
    phase: int = 0
    epoch: int = 0
    operation: str = ""
    kind: str = "compute"
    kernel: str = ""
    metadata: list = field(default_factory=list)          # [(name, value)]
    exchange_activities: list = field(default_factory=list)
    exchange_event_cycles: int = 0


@dataclass
class CycleSample:
    step: ProfileStep
    start_cycle: int
    end_cycle: int


@dataclass
class TileProfile:
    physical_tile: int
    samples: list


@dataclass
class ProfileReport:
    clock_hz: int
    tiles: list


# ---------------------------------------------------------------------------
# Encoding (through the library)
# ---------------------------------------------------------------------------

class _Activity(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_uint32), ("start_cycle", ctypes.c_uint32), ("end_cycle", ctypes.c_uint32)]


class _Sample(ctypes.Structure):
    _fields_ = [("local_index", ctypes.c_uint32), ("phase", ctypes.c_uint32), ("epoch", ctypes.c_uint32),
                ("kind", ctypes.c_uint32), ("operation", ctypes.c_char_p), ("kernel", ctypes.c_char_p),
                ("metadata", ctypes.POINTER(ctypes.c_char_p)), ("metadata_count", ctypes.c_uint32),
                ("activities", ctypes.POINTER(_Activity)), ("activity_count", ctypes.c_uint32),
                ("exchange_event_cycles", ctypes.c_uint32), ("start_cycle", ctypes.c_uint32),
                ("end_cycle", ctypes.c_uint32)]


class _Tile(ctypes.Structure):
    _fields_ = [("physical_tile", ctypes.c_uint32), ("samples", ctypes.POINTER(_Sample)),
                ("sample_count", ctypes.c_uint64)]


def _encoder():
    from . import lib
    fn = lib().ipug_profile_encode
    fn.restype = ctypes.c_int32
    fn.argtypes = [ctypes.c_uint64, ctypes.POINTER(_Tile), ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64,
                   ctypes.POINTER(ctypes.c_uint64)]
    return fn


def write(report: ProfileReport) -> bytes:
    """Encode `report` as a framed Profile message (ProfileReport::write)."""
    keep = []   # ctypes objects that must outlive the call
    tiles = (_Tile * max(1, len(report.tiles)))()
    for t, tile in enumerate(report.tiles):
        samples = (_Sample * max(1, len(tile.samples)))()
        keep.append(samples)
        for i, smp in enumerate(tile.samples):
            st = smp.step
            meta = (ctypes.c_char_p * max(1, 2 * len(st.metadata)))()
            for j, (name, value) in enumerate(st.metadata):
                meta[2 * j], meta[2 * j + 1] = name.encode(), value.encode()
            acts = (_Activity * max(1, len(st.exchange_activities)))()
            for j, a in enumerate(st.exchange_activities):
                acts[j] = _Activity(ACTIVITY_KINDS.index(a.kind), a.start_cycle, a.end_cycle)
            keep += [meta, acts]
            samples[i] = _Sample(st.local_index, st.phase, st.epoch, STEP_KINDS.index(st.kind),
                                 st.operation.encode(), st.kernel.encode(), meta, len(st.metadata), acts,
                                 len(st.exchange_activities), st.exchange_event_cycles, smp.start_cycle,
                                 smp.end_cycle)
        tiles[t] = _Tile(tile.physical_tile, samples, len(tile.samples))
    fn = _encoder()
    need = ctypes.c_uint64(0)
    fn(report.clock_hz, tiles, len(report.tiles), None, 0, ctypes.byref(need))
    buf = ctypes.create_string_buffer(int(need.value))
    rc = fn(report.clock_hz, tiles, len(report.tiles), buf, len(buf), ctypes.byref(need))
    if rc != 0:
        from . import lib
        raise IpucError("ipug_profile_encode", rc, (lib().ipuc_last_error_string() or b"").decode())
    return buf.raw[:need.value]


# ---------------------------------------------------------------------------
# Decoding (Cap'n Proto wire format, read side)
# ---------------------------------------------------------------------------

class _Message:
    def __init__(self, data: bytes):
        if len(data) < 8:
            raise ProfileError("Cap'n Proto error: message shorter than its segment table")
        count = struct.unpack_from("<I", data, 0)[0] + 1
        head = 4 * (1 + count)
        head += head % 8
        if count > 512 or len(data) < head:
            raise ProfileError("Cap'n Proto error: bad segment table")
        sizes = struct.unpack_from(f"<{count}I", data, 4)
        self.segments, off = [], head
        for n in sizes:
            if off + 8 * n > len(data):
                raise ProfileError("Cap'n Proto error: segment runs past the end of the message")
            self.segments.append(data[off:off + 8 * n])
            off += 8 * n

    def word(self, seg: int, idx: int) -> int:
        s = self.segments[seg]
        if not 0 <= idx < len(s) // 8:
            raise ProfileError("Cap'n Proto error: pointer out of bounds")
        return struct.unpack_from("<Q", s, 8 * idx)[0]

    def resolve(self, seg: int, idx: int):
        """Follow the pointer at (seg, idx): returns (tag word, seg, first word of
        the target), or None for a null pointer."""
        p = self.word(seg, idx)
        if p == 0:
            return None
        if p & 3 == 2:                     # far pointer
            double = (p >> 2) & 1
            pad, tseg = (p >> 3) & 0x1FFFFFFF, p >> 32
            if tseg >= len(self.segments):
                raise ProfileError("Cap'n Proto error: far pointer to a missing segment")
            if not double:
                return self.resolve(tseg, pad)
            land, tag = self.word(tseg, pad), self.word(tseg, pad + 1)
            if land & 3 != 2:
                raise ProfileError("Cap'n Proto error: bad double-far landing pad")
            return tag, land >> 32, (land >> 3) & 0x1FFFFFFF
        off = (p >> 2) & 0x3FFFFFFF
        if off & 0x20000000:
            off -= 0x40000000
        return p, seg, idx + 1 + off


class _Struct:
    def __init__(self, msg: _Message, seg: int, at: int, dwords: int, pwords: int):
        self.msg, self.seg, self.at, self.dwords, self.pwords = msg, seg, at, dwords, pwords

    def _data(self, byte: int, fmt: str) -> int:
        size = struct.calcsize(fmt)
        if byte + size > 8 * self.dwords:   # field beyond an older, shorter struct: default 0
            return 0
        s = self.msg.segments[self.seg]
        return struct.unpack_from("<" + fmt, s, 8 * self.at + byte)[0]

    def u16(self, byte): return self._data(byte, "H")
    def u32(self, byte): return self._data(byte, "I")
    def u64(self, byte): return self._data(byte, "Q")

    def _ptr(self, i: int):
        if i >= self.pwords:
            return None
        return self.msg.resolve(self.seg, self.at + self.dwords + i)

    def struct(self, i: int):
        r = self._ptr(i)
        if r is None:
            return None
        p, seg, at = r
        if p & 3 != 0:
            raise ProfileError("Cap'n Proto error: expected a struct pointer")
        return _Struct(self.msg, seg, at, (p >> 32) & 0xFFFF, p >> 48)

    def structs(self, i: int) -> list:
        r = self._ptr(i)
        if r is None:
            return []
        p, seg, at = r
        if p & 3 != 1 or (p >> 32) & 7 != 7:
            raise ProfileError("Cap'n Proto error: expected a list of structs")
        tag = self.msg.word(seg, at)
        n, dw, pw = (tag >> 2) & 0x3FFFFFFF, (tag >> 32) & 0xFFFF, tag >> 48
        if n * (dw + pw) > p >> 35:
            raise ProfileError("Cap'n Proto error: list elements exceed the list's word count")
        return [_Struct(self.msg, seg, at + 1 + k * (dw + pw), dw, pw) for k in range(n)]

    def text(self, i: int) -> str:
        r = self._ptr(i)
        if r is None:
            return ""
        p, seg, at = r
        if p & 3 != 1 or (p >> 32) & 7 != 2:
            raise ProfileError("Cap'n Proto error: expected Text")
        n = p >> 35
        raw = self.msg.segments[seg][8 * at:8 * at + n]
        if len(raw) != n or n == 0 or raw[-1] != 0:
            raise ProfileError("Cap'n Proto error: Text is not NUL-terminated")
        try:
            return raw[:-1].decode("utf-8")
        except UnicodeDecodeError as e:
            raise ProfileError(f"Cap'n Proto error: {e}") from None


def _enum(names, v, what):
    if v >= len(names):
        raise ProfileError(f"Cap'n Proto error: enum value {v} not in {what}")
    return names[v]


def read(data: bytes) -> ProfileReport:
    """Decode a framed Profile message (ProfileReport::read,
    crates/ipu-package/src/lib.rs:225-259): schema versions 1-5 only."""
    msg = _Message(bytes(data))
    root = msg.resolve(0, 0)
    if root is None or root[0] & 3 != 0:
        raise ProfileError("Cap'n Proto error: root is not a struct")
    p, seg, at = root
    r = _Struct(msg, seg, at, (p >> 32) & 0xFFFF, p >> 48)
    version = r.u32(0)
    if not 1 <= version <= 5:
        raise ProfileError(f"unsupported profile schema version {version}")
    tiles = []
    for t in r.structs(0):
        samples = []
        for s in t.structs(0):
            st = s.struct(0)
            step = ProfileStep()
            if st is not None:
                step = ProfileStep(
                    local_index=st.u32(0), phase=st.u32(4), epoch=st.u32(8), operation=st.text(0),
                    kind=_enum(STEP_KINDS, st.u16(12), "StepKind"), kernel=st.text(1),
                    metadata=[(m.text(0), m.text(1)) for m in st.structs(2)],
                    exchange_activities=[ExchangeActivity(_enum(ACTIVITY_KINDS, a.u16(0), "ExchangeActivityKind"),
                                                          a.u32(4), a.u32(8)) for a in st.structs(3)],
                    exchange_event_cycles=st.u32(16))
            samples.append(CycleSample(step, s.u32(0), s.u32(4)))
        tiles.append(TileProfile(t.u32(0), samples))
    return ProfileReport(r.u64(8), tiles)


# ---------------------------------------------------------------------------
# Multi-GPU merge and query
# ---------------------------------------------------------------------------

def merge(reports) -> ProfileReport:
    """One report with every tile of `reports` (e.g. one per GPU rank); all
    must share clock_hz, as ipu-profile requires of the reports it joins
    (crates/ipu-profile/src/lib.rs:215-224)."""
    reports = list(reports)
    if not reports:
        raise ProfileError("no profile reports")
    clock = reports[0].clock_hz
    if any(r.clock_hz != clock for r in reports):
        raise ProfileError("profile reports have different clock rates")
    return ProfileReport(clock, [t for r in reports for t in r.tiles])


GROUP_BY = ("kind", "kernel", "operation", "phase", "tile", "metadata")
SORT_BY = ("phase-cycles", "work-cycles", "maximum-cycles", "samples", "name")


def _i32(x: int) -> int:
    x &= 0xFFFFFFFF
    return x - (1 << 32) if x >= (1 << 31) else x


def _duration(smp: CycleSample) -> int:
    return (smp.end_cycle - smp.start_cycle) & 0xFFFFFFFF


def cycle_origin(report: ProfileReport) -> int:
    """The common cycle origin of the tiles' first samples on the wrapping
    32-bit counter (crates/ipu-profile/src/lib.rs:285-299)."""
    firsts = [t.samples[0].start_cycle for t in report.tiles if t.samples]
    if not firsts:
        return 0
    ref = firsts[0]
    return (ref + min(_i32(f - ref) for f in firsts)) & 0xFFFFFFFF


def _union_length(intervals) -> int:
    total, cur = 0, None
    for lo, hi in sorted(intervals):
        if cur is None:
            cur = [lo, hi]
        elif lo <= cur[1]:
            cur[1] = max(cur[1], hi)
        else:
            total += cur[1] - cur[0]
            cur = [lo, hi]
    return total + (cur[1] - cur[0] if cur else 0)


def query(report: ProfileReport, group_by: str = "kernel", sort_by: str = "phase-cycles", kind: str | None = None,
          kernel: str | None = None, operation_contains: str | None = None, tiles=(), phases=(), metadata=(),
          metadata_key: str | None = None, at_offset: int | None = None, shared_clock: bool = False,
          limit: int | None = None, sample_limit: int = 0) -> dict:
    """`ipu-profile query` on a report (crates/ipu-profile/src/lib.rs:450-585):
    the same filters (kind, kernel, operation substring, tiles, phases, metadata
    name[=value] pairs, a cycle offset the sample must cover), group-by
    (kind, kernel, operation, phase, tile, metadata value under metadata_key),
    sort order and limits, and the same report fields in camelCase.  Offsets
    count from the tiles' common cycle origin; unless shared_clock, the span
    before the last tile's first sample is cropped.  Per group, phaseCycles is
    the length of the union of its samples' intervals and workCycles their sum."""
    if group_by not in GROUP_BY or sort_by not in SORT_BY:
        raise ValueError(f"group_by one of {GROUP_BY}, sort_by one of {SORT_BY}")
    tiles, phases = set(tiles), set(phases)
    metadata = [(m, None) if isinstance(m, str) else tuple(m) for m in metadata]
    base = cycle_origin(report)
    crop = 0 if shared_clock else max(
        (((t.samples[0].start_cycle - base) & 0xFFFFFFFF) for t in report.tiles if t.samples), default=0)
    sample_count = sum(len(t.samples) for t in report.tiles)
    span = 0
    groups, candidates, matched = {}, [], 0
    for tile in report.tiles:
        for smp in tile.samples:
            raw = (smp.start_cycle - base) & 0xFFFFFFFF
            raw_end = raw + _duration(smp)
            span = max(span, max(raw_end - crop, 0))
            off, end = max(raw - crop, 0), max(raw_end - crop, 0)
            dur = min(end - off, 0xFFFFFFFF)
            st = smp.step
            if dur == 0:
                continue
            if ((kind is not None and st.kind != kind) or (kernel is not None and st.kernel != kernel)
                    or (operation_contains is not None and operation_contains not in st.operation)
                    or (tiles and tile.physical_tile not in tiles) or (phases and st.phase not in phases)
                    or (at_offset is not None and not off <= at_offset < off + dur)):
                continue
            if not all(any(n == name and (v is None or val == v) for n, val in st.metadata) for name, v in metadata):
                continue
            matched += 1
            dims = {}
            if group_by == "kind":
                name = st.kind
            elif group_by == "kernel":
                name = st.kernel or "(no kernel)"
            elif group_by == "operation":
                name = st.operation
            elif group_by == "phase":
                dims = {"phase": str(st.phase), "epoch": str(st.epoch)}
                name = f"phase {st.phase}/{st.epoch}"
            elif group_by == "tile":
                dims = {"physicalTile": str(tile.physical_tile)}
                name = f"tile {tile.physical_tile}"
            else:
                key = metadata_key or ""
                value = next((val for n, val in st.metadata if n == key), "(missing)")
                dims = {"metadataKey": key, "metadataValue": value}
                name = value
            g = groups.setdefault(name, {"dims": dims, "durations": [], "tiles": set(), "phases": set(),
                                         "intervals": [], "first": off, "last": 0})
            g["durations"].append(dur)
            g["tiles"].add(tile.physical_tile)
            g["phases"].add((st.phase, st.epoch))
            g["intervals"].append((off, off + dur))
            g["first"] = min(g["first"], off)
            g["last"] = max(g["last"], off + dur)
            if sample_limit > 0:
                candidates.append((tile.physical_tile, off, dur, smp))
    ms = (lambda c: c * 1e3 / report.clock_hz) if report.clock_hz else (lambda c: 0.0)
    summaries = []
    for name, g in groups.items():
        d = sorted(g["durations"])
        work, phase = sum(d), _union_length(g["intervals"])
        summaries.append({
            "name": name, "dimensions": g["dims"], "sampleCount": len(d), "tileCount": len(g["tiles"]),
            "phaseCount": len(g["phases"]), "phaseCycles": phase, "phaseMs": ms(phase), "workCycles": work,
            "averageActiveTiles": work / phase if phase else 0.0, "meanCycles": work / len(d),
            "p50Cycles": d[(len(d) - 1) * 50 // 100], "p95Cycles": d[(len(d) - 1) * 95 // 100],
            "maximumCycles": d[-1], "firstOffset": g["first"], "lastOffset": g["last"]})
    primary = {"phase-cycles": lambda s: -s["phaseCycles"], "work-cycles": lambda s: -s["workCycles"],
               "maximum-cycles": lambda s: -s["maximumCycles"], "samples": lambda s: -s["sampleCount"],
               "name": lambda s: s["name"]}[sort_by]
    summaries.sort(key=lambda s: (primary(s), s["firstOffset"], s["name"]))
    if limit is not None:
        summaries = summaries[:limit]
    candidates.sort(key=lambda c: (-c[2], c[0], c[1]))
    samples = [{"physicalTile": t, "offset": off, "duration": dur, "phase": smp.step.phase,
                "epoch": smp.step.epoch, "kind": smp.step.kind, "operation": smp.step.operation,
                "kernel": smp.step.kernel, "metadata": [{"name": n, "value": v} for n, v in smp.step.metadata]}
               for t, off, dur, smp in candidates[:sample_limit]]
    return {"clockHz": report.clock_hz, "tileCount": len(report.tiles), "sampleCount": sample_count,
            "matchedSampleCount": matched, "profileSpanCycles": span, "profileSpanMs": ms(span),
            "atOffset": at_offset, "groups": summaries, "samples": samples}


def gather(data: bytes, group=None, dst: int = 0):
    """Join the encoded one-tile reports of every rank of a torch.distributed
    process group into one multi-tile report on rank `dst` (other ranks get
    None): the multi-GPU counterpart of a whole-device profile, one tile per
    GPU.  Collective: every rank of the group must call it."""
    import torch.distributed as dist
    rank = dist.get_rank(group)
    parts = [None] * dist.get_world_size(group) if rank == dst else None
    dist.gather_object(bytes(data), parts, dst=dst, group=group)
    if rank != dst:
        return None
    return merge(read(p) for p in parts)
