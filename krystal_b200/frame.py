"""Host frames: records in, the SoA arrays the forward reads out.

Mirrors packages/krystal/src/host/frame.ts (``packHostFrame``, :72-115) and
packages/krystal/src/forward/masks.ts (``compileActiveFrame`` :65-101,
``recordRanges`` :120-133) of the reference, with the same refusals.

Also packs a *batch* of frames into the flat ragged layout the device batch
entry point takes: per-record arrays concatenated frame after frame plus a
record-offset table (CSR). Everything else — token offsets, bank/query row
lists, output offsets — is derived on the GPU.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Mapping, Sequence, Union

import numpy as np

from .model import RECORD_WIDTH, STREAM_QUERY

PAD_TOKEN = 0  # KRYSTAL_SENTINEL_TOKENS.pad
QUERY_BAND = 5  # index of "query" in BRAIN_FRAME_BANDS (masks.ts:41)
INVALID_U32 = 0xFFFFFFFF


class HostFrameError(ValueError):
    """HostFrameError (frame.ts:30-35)."""


@dataclass(frozen=True)
class HostToken:
    token: int
    role: int | None = None


TokenEntry = Union[int, HostToken, Mapping]


@dataclass
class HostRecord:
    tokens: Sequence[TokenEntry]
    schema_id: int | None = None
    band: int | None = None
    query: bool = False


@dataclass
class BrainFrameGpu:
    token_ids: np.ndarray  # u32 [slots*8]
    field_roles: np.ndarray  # u32 [slots*8]
    schema_ids: np.ndarray  # u32 [slots]
    band_ids: np.ndarray  # u32 [slots]
    active_record_indices: np.ndarray  # u32 [slots]


@dataclass
class ActiveFrame:
    active_tokens: np.ndarray
    record_compact_offset: np.ndarray
    record_compact_count: np.ndarray
    stream_ids: np.ndarray
    active_records: np.ndarray
    bank_records: np.ndarray
    query_records: np.ndarray


@dataclass
class HostFrame:
    gpu: BrainFrameGpu
    active: ActiveFrame
    slots: int


def _record_fields(rec) -> tuple[Sequence[TokenEntry], int | None, int | None, bool]:
    if isinstance(rec, HostRecord):
        return rec.tokens, rec.schema_id, rec.band, bool(rec.query)
    return rec.get("tokens", []), rec.get("schemaId", rec.get("schema_id")), rec.get("band"), bool(rec.get("query"))


def _token_of(entry) -> tuple[int, int | None]:
    if isinstance(entry, HostToken):
        return entry.token, entry.role
    if isinstance(entry, Mapping):
        return entry["token"], entry.get("role")
    return entry, None


def pack_host_frame(records: Sequence) -> HostFrame:
    """packHostFrame (frame.ts:72-115)."""
    slots = len(records)
    if not slots:
        raise HostFrameError("a frame with no records has nothing to think about")
    token_ids = np.full(slots * RECORD_WIDTH, PAD_TOKEN, dtype=np.uint32)
    field_roles = np.zeros(slots * RECORD_WIDTH, dtype=np.uint32)
    schema_ids = np.zeros(slots, dtype=np.uint32)
    band_ids = np.zeros(slots, dtype=np.uint32)
    active = np.full(slots, INVALID_U32, dtype=np.uint32)
    for slot, rec in enumerate(records):
        tokens, schema_id, band, query = _record_fields(rec)
        tokens = tokens or []
        if len(tokens) > RECORD_WIDTH:
            raise HostFrameError(
                f"record {slot} carries {len(tokens)} tokens; {RECORD_WIDTH} is the width the model has positions "
                "for — split it into a base record and a continuation")
        schema_ids[slot] = schema_id or 0
        band_ids[slot] = QUERY_BAND if query else (band or 0)
        active[slot] = slot
        for local, entry in enumerate(tokens):
            token, role = _token_of(entry)
            if not isinstance(token, (int, np.integer)) or isinstance(token, bool) or token < 0:
                raise HostFrameError(f"record {slot} token {local} is not a token id")
            if token == PAD_TOKEN:
                continue  # a hole in a record is simply absent
            at = slot * RECORD_WIDTH + local
            token_ids[at] = token
            field_roles[at] = role or 0
    gpu = BrainFrameGpu(token_ids, field_roles, schema_ids, band_ids, active)
    return HostFrame(gpu, compile_active_frame(gpu), slots)


def compile_active_frame(frame: BrainFrameGpu) -> ActiveFrame:
    """compileActiveFrame (masks.ts:65-101)."""
    slots = frame.schema_ids.size
    offset = np.full(slots, INVALID_U32, dtype=np.uint32)
    count = np.zeros(slots, dtype=np.uint32)
    stream = np.zeros(slots, dtype=np.uint32)
    tokens: list[int] = []
    records: list[int] = []
    for slot in frame.active_record_indices.tolist():
        if slot == INVALID_U32 or slot >= slots:
            break  # unoccupied tail
        records.append(slot)
        offset[slot] = len(tokens)
        row = frame.token_ids[slot * RECORD_WIDTH:(slot + 1) * RECORD_WIDTH]
        live = np.nonzero(row != PAD_TOKEN)[0]
        tokens.extend((slot * RECORD_WIDTH + live).tolist())
        count[slot] = live.size
        stream[slot] = STREAM_QUERY if frame.band_ids[slot] == QUERY_BAND else 0
    rec = np.asarray(records, dtype=np.uint32)
    is_q = stream[rec] == STREAM_QUERY if rec.size else np.zeros(0, dtype=bool)
    return ActiveFrame(np.asarray(tokens, dtype=np.uint32), offset, count, stream, rec,
                       rec[~is_q].astype(np.uint32), rec[is_q].astype(np.uint32))


def record_ranges(active: ActiveFrame) -> tuple[np.ndarray, np.ndarray]:
    """recordRanges (masks.ts:120-133): each compact token's own record range."""
    t = active.active_tokens.size
    start = np.zeros(t, dtype=np.uint32)
    cnt = np.zeros(t, dtype=np.uint32)
    for slot in active.active_records.tolist():
        f, n = int(active.record_compact_offset[slot]), int(active.record_compact_count[slot])
        start[f:f + n] = f
        cnt[f:f + n] = n
    return start, cnt


@dataclass
class FrameBatch:
    """A packed ragged batch: frame f owns records rec_off[f]..rec_off[f+1].

    Every record is active, in order, as ``packHostFrame`` leaves them.
    """

    rec_off: np.ndarray  # u64 [F+1]
    token_ids: np.ndarray  # u32 [N*8]
    field_roles: np.ndarray  # u32 [N*8]
    schema_ids: np.ndarray  # u32 [N]
    band_ids: np.ndarray  # u32 [N]

    @property
    def frames(self) -> int:
        return int(self.rec_off.size - 1)

    @property
    def records(self) -> int:
        return int(self.rec_off[-1])

    def frame(self, f: int) -> BrainFrameGpu:
        a, b = int(self.rec_off[f]), int(self.rec_off[f + 1])
        return BrainFrameGpu(self.token_ids[a * RECORD_WIDTH:b * RECORD_WIDTH].copy(),
                             self.field_roles[a * RECORD_WIDTH:b * RECORD_WIDTH].copy(),
                             self.schema_ids[a:b].copy(), self.band_ids[a:b].copy(),
                             np.arange(b - a, dtype=np.uint32))

    def subset(self, frames: Sequence[int] | slice) -> "FrameBatch":
        idx = np.arange(self.frames)[frames] if isinstance(frames, slice) else np.asarray(frames)
        counts = (self.rec_off[idx + 1] - self.rec_off[idx]).astype(np.uint64)
        rec_off = np.zeros(idx.size + 1, dtype=np.uint64)
        np.cumsum(counts, out=rec_off[1:])
        off = self.rec_off.astype(np.int64)
        recs = np.concatenate([np.arange(off[i], off[i + 1]) for i in idx]) if idx.size else \
            np.zeros(0, dtype=np.int64)
        tok = (recs[:, None] * RECORD_WIDTH + np.arange(RECORD_WIDTH)).reshape(-1)
        return FrameBatch(rec_off, self.token_ids[tok], self.field_roles[tok], self.schema_ids[recs],
                          self.band_ids[recs])

    def offsets(self) -> dict[str, np.ndarray]:
        """Per-frame T/R/Q and output offsets, computed on the host (for checks)."""
        f = self.frames
        live = (self.token_ids.reshape(-1, RECORD_WIDTH) != PAD_TOKEN).sum(1)
        isq = self.band_ids == QUERY_BAND
        cs = lambda v: np.concatenate([[0], np.cumsum(v)]).astype(np.uint64)  # noqa: E731
        t = np.add.reduceat(live, self.rec_off[:-1].astype(np.int64)) if f else np.zeros(0)
        q = np.add.reduceat(isq.astype(np.int64), self.rec_off[:-1].astype(np.int64)) if f else np.zeros(0)
        n = np.diff(self.rec_off.astype(np.int64))
        # reduceat on an empty segment returns the next element; no frame here is empty
        r = n - q
        return {"t": t, "q": q, "r": r, "t_off": cs(t), "q_off": cs(q), "r_off": cs(r), "p_off": cs(q * r)}


def pack_frame_batch(frames: Sequence[Sequence]) -> FrameBatch:
    """Pack several record lists (each as for ``pack_host_frame``) into a batch."""
    packed = [pack_host_frame(recs).gpu for recs in frames]
    counts = np.array([p.schema_ids.size for p in packed], dtype=np.uint64)
    rec_off = np.zeros(len(packed) + 1, dtype=np.uint64)
    np.cumsum(counts, out=rec_off[1:])
    return FrameBatch(rec_off, np.concatenate([p.token_ids for p in packed]),
                      np.concatenate([p.field_roles for p in packed]),
                      np.concatenate([p.schema_ids for p in packed]),
                      np.concatenate([p.band_ids for p in packed]))
