"""Rolling batches over the C ABI's streaming packer (``kc_stream_*``).

An interactive host sees think() turns (host/session.ts:128-181) arrive one
at a time from many sessions. ``FrameStream`` queues each packed frame as it
arrives (validated on the host, so a malformed frame is refused alone),
seals the open batch when the caller flushes, and a worker thread inside the
library runs sealed batches back to back on the backend's GPU while more
frames are queued. ``poll`` returns finished batches with the steady-clock
times they were sealed and finished (``clock_ms`` reads the same clock).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import abi
from .backend import CudaBrainBackend, _u32
from .frame import BrainFrameGpu, FrameBatch, HostFrame


@dataclass
class StreamBatch:
    """One finished batch: tickets first_ticket .. first_ticket+frames-1."""
    first_ticket: int
    frames: int
    p_off: np.ndarray   # [frames+1]
    q_off: np.ndarray   # [frames+1]
    p: np.ndarray       # [total_p]
    index: np.ndarray   # [questions]
    status: int
    error: str | None
    sealed_ms: float
    done_ms: float
    started_ms: float = 0.0     # when the worker took the batch up
    sync_wait_ms: float = 0.0   # of done_ms - started_ms, blocked until the device finished


def clock_ms() -> float:
    """The steady clock the stream's timestamps use (milliseconds)."""
    return float(abi.load().kc_stream_clock_ms())


class FrameStream:
    def __init__(self, backend: CudaBrainBackend, max_frames: int = 4096, max_records: int = 1 << 20,
                 max_p: int = 0, depth: int = 3, copy_results: bool = True, push_threads: int = 0,
                 bind_cpus: bool = True):
        """push_threads: threads that check and stage a large push_many (0:
        one per 4 CPUs local to the GPU, at most 8); bind_cpus: the worker and
        helpers run on the GPU's local CPUs and the staging lies on its NUMA
        node."""
        self._lib = abi.load()
        self.backend = backend
        self.copy_results = copy_results
        s = C.c_void_p()
        opts = abi.KcStreamOptions(push_threads, 1 if bind_cpus else 0)
        abi.check(self._lib.kc_stream_create_ex(backend._h, max_frames, max_records, max_p, depth, C.byref(opts),
                                                C.byref(s)), backend._h)
        self._s = s

    def _check(self, status: int) -> None:
        if status != abi.KC_OK:
            msg = self._lib.kc_stream_last_error(self._s)
            raise abi.KrystalCudaError(status, msg.decode() if msg else "")

    def push(self, frame: BrainFrameGpu | HostFrame, schema_allow=None, band_allow=None) -> int:
        """Queue one frame; returns its ticket."""
        g = frame.gpu if isinstance(frame, HostFrame) else frame
        keep = [_u32(g.token_ids), _u32(g.field_roles), _u32(g.schema_ids), _u32(g.band_ids),
                _u32(g.active_record_indices)]
        tok, role, sch, band, act = keep
        fv = abi.KcFrameView(sch.size, tok.ctypes.data, role.ctypes.data, sch.ctypes.data, band.ctypes.data,
                             act.ctypes.data)
        sa = _u32(schema_allow) if schema_allow is not None else None
        ba = _u32(band_allow) if band_allow is not None else None
        t = C.c_uint64()
        self._check(self._lib.kc_stream_push(self._s, C.byref(fv), abi.ptr(sa), abi.ptr(ba), C.byref(t)))
        return int(t.value)

    def push_many(self, batch: FrameBatch, start: int, stop: int, schema_allow=None, band_allow=None,
                  q_start: int = 0) -> tuple[int, int]:
        """Queue frames start..stop-1 of a packed batch in one call (the rule,
        if given, is the batch's per-question rule, its questions from
        q_start). Returns (first ticket, frames queued); stops early, without
        raising, when the open buffer is full or every buffer is in flight."""
        if stop <= start:
            return 0, 0
        rec_off = batch.rec_off if batch.rec_off.dtype == np.uint64 else batch.rec_off.astype(np.uint64)
        keep = [rec_off, _u32(batch.token_ids), _u32(batch.field_roles), _u32(batch.schema_ids),
                _u32(batch.band_ids)]
        sa = _u32(schema_allow) if schema_allow is not None else None
        ba = _u32(band_allow) if band_allow is not None else None
        bv = abi.KcBatchView(stop - start, 0, rec_off.ctypes.data + 8 * start, keep[1].ctypes.data,
                             keep[2].ctypes.data, keep[3].ctypes.data, keep[4].ctypes.data,
                             sa.ctypes.data + 32 * q_start if sa is not None else None,
                             ba.ctypes.data + 4 * q_start if ba is not None else None, None)
        first, n = C.c_uint64(), C.c_uint32()
        st = self._lib.kc_stream_push_many(self._s, C.byref(bv), C.byref(first), C.byref(n))
        if st != abi.KC_OK:
            msg = (self._lib.kc_stream_last_error(self._s) or b"").decode()
            # a full buffer or buffers in flight are flow control; anything else refuses a frame
            if not (st == abi.KC_ERR_CAPACITY and ("flush first" in msg or "poll first" in msg)):
                raise abi.KrystalCudaError(st, f"{msg} (frame {start + n.value})")
        return int(first.value), int(n.value)

    def flush(self) -> None:
        self._check(self._lib.kc_stream_flush(self._s))

    def pending(self) -> int:
        return int(self._lib.kc_stream_pending(self._s))

    def poll(self, wait: bool = False) -> StreamBatch | None:
        r = abi.KcStreamResult()
        self._check(self._lib.kc_stream_poll(self._s, int(wait), C.byref(r)))
        if r.frames == 0:
            return None
        view = lambda ptr, n, dt: np.ctypeslib.as_array(C.cast(ptr, C.POINTER(dt)), (n,)) if n else \
            np.zeros(0, np.dtype(dt))  # noqa: E731
        p_off = view(r.p_off, r.frames + 1, C.c_uint64)
        q_off = view(r.q_off, r.frames + 1, C.c_uint64)
        p = view(r.p, r.total_p, C.c_float)
        idx = view(r.index, r.questions, C.c_uint32)
        if self.copy_results:
            p_off, q_off, p, idx = p_off.copy(), q_off.copy(), p.copy(), idx.copy()
        return StreamBatch(int(r.first_ticket), int(r.frames), p_off, q_off, p, idx, int(r.status),
                           r.error.decode() if r.error else None, float(r.sealed_ms), float(r.done_ms),
                           float(r.started_ms), float(r.sync_wait_ms))

    def stats(self, reset: bool = False) -> dict:
        """Where the stream's host time went since the last reset
        (kc_stream_read_stats): push and worker times, faults, context
        switches, and the NUMA nodes of the GPU, the staging and the threads."""
        st = abi.KcStreamStats()
        self._check(self._lib.kc_stream_read_stats(self._s, int(reset), C.byref(st)))
        return {name: getattr(st, name) for name, _ in abi.KcStreamStats._fields_}

    def close(self) -> None:
        if getattr(self, "_s", None):
            self._lib.kc_stream_destroy(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
