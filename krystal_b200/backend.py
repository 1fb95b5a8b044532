"""The CUDA device backend: ``BrainBackend`` over the C ABI.

Mirrors the seam of packages/krystal/src/host/backend.ts (``EncodedFrame``
:33-39, ``BackwardRequest`` :74-94, ``BackwardResult`` :105-123,
``WeightChanges`` :134-145, ``BrainBackend`` :146-169, ``BrainBackendFactory``
:177-180) and the WebGPU adapter that implements it
(packages/webgpu/src/backend.ts:91-181): ``cuda_backend(device)`` returns a
factory that the session calls with its config and the weights it owns; the
backend keeps a device copy and is told of changes through ``sync``.

``backward`` is the seam's optional ``backward?`` (:158): the gradients of one
frame, computed on the device in the reference's arithmetic.

Beyond the reference seam it offers ``select`` (the selector on the device,
the optional ``select?`` extension ``choose()`` uses when present),
``forward_batch`` (a packed ragged batch of frames, pack → encode → select in
one call) and ``backward_batch_device`` (the backward of a whole batch).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Callable, Sequence

import numpy as np

from . import abi
from .frame import FrameBatch, HostFrame
from .model import BrainForwardConfig, BrainForwardWeights


@dataclass
class EncodedFrame:
    """[Q,H] mixed query output and the [R,H] pooled bank (backend.ts:33-39)."""

    query_output: np.ndarray
    bank_keys: np.ndarray
    bank_values: np.ndarray

    @property
    def q(self) -> int:
        return self.query_output.size // 128

    @property
    def r(self) -> int:
        return self.bank_keys.size // 128


@dataclass
class WeightChanges:
    """Which arrays an update wrote (backend.ts:134-145); all None/False = nothing."""

    selector: bool = False
    pool: bool = False
    value_head: bool = False
    decision_head: bool = False
    blocks: bool = False
    embedding_rows: Sequence[int] = field(default_factory=list)


@dataclass
class Selection:
    """selectorOracle's result (forward/oracle.ts:305-319)."""

    p: np.ndarray  # [Q*R]
    index: np.ndarray  # [Q] u32, KC_NO_SELECTION when a row is all blocked
    gather: np.ndarray | None  # [Q*H]


@dataclass
class BackwardResult:
    """BackwardResult (backend.ts:105-123): the policy the update differentiates,
    the critic's predictions and loss, and the gradients the host may apply."""
    policy: np.ndarray            # [Q*R]
    value_prediction: np.ndarray  # [Q]
    value_loss: float
    d_selector_wq: np.ndarray     # [H*H]
    d_selector_wk: np.ndarray     # [H*H]
    d_pool: np.ndarray            # [2H]
    d_field_states: np.ndarray    # [T*H], active-token order
    d_value_wv: np.ndarray        # [3H]


@dataclass
class MaskRule:
    """Device form of `allows`: 256-bit schema and 8-bit band masks per question."""

    schema_allow: np.ndarray  # u32 [Q*8]
    band_allow: np.ndarray  # u32 [Q]


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


class _Views:
    """Keeps the arrays a kc_weights_view points at alive for one call."""

    def __init__(self, weights: BrainForwardWeights):
        self.keep = []

        def p(a):
            a = _f32(a)
            self.keep.append(a)
            return a.ctypes.data

        def blocks(bs):
            arr = (abi.KcBlockView * max(1, len(bs)))()
            for i, b in enumerate(bs):
                arr[i] = abi.KcBlockView(p(b.wq), p(b.wk), p(b.wv), p(b.w1), p(b.w2))
            self.keep.append(arr)
            return arr

        self.view = abi.KcWeightsView(
            p(weights.embeddings), blocks(weights.enc), p(weights.pool), blocks(weights.mixer),
            p(weights.selector.wq), p(weights.selector.wk), p(weights.decision_head_wh), p(weights.value_head_wv))


def _config_struct(config: BrainForwardConfig) -> tuple[abi.KcConfig, np.ndarray]:
    rows = _u32(config.token_rows)
    c = abi.KcConfig(config.hidden_size, config.head_count, config.head_dim, config.ffn_size, config.encoder_blocks,
                     config.mixer_blocks, config.token_space, config.field_space, config.schema_space,
                     config.band_space, config.stream_space, config.pos_space, config.route_kind_count,
                     rows.ctypes.data if rows.size else None, rows.size)
    return c, rows


class CudaBrainBackend:
    """One device, one handle (GpuBrainBackend's role, webgpu/src/backend.ts:91-168)."""

    def __init__(self, config: BrainForwardConfig, weights: BrainForwardWeights, device: int = 0):
        self._lib = abi.load()
        self.config = config
        self.device = device
        cfg, self._rows = _config_struct(config)
        views = _Views(weights)
        h = C.c_void_p()
        abi.check(self._lib.kc_create(C.byref(cfg), C.byref(views.view), device, C.byref(h)))
        self._h = h

    # --- BrainBackend -----------------------------------------------------
    def encode(self, frame: HostFrame) -> EncodedFrame:
        g = frame.gpu
        tok, role, sch, band, act = (_u32(g.token_ids), _u32(g.field_roles), _u32(g.schema_ids), _u32(g.band_ids),
                                     _u32(g.active_record_indices))
        fv = abi.KcFrameView(sch.size, tok.ctypes.data, role.ctypes.data, sch.ctypes.data, band.ctypes.data,
                             act.ctypes.data)
        q_cap = max(1, frame.active.query_records.size)
        r_cap = max(1, frame.active.bank_records.size)
        h = self.config.hidden_size
        qo = np.empty(q_cap * h, dtype=np.float32)
        bk = np.empty(r_cap * h, dtype=np.float32)
        bvv = np.empty(r_cap * h, dtype=np.float32)
        q, r = C.c_uint32(), C.c_uint32()
        abi.check(self._lib.kc_encode(self._h, C.byref(fv), qo.ctypes.data, bk.ctypes.data, bvv.ctypes.data, q_cap,
                                      r_cap, C.byref(q), C.byref(r)), self._h)
        return EncodedFrame(qo[:q.value * h], bk[:r.value * h], bvv[:r.value * h])

    def sync(self, weights: BrainForwardWeights, changes: WeightChanges | None = None) -> None:
        views = _Views(weights)
        if changes is None:
            abi.check(self._lib.kc_sync(self._h, C.byref(views.view), None), self._h)
            return
        rows = _u32(list(changes.embedding_rows))
        ch = abi.KcChanges(int(changes.selector), int(changes.pool), int(changes.value_head),
                           int(changes.decision_head), int(changes.blocks), rows.ctypes.data if rows.size else None,
                           rows.size)
        abi.check(self._lib.kc_sync(self._h, C.byref(views.view), C.byref(ch)), self._h)

    def destroy(self) -> None:
        if getattr(self, "_h", None):
            self._lib.kc_destroy(self._h)
            self._h = None

    def backward(self, frame: HostFrame, selection=None, targets=None,
                 valence_target: float | None = None) -> BackwardResult:
        """BrainBackend.backward (backend.ts:158): one frame differentiated on the
        device. selection: [Q,R] mask (None = open); targets: [Q] bank rows,
        KC_NO_TARGET, or row | KC_AWAY_TARGET (None = none); valence_target:
        the value head's target (None = none)."""
        g = frame.gpu
        tok, role, sch, band, act = (_u32(g.token_ids), _u32(g.field_roles), _u32(g.schema_ids), _u32(g.band_ids),
                                     _u32(g.active_record_indices))
        fv = abi.KcFrameView(sch.size, tok.ctypes.data, role.ctypes.data, sch.ctypes.data, band.ctypes.data,
                             act.ctypes.data)
        q, r = frame.active.query_records.size, frame.active.bank_records.size
        t = frame.active.active_tokens.size
        h = self.config.hidden_size
        sel = _f32(selection) if selection is not None else None
        if sel is not None and sel.size != q * r:
            raise ValueError(f"the selection mask must be [{q}, {r}]")
        tg = _u32(targets) if targets is not None else None
        if tg is not None and tg.size != q:
            raise ValueError(f"targets must have one entry per question ({q})")
        res = BackwardResult(np.empty(max(1, q * r), np.float32), np.empty(max(1, q), np.float32), 0.0,
                             np.empty(h * h, np.float32), np.empty(h * h, np.float32), np.empty(2 * h, np.float32),
                             np.empty(max(1, t) * h, np.float32), np.empty(3 * h, np.float32))
        out = abi.KcBackwardOut(res.policy.ctypes.data, res.value_prediction.ctypes.data, 0.0,
                                res.d_selector_wq.ctypes.data, res.d_selector_wk.ctypes.data, res.d_pool.ctypes.data,
                                res.d_field_states.ctypes.data, res.d_value_wv.ctypes.data, res.policy.size,
                                res.value_prediction.size, max(1, t), 0, 0, 0)
        abi.check(self._lib.kc_backward(self._h, C.byref(fv), abi.ptr(sel), abi.ptr(tg),
                                        int(valence_target is not None), float(valence_target or 0.0),
                                        C.byref(out)), self._h)
        res.policy = res.policy[:out.q * out.r]
        res.value_prediction = res.value_prediction[:out.q]
        res.d_field_states = res.d_field_states[:out.t * h]
        res.value_loss = out.value_loss
        return res

    def backward_batch_device(self, frames: int, records: int, rec_off: int, token_ids: int, field_roles: int,
                              schema_ids: int, band_ids: int, selection: int | None = None,
                              targets: int | None = None, valence: int | None = None,
                              schema_allow: int | None = None,
                              band_allow: int | None = None) -> abi.KcBackwardResult:
        """The backward of a device-resident batch (raw device pointers);
        results stay on the device (library-owned, valid until the next call)."""
        bv = abi.KcBatchView(frames, records, rec_off, token_ids, field_roles, schema_ids, band_ids, schema_allow,
                             band_allow, None)
        res = abi.KcBackwardResult()
        abi.check(self._lib.kc_backward_batch_device(self._h, C.byref(bv), selection, targets, valence,
                                                     C.byref(res)), self._h)
        return res

    def learn_frame_stats(self, targets: int | None, stats: int) -> None:
        """kc_learn_frame_stats over the last batch differentiated (device pointers)."""
        abi.check(self._lib.kc_learn_frame_stats(self._h, targets, stats), self._h)

    def learn_accumulate(self, step: int, value_weight: int, sums: int) -> None:
        """kc_learn_accumulate over the last batch differentiated (device pointers)."""
        abi.check(self._lib.kc_learn_accumulate(self._h, step, value_weight, sums), self._h)

    def learn_plan(self, rows: int, frames: int, options: abi.KcLearnOptions, step: int, value_weight: int,
                   pending: int, report: int) -> None:
        """kc_learn_plan (device pointers)."""
        abi.check(self._lib.kc_learn_plan(self._h, rows, frames, C.byref(options), step, value_weight, pending,
                                          report), self._h)

    def learn_accumulate_rows(self, token_ids: int, field_roles: int, step: int, pending: int, row_sums: int,
                              touched: int) -> None:
        """kc_learn_accumulate_rows over the last batch differentiated (device pointers)."""
        abi.check(self._lib.kc_learn_accumulate_rows(self._h, token_ids, field_roles, step, pending, row_sums,
                                                     touched), self._h)

    def learn_apply(self, sums: int, row_sums: int | None, touched: int | None, report: int,
                    options: abi.KcLearnOptions) -> np.ndarray:
        """kc_learn_apply: the update on the device's weight page; returns the
        KC_LEARN_RESULT values (host)."""
        out = np.zeros(abi.KC_LEARN_RESULT, np.float64)
        abi.check(self._lib.kc_learn_apply(self._h, sums, row_sums, touched, report, C.byref(options),
                                           out.ctypes.data), self._h)
        return out

    def copy_weights(self, offset: int, out: np.ndarray) -> None:
        """The device weight page from `offset` into the float32 array `out`."""
        if out.dtype != np.float32 or not out.flags.c_contiguous:
            raise ValueError("out must be a contiguous float32 array")
        abi.check(self._lib.kc_copy_weights(self._h, offset, out.size, out.ctypes.data), self._h)

    def load_checkpoint(self, data) -> str | None:
        """A KRY1 checkpoint straight into the device weight page
        (kc_load_checkpoint); None when taken up, else the refusal."""
        buf = np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)
        refusal = C.c_int()
        abi.check(self._lib.kc_load_checkpoint(self._h, buf.ctypes.data if buf.size else None, buf.size,
                                               C.byref(refusal)), self._h)
        return abi.CHECKPOINT_REFUSALS.get(refusal.value)

    def save_checkpoint(self) -> bytes:
        """KRY1 bytes of the device weight page (kc_save_checkpoint)."""
        n = C.c_uint64()
        self._lib.kc_save_checkpoint(self._h, None, 0, C.byref(n))
        out = np.empty(n.value, dtype=np.uint8)
        abi.check(self._lib.kc_save_checkpoint(self._h, out.ctypes.data, out.size, C.byref(n)), self._h)
        return out.tobytes()

    # --- seam extension: the selector on the device -------------------------
    def select(self, encoded: EncodedFrame, mask: np.ndarray | None = None, rule: MaskRule | None = None,
               bank_schema_ids=None, bank_band_ids=None, uniforms=None, gather: bool = True) -> Selection:
        h = self.config.hidden_size
        qo, bk, bvv = _f32(encoded.query_output), _f32(encoded.bank_keys), _f32(encoded.bank_values)
        q, r = qo.size // h, bk.size // h
        ev = abi.KcEncodedView(q, r, qo.ctypes.data, bk.ctypes.data if r else None, bvv.ctypes.data if r else None)
        p = np.empty(max(1, q * r), dtype=np.float32)
        idx = np.empty(max(1, q), dtype=np.uint32)
        g = np.empty(max(1, q * h), dtype=np.float32) if gather else None
        m = _f32(mask) if mask is not None else None
        if m is not None and m.size != q * r:
            raise ValueError(f"the selection mask must be [{q}, {r}]")
        rule_s = None
        keep = []
        if rule is not None:
            sa, ba, bs, bb = _u32(rule.schema_allow), _u32(rule.band_allow), _u32(bank_schema_ids), \
                _u32(bank_band_ids)
            keep += [sa, ba, bs, bb]
            rule_s = abi.KcMaskRule(sa.ctypes.data, ba.ctypes.data, bs.ctypes.data, bb.ctypes.data)
        u = np.ascontiguousarray(uniforms, dtype=np.float64) if uniforms is not None else None
        abi.check(self._lib.kc_select(self._h, C.byref(ev), abi.ptr(m), C.byref(rule_s) if rule_s else None,
                                      abi.ptr(u), p.ctypes.data, idx.ctypes.data, abi.ptr(g)), self._h)
        return Selection(p[:q * r], idx[:q], g[:q * h] if g is not None else None)

    def select_noalloc(self, q: int, r: int, query_output: int, bank_keys: int, bank_values: int | None,
                       mask: int | None, p: int, index: int, gather: int | None = None) -> None:
        """kc_select_noalloc: the selector on caller-owned DEVICE buffers (raw
        pointers), with no device allocation; queued on the handle's stream."""
        abi.check(self._lib.kc_select_noalloc(self._h, q, r, query_output, bank_keys, bank_values, mask, p, index,
                                              gather), self._h)

    # --- packed ragged batches ------------------------------------------------
    def forward_batch(self, batch: FrameBatch, rule: MaskRule | None = None, uniforms=None,
                      want_query_output: bool = False, p_capacity: int | None = None, word_ids=None,
                      word_alpha: float = 0.0, out: dict | None = None, mask=None) -> dict:
        """Pack, encode and select a whole batch; host arrays in and out.
        word_ids [records*8] / word_alpha: the same-word bias (WordBias).
        mask: an explicit selection mask laid out like p (frame f's [Q_f, R_f]
        block at p_off[f]; NEG_INF blocked, 0 open), for a grammar that is not
        a schema x band rule; exclusive with `rule`.
        out: caller-owned result arrays to fill instead of fresh ones — "p"
        (f32), "index" (u32), "p_off" and "q_off" (u64, frames + 1), e.g.
        pinned buffers reused across calls; p and index set the capacities."""
        keep = [_u32(batch.token_ids), _u32(batch.field_roles), _u32(batch.schema_ids), _u32(batch.band_ids),
                np.ascontiguousarray(batch.rec_off, dtype=np.uint64)]
        tok, role, sch, band, off = keep
        sa = ba = u = None
        if rule is not None:
            sa, ba = _u32(rule.schema_allow), _u32(rule.band_allow)
        if uniforms is not None:
            u = np.ascontiguousarray(uniforms, dtype=np.float64)
        wid = _u32(word_ids) if word_ids is not None else None
        if wid is not None and wid.size != batch.records * 8:
            raise ValueError("word_ids must hold one label per token slot (records * 8)")
        m = _f32(mask) if mask is not None else None
        bv = abi.KcBatchView(batch.frames, batch.records, off.ctypes.data, tok.ctypes.data, role.ctypes.data,
                             sch.ctypes.data, band.ctypes.data, abi.ptr(sa), abi.ptr(ba), abi.ptr(u), abi.ptr(wid),
                             float(word_alpha), abi.ptr(m))
        nq = int((band == 5).sum()) if out is None or want_query_output else 0
        if p_capacity is None and out is None:
            rec = np.diff(off.astype(np.int64))
            fid = np.repeat(np.arange(batch.frames), rec)
            isq = np.bincount(fid, weights=(band == 5), minlength=batch.frames).astype(np.int64)
            p_capacity = int((isq * (rec - isq)).sum())
        if out is not None:
            p, idx, p_off, q_off = out["p"], out["index"], out["p_off"], out["q_off"]
            for a, dt in ((p, np.float32), (idx, np.uint32), (p_off, np.uint64), (q_off, np.uint64)):
                if a.dtype != dt or not a.flags.c_contiguous:
                    raise ValueError("out arrays must be contiguous p f32, index u32, p_off / q_off u64")
            if p_off.size < batch.frames + 1 or q_off.size < batch.frames + 1:
                raise ValueError("out p_off / q_off need frames + 1 entries")
        else:
            p = np.empty(max(1, p_capacity), dtype=np.float32)
            idx = np.empty(max(1, nq), dtype=np.uint32)
            p_off = np.empty(batch.frames + 1, dtype=np.uint64)
            q_off = np.empty(batch.frames + 1, dtype=np.uint64)
        qo = np.empty(max(1, nq) * self.config.hidden_size, dtype=np.float32) if want_query_output else None
        bo = abi.KcBatchOut(p.ctypes.data, p.size, idx.ctypes.data, idx.size, p_off.ctypes.data, q_off.ctypes.data,
                            abi.ptr(qo), 0, 0, 0, 0)
        abi.check(self._lib.kc_forward_batch(self._h, C.byref(bv), C.byref(bo)), self._h)
        res = {"p": p[:bo.total_p], "index": idx[:bo.total_q], "p_off": p_off, "q_off": q_off,
               "total_t": bo.total_t, "total_r": bo.total_r}
        self._last_batch_sizes = (int(bo.total_p), int(bo.total_q), batch.frames)
        if qo is not None:
            res["query_output"] = qo[:bo.total_q * self.config.hidden_size]
        return res

    def select_batch(self, rule: MaskRule | None = None, uniforms=None, out: dict | None = None,
                     mask=None) -> dict:
        """kc_select_batch: the last forward_batch's batch selected again under
        `rule` and/or `uniforms` (per question), without encoding it again
        (consider once, choose many: host/session.ts:128-176). `out` as for
        forward_batch; without it the result arrays are sized from that batch."""
        sa = ba = u = None
        if rule is not None:
            sa, ba = _u32(rule.schema_allow), _u32(rule.band_allow)
        if uniforms is not None:
            u = np.ascontiguousarray(uniforms, dtype=np.float64)
        m = _f32(mask) if mask is not None else None
        sv = abi.KcBatchSelectView(abi.ptr(sa), abi.ptr(ba), abi.ptr(u), abi.ptr(m))
        if out is None:
            last = getattr(self, "_last_batch_sizes", None)
            if last is None:
                raise RuntimeError("no batch has been run through forward_batch on this backend")
            p_cap, nq, frames = last
            out = {"p": np.empty(max(1, p_cap), np.float32), "index": np.empty(max(1, nq), np.uint32),
                   "p_off": np.empty(frames + 1, np.uint64), "q_off": np.empty(frames + 1, np.uint64)}
        p, idx, p_off, q_off = out["p"], out["index"], out["p_off"], out["q_off"]
        bo = abi.KcBatchOut(p.ctypes.data, p.size, idx.ctypes.data, idx.size, p_off.ctypes.data, q_off.ctypes.data,
                            None, 0, 0, 0, 0)
        abi.check(self._lib.kc_select_batch(self._h, C.byref(sv), C.byref(bo)), self._h)
        return {"p": p[:bo.total_p], "index": idx[:bo.total_q], "p_off": p_off, "q_off": q_off,
                "total_t": bo.total_t, "total_r": bo.total_r}

    def forward_batch_device(self, frames: int, records: int, rec_off: int, token_ids: int, field_roles: int,
                             schema_ids: int, band_ids: int, schema_allow: int | None = None,
                             band_allow: int | None = None, uniforms: int | None = None,
                             word_ids: int | None = None, word_alpha: float = 0.0,
                             mask: int | None = None) -> abi.KcDeviceResult:
        """Device-resident batch (raw device pointers); results stay on the device."""
        bv = abi.KcBatchView(frames, records, rec_off, token_ids, field_roles, schema_ids, band_ids, schema_allow,
                             band_allow, uniforms, word_ids, float(word_alpha), mask)
        res = abi.KcDeviceResult()
        abi.check(self._lib.kc_forward_batch_device(self._h, C.byref(bv), C.byref(res)), self._h)
        return res

    # --- plumbing -------------------------------------------------------------
    def set_stream(self, stream_ptr: int | None) -> None:
        abi.check(self._lib.kc_set_stream(self._h, stream_ptr), self._h)

    def stream_ptr(self) -> int:
        """The cudaStream_t the handle launches on (kc_get_stream)."""
        return int(self._lib.kc_get_stream(self._h) or 0)

    def synchronize(self) -> None:
        abi.check(self._lib.kc_synchronize(self._h), self._h)

    def set_precision(self, mode: int | str, tau: float = 0.0) -> None:
        """KC_PRECISION_EXACT / CERTIFIED (default) / FAST for the batch entry points."""
        modes = {"exact": abi.KC_PRECISION_EXACT, "certified": abi.KC_PRECISION_CERTIFIED,
                 "fast": abi.KC_PRECISION_FAST}
        m = modes[mode] if isinstance(mode, str) else int(mode)
        abi.check(self._lib.kc_set_precision(self._h, m, float(tau)), self._h)

    def inject_wait_expiry(self, kernel: str) -> None:
        """Test hook (kc_inject_wait_expiry): the next launch of the named
        tensor-core kernel ("attn", "ffn" or "gemm") reports an expired
        bounded wait before it issues any copy; the batch call then fails
        with KC_ERR_TIMEOUT and the handle stays usable."""
        k = {"attn": abi.KC_INJECT_ATTN, "ffn": abi.KC_INJECT_FFN, "gemm": abi.KC_INJECT_GEMM,
             "exact_gemm": abi.KC_INJECT_EXACT_GEMM}[kernel]
        abi.check(self._lib.kc_inject_wait_expiry(self._h, k), self._h)

    def profile(self, enable: bool) -> None:
        abi.check(self._lib.kc_profile(self._h, int(enable)), self._h)

    def profile_read(self, reset: bool = False) -> dict:
        st = abi.KcStageTimes()
        abi.check(self._lib.kc_profile_read(self._h, C.byref(st), int(reset)), self._h)
        return st.as_dict()

    def launch_count(self) -> int:
        return int(self._lib.kc_launch_count(self._h))

    def __del__(self):
        try:
            self.destroy()
        except Exception:
            pass


def cuda_backend(device: int = 0) -> Callable[[BrainForwardConfig, BrainForwardWeights], CudaBrainBackend]:
    """BrainBackendFactory for the CUDA backend (cf. gpuBackend, webgpu/src/backend.ts:174-181)."""
    return lambda config, weights: CudaBrainBackend(config, weights, device)
