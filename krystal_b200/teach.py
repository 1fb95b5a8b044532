"""teachFromDemonstration (packages/krystal/src/host/teach.ts:126-272) with the
CUDA backend as the gradient source.

Being shown an answer applies the pointer loss alone: no reward, no baseline,
no critic (teach.ts:1-21). Showings are sequential by contract: each one is
differentiated on the device (``kc_backward``: the frame's pointer-loss
gradients, in the oracle's exact arithmetic), its update is applied to the
host's arrays, and the backend takes up what moved (``kc_sync`` with the
selector and the touched embedding rows) before the next showing is
differentiated (teach.ts:120-125, 258-261). Several GPUs cannot share one
teaching pass; replicas teach separate sessions.

The update follows the reference element by element: the step capped so that
no weight moves by more than ``max_update_abs`` (one factor for the whole
update, :210-217), the touched weights decayed by ``1 - decay`` (the rows
once each, however many tokens read them), the token and field rows moved
token after token (each write rounded to f32, as a Float32Array store
rounds), and a showing whose largest written value is not finite or exceeds
``max_parameter_abs`` thrown away to the last weight (:246-255).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Sequence

import numpy as np

from . import abi
from .backend import CudaBrainBackend, WeightChanges
from .frame import pack_host_frame
from .model import BrainForwardWeights, embedding_table_bases
from .session import selection_mask

NO_TARGET = abi.KC_NO_TARGET
AWAY = abi.KC_AWAY_TARGET


@dataclass
class HostDemonstration:
    """HostDemonstration (teach.ts:29-46): the records, the slot each question
    should have chosen (None: nothing said), the slot it should not have
    chosen, and the grammar in force."""
    records: Sequence
    gold: Sequence[int | None]
    forbidden: Sequence[int | None] | None = None
    allows: Callable[[int, int], bool] | None = None


@dataclass
class TeachOptions:
    """TeachOptions (teach.ts:48-86) with the reference's defaults (:133-138)."""
    learning_rate: float = 0.2
    token_rate: float = 0.5
    unfreeze_tokens: bool = True
    max_update_abs: float = 0.05
    decay: float = 1e-3
    max_parameter_abs: float = 1.0


@dataclass
class TeachReport:
    """TeachReport (teach.ts:88-117)."""
    frames_seen: int
    shown: int
    mean_agreement: float
    max_parameter_abs: float
    rejected: int
    clipped: int


def _f32(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float32)


def teach_from_demonstration(demonstrations: Sequence[HostDemonstration], weights: BrainForwardWeights,
                             backend: CudaBrainBackend, options: TeachOptions = TeachOptions()) -> TeachReport:
    config = weights.config
    h = config.hidden_size
    bases = embedding_table_bases(config)
    rows_map = np.asarray(config.token_rows, np.int64)
    lr, token_rate = options.learning_rate, options.token_rate
    keep = 1.0 - options.decay
    table = weights.embeddings
    wq, wk = weights.selector.wq, weights.selector.wk
    seen = shown = rejected = clipped = 0
    agreement_total = 0.0
    touched = 0.0
    for demo in demonstrations:
        if not len(demo.records):
            continue
        frame = pack_host_frame(demo.records)
        act = frame.active
        queries, bank = act.query_records.size, act.bank_records.size
        if not queries or not bank:
            continue
        bank_slots = act.bank_records.tolist()
        targets = np.full(queries, NO_TARGET, np.uint32)
        answered = False
        for q in range(queries):
            slot = demo.gold[q] if q < len(demo.gold) else None
            not_ = demo.forbidden[q] if demo.forbidden is not None and q < len(demo.forbidden) else None
            toward = slot is not None and slot >= 0
            chosen = slot if toward else not_
            if chosen is None or chosen < 0 or chosen not in bank_slots:
                continue
            row = bank_slots.index(chosen)
            targets[q] = row if toward else (row | AWAY)
            answered = True
        if not answered:
            continue
        mask = selection_mask(act, demo.allows)
        res = backend.backward(frame, selection=mask, targets=targets)
        for q in range(queries):
            t = int(targets[q])
            if t == NO_TARGET:
                continue
            on = float(res.policy[q * bank + (t & ~AWAY)])
            if not math.isfinite(on):
                continue
            agreement_total += (1.0 - on) if t & AWAY else on
            shown += 1
        tokens = act.active_tokens
        g = frame.gpu
        tok_rows = bases.token + rows_map[g.token_ids[tokens]] * h
        role_rows = bases.field + rows_map[g.field_roles[tokens]] * h
        rows: list[int] = []
        if options.unfreeze_tokens:  # the Set's insertion order: token row, then role row, token by token
            seen_rows = set()
            for a, b in zip(tok_rows.tolist(), role_rows.tolist()):
                for r in (a, b):
                    if r not in seen_rows:
                        seen_rows.add(r)
                        rows.append(r)
        before = (wq.copy(), wk.copy(), [(r, table[r:r + h].copy()) for r in rows])
        dq = res.d_selector_wq.astype(np.float64)
        dk = res.d_selector_wk.astype(np.float64)
        dfs = res.d_field_states[:tokens.size * h].astype(np.float64).reshape(tokens.size, h)
        asked = max(float(np.abs(lr * dq).max(initial=0.0)), float(np.abs(lr * dk).max(initial=0.0)))
        if options.unfreeze_tokens and tokens.size:
            asked = max(asked, float(np.abs((lr * token_rate) * dfs).max()))
        scale = options.max_update_abs / asked if asked > options.max_update_abs else 1.0
        if scale < 1.0:
            clipped += 1
        wq[:] = _f32(wq.astype(np.float64) * keep - (scale * lr) * dq)
        wk[:] = _f32(wk.astype(np.float64) * keep - (scale * lr) * dk)
        written = max(float(np.abs(wq).max()), float(np.abs(wk).max()))
        if not (np.isfinite(wq).all() and np.isfinite(wk).all()):
            written = math.nan
        if options.unfreeze_tokens:
            step = scale * lr * token_rate
            for r in rows:  # decayed once per row
                table[r:r + h] = _f32(table[r:r + h].astype(np.float64) * keep)
            for t in range(tokens.size):
                grad = step * dfs[t]
                for r in (int(tok_rows[t]), int(role_rows[t])):
                    table[r:r + h] = _f32(table[r:r + h].astype(np.float64) - grad)
                    v = table[r:r + h]
                    if not np.isfinite(v).all():
                        written = math.nan
                    elif not math.isnan(written):
                        written = max(written, float(np.abs(v).max()))
        if not math.isfinite(written) or written > options.max_parameter_abs:
            wq[:], wk[:] = before[0], before[1]
            for r, v in before[2]:
                table[r:r + h] = v
            rejected += 1
            continue
        touched = max(touched, written)
        seen += 1
        # before the next showing is differentiated (teach.ts:258-261)
        backend.sync(weights, WeightChanges(selector=True, embedding_rows=rows))
    return TeachReport(seen, shown, agreement_total / shown if shown else 0.0, touched, rejected, clipped)
