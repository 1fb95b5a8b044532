"""teachFromDemonstration (packages/krystal/src/host/teach.ts:126-272)
restated on the CPU oracle's backward, for checking the device teach path.

TEST INFRASTRUCTURE ONLY: the checker. Imported by tests/ — never by the
product package.

One demonstration = a packed frame, per question the gold slot (or None) and
the forbidden slot (or None), and the selection mask it is shown under. The
weight page is updated the way the reference updates its Float32Arrays: f64
arithmetic, f32 store, element after element in the reference's loop order,
each showing applied before the next is differentiated.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import oracle as O

NO_TARGET = 0xFFFFFFFF
AWAY = 0x80000000


@dataclass
class Options:
    learning_rate: float = 0.2       # teach.ts:133
    token_rate: float = 0.5          # :134
    unfreeze_tokens: bool = True     # :135
    max_update_abs: float = 0.05     # :136
    decay: float = 1e-3              # :137
    max_parameter_abs: float = 1.0   # :138


def _f32(x: float) -> float:
    return float(np.float32(x))


def teach_from_demonstration(config, page: np.ndarray, demonstrations, options: Options = Options()):
    """Returns the updated page (a copy) and the TeachReport fields."""
    h = config.hidden_size
    page = page.copy()
    off = {k: O.weight_offset(config, k) for k in O.WEIGHT_PARTS}
    wq = page[off["selector_wq"]:off["selector_wq"] + h * h]
    wk = page[off["selector_wk"]:off["selector_wk"] + h * h]
    base_tok = off["embeddings"]
    base_field = base_tok + config.token_space * h
    tr = np.asarray(config.token_rows, np.int64)
    lr, token_rate = options.learning_rate, options.token_rate
    keep = 1 - options.decay
    seen = shown = rejected = clipped = 0
    agreement = 0.0
    touched = 0.0
    for demo in demonstrations:
        frame = demo["frame"]
        act = O.compile_active(frame.token_ids, frame.band_ids, frame.active_record_indices)
        queries, bank = act["query_records"].size, act["bank_records"].size
        if not queries or not bank:
            continue
        bank_slots = act["bank_records"].tolist()
        targets = np.full(queries, NO_TARGET, np.uint32)
        answered = False
        for q in range(queries):
            slot = demo["gold"][q] if q < len(demo["gold"]) else None
            forbidden = demo.get("forbidden")
            not_ = forbidden[q] if forbidden is not None and q < len(forbidden) else None
            toward = slot is not None and slot >= 0
            chosen = slot if toward else not_
            if chosen is None or chosen < 0 or chosen not in bank_slots:
                continue
            row = bank_slots.index(chosen)
            targets[q] = row if toward else (row | AWAY)
            answered = True
        if not answered:
            continue
        res = O.backward(config, page, frame, np.ascontiguousarray(demo["mask"], np.float32), targets, None)
        pol = res["policy"]
        for q in range(queries):
            t = int(targets[q])
            if t == NO_TARGET:
                continue
            on = float(pol[q * bank + (t & ~AWAY)])
            if not math.isfinite(on):
                continue
            agreement += (1 - on) if t & AWAY else on
            shown += 1
        tokens = act["active_tokens"]
        rows = []
        if options.unfreeze_tokens:
            for ft in tokens:
                for r in (base_tok + int(tr[frame.token_ids[ft]]) * h, base_field + int(tr[frame.field_roles[ft]]) * h):
                    if r not in rows:
                        rows.append(r)
        before = (wq.copy(), wk.copy(), [(r, page[r:r + h].copy()) for r in rows])
        dq, dk, ds = res["d_selector_wq"], res["d_selector_wk"], res["d_field_states"]
        asked = 0.0
        for i in range(dq.size):
            asked = max(asked, abs(lr * float(dq[i])))
        for i in range(dk.size):
            asked = max(asked, abs(lr * float(dk[i])))
        if options.unfreeze_tokens:
            for i in range(tokens.size * h):
                asked = max(asked, abs(lr * token_rate * float(ds[i])))
        scale = options.max_update_abs / asked if asked > options.max_update_abs else 1
        if scale < 1:
            clipped += 1
        written = 0.0

        def note(v: float) -> None:  # Math.max carries NaN through
            nonlocal written
            written = math.nan if (math.isnan(written) or math.isnan(v)) else max(written, abs(v))

        for w, d in ((wq, dq), (wk, dk)):
            for i in range(w.size):
                w[i] = _f32(float(w[i]) * keep - scale * lr * float(d[i]))
                note(float(w[i]))
        if options.unfreeze_tokens:
            step = scale * lr * token_rate
            for r in rows:
                for d in range(h):
                    page[r + d] = _f32(float(page[r + d]) * keep)
            for t, ft in enumerate(tokens):
                tok = base_tok + int(tr[frame.token_ids[ft]]) * h
                role = base_field + int(tr[frame.field_roles[ft]]) * h
                for d in range(h):
                    grad = step * float(ds[t * h + d])
                    page[tok + d] = _f32(float(page[tok + d]) - grad)
                    page[role + d] = _f32(float(page[role + d]) - grad)
                    note(float(page[tok + d]))
                    note(float(page[role + d]))
        if not math.isfinite(written) or written > options.max_parameter_abs:
            wq[:], wk[:] = before[0], before[1]
            for r, v in before[2]:
                page[r:r + h] = v
            rejected += 1
            continue
        touched = max(touched, written)
        seen += 1
    return page, dict(frames_seen=seen, shown=shown, mean_agreement=agreement / shown if shown else 0.0,
                      max_parameter_abs=touched, rejected=rejected, clipped=clipped)
