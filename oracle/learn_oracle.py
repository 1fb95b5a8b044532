"""learnFromExperience (packages/krystal/src/host/learn.ts:280-512) restated
on the CPU oracle's backward, for checking the device learn step.

TEST INFRASTRUCTURE ONLY: the checker. Imported by tests/ and by the
benchmark's CPU-baseline leg and reference arm — never by the product package.

One experience = a packed frame, the slot each question chose (or -1), the
reward (None = the experience is skipped, learn.ts:320) and the selection mask
it was asked under (selectionMask, learn.ts:215-232). The weight page is
updated the way the reference updates its Float32Arrays: f64 arithmetic,
f32 store, frame after frame in batch order.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from . import oracle as O

NO_TARGET = 0xFFFFFFFF
NEG_INF = np.float32(-1e30)


@dataclass
class Options:
    learning_rate: float = 0.05   # learn.ts:292
    policy_scale: float = 1.0     # :293
    advantage_clip: float = 3.0   # :294
    max_parameter_abs: float = math.inf  # :295
    unfreeze_pool: bool = False   # :297
    unfreeze_tokens: bool = False  # :298
    token_rate: float = 0.1       # :299


def _f32_update(dst: np.ndarray, delta: np.ndarray) -> None:
    """dst[i] = dst[i] - delta[i] in f64, stored f32 (a Float32Array write)."""
    dst[:] = (dst.astype(np.float64) - delta).astype(np.float32)


def _max_abs(a: np.ndarray) -> float:
    a = np.abs(a.astype(np.float64))
    if not np.all(np.isfinite(a)):
        return math.inf
    return float(a.max()) if a.size else 0.0


def learn_from_experience(config, page: np.ndarray, experiences, options: Options = Options(),
                          threads: int = 0) -> tuple[np.ndarray, dict]:
    """Returns the updated weight page (a copy) and the LearnReport fields.
    threads > 1 runs the per-frame backwards on that many threads. With
    unfreeze_tokens the token and field rows of the answered frames move too
    (scatterEmbeddings, learn.ts:242-263, frame after frame, token after
    token, each write rounded to f32), and join the health check and the
    rollback (:401-425, :477-495)."""
    h = config.hidden_size
    page = page.copy()
    off = {k: O.weight_offset(config, k) for k in O.WEIGHT_PARTS}
    wq = page[off["selector_wq"]:off["selector_wq"] + h * h]
    wk = page[off["selector_wk"]:off["selector_wk"] + h * h]
    wv = page[off["value_head"]:off["value_head"] + 3 * h]
    pool = page[off["pool"]:off["pool"] + 2 * h]
    lr, clip = options.learning_rate, options.advantage_clip
    pending = []
    d_value = np.zeros(3 * h, np.float32)
    seen = 0
    adv_total = loss_total = ent_total = conf_total = 0.0
    ent_rows = conf_rows = 0
    # Every frame is differentiated against the weights as they stand before
    # the update (the gradients are collected first, learn.ts:349-357), so the
    # per-frame backwards may run in parallel; the host logic then walks the
    # frames in order.
    work = []
    for ex in experiences:
        if ex["reward"] is None:
            continue
        frame = ex["frame"]
        act = O.compile_active(frame.token_ids, frame.band_ids, frame.active_record_indices)
        q, r = act["query_records"].size, act["bank_records"].size
        if not q or not r:
            continue
        bank = act["bank_records"].tolist()
        targets = np.full(q, NO_TARGET, np.uint32)
        answered = False
        chosen = ex.get("chosen") or []
        for i in range(q):
            slot = chosen[i] if i < len(chosen) else None
            if slot is None or slot < 0 or slot not in bank:
                continue
            targets[i] = bank.index(slot)
            answered = True
        mask = np.ascontiguousarray(ex["mask"], np.float32)
        work.append((ex, q, r, targets, answered, mask))

    def diff(item):
        ex, _, _, targets, answered, mask = item
        return O.backward(config, page, ex["frame"], mask, targets if answered else None, float(ex["reward"]))

    if threads > 1 and len(work) > 1:
        from concurrent.futures import ThreadPoolExecutor
        with ThreadPoolExecutor(threads) as workers:
            results = list(workers.map(diff, work))
    else:
        results = [diff(item) for item in work]
    for (ex, q, r, targets, answered, mask), res in zip(work, results):
        pred = res["value_prediction"]
        baseline = 0.0
        for v in pred:
            baseline += float(v)
        baseline = baseline / pred.size if pred.size else 0.0
        advantage = float(ex["reward"]) - baseline
        d_value[:] = (d_value.astype(np.float64) + res["d_value_wv"]).astype(np.float32)
        if answered and math.isfinite(advantage):
            pending.append((advantage, res["d_selector_wq"], res["d_selector_wk"], res["d_pool"],
                            (ex["frame"], res["d_field_states"]) if options.unfreeze_tokens else None))
        pol = res["policy"]
        for i in range(q):
            allowed, ent = 0, 0.0
            for j in range(r):
                p = float(pol[i * r + j])
                if mask[i * r + j] <= NEG_INF / 2:
                    continue
                allowed += 1
                if p > 0:
                    ent -= p * math.log(p)
            if allowed > 1:
                ent_total += ent / math.log(allowed)
                ent_rows += 1
            if targets[i] != NO_TARGET:
                conf_total += float(pol[i * r + int(targets[i])])
                conf_rows += 1
        adv_total += advantage
        loss_total += res["value_loss"]
        seen += 1
    # the rows this batch can move (:401-414): token and field rows of the answered frames
    base_tok = O.weight_offset(config, "embeddings")
    base_field = base_tok + config.token_space * h
    rows_hit = set()
    if options.unfreeze_tokens:
        tr = np.asarray(config.token_rows, np.int64)
        for *_, emb in pending:
            frame, _ = emb
            act = O.compile_active(frame.token_ids, frame.band_ids, frame.active_record_indices)
            for ft in act["active_tokens"]:
                rows_hit.add(base_tok + int(tr[frame.token_ids[ft]]) * h)
                rows_hit.add(base_field + int(tr[frame.field_roles[ft]]) * h)
    touched = sorted(rows_hit)
    before = page.copy()
    if seen:
        wv[:] = (wv.astype(np.float64) - (lr * d_value.astype(np.float64)) / seen).astype(np.float32)
    reinforced = discouraged = 0
    actor_moved = False
    if pending:
        mean = 0.0
        for a, *_ in pending:
            mean += a
        mean /= len(pending)
        var = 0.0
        for a, *_ in pending:
            var += (a - mean) ** 2
        var /= len(pending)
        dev = math.sqrt(var)
        if dev > 1e-6:
            actor_moved = True
            for a, gq, gk, gp, emb in pending:
                st = max(-clip, min(clip, (a - mean) / dev))
                step = (lr * options.policy_scale * st) / len(pending)
                _f32_update(wq, step * gq.astype(np.float64))
                _f32_update(wk, step * gk.astype(np.float64))
                if options.unfreeze_pool:
                    _f32_update(pool, step * gp.astype(np.float64))
                if emb is not None:  # scatterEmbeddings(..., step * tokenRate)
                    frame, ds = emb
                    act = O.compile_active(frame.token_ids, frame.band_ids, frame.active_record_indices)
                    tr = np.asarray(config.token_rows, np.int64)
                    s_tok = step * options.token_rate
                    for t, ft in enumerate(act["active_tokens"]):
                        g = s_tok * ds[t * h:(t + 1) * h].astype(np.float64)
                        for row in (base_tok + int(tr[frame.token_ids[ft]]) * h,
                                    base_field + int(tr[frame.field_roles[ft]]) * h):
                            _f32_update(page[row:row + h], g)
                if st > 0:
                    reinforced += 1
                elif st < 0:
                    discouraged += 1
    sel_max = max(_max_abs(wq), _max_abs(wk))
    sem = max((_max_abs(page[r:r + h]) for r in touched), default=0.0)
    health = dict(semantic_embedding_max_abs=sem, selector_max_abs=sel_max, value_max_abs=_max_abs(wv),
                  pool_max_abs=_max_abs(pool))
    finite = all(math.isfinite(v) for v in health.values())
    over = any(v > options.max_parameter_abs for v in health.values())
    rejected = "non-finite" if not finite else "parameter-limit" if over else None
    if rejected:
        page = before
        wq, wk = (page[off[k]:off[k] + h * h] for k in ("selector_wq", "selector_wk"))
        wv = page[off["value_head"]:off["value_head"] + 3 * h]
        pool = page[off["pool"]:off["pool"] + 2 * h]
        health = dict(semantic_embedding_max_abs=max((_max_abs(page[r:r + h]) for r in touched), default=0.0),
                      selector_max_abs=max(_max_abs(wq), _max_abs(wk)), value_max_abs=_max_abs(wv),
                      pool_max_abs=_max_abs(pool))
    report = dict(frames_seen=seen, mean_advantage=adv_total / seen if seen else 0.0,
                  mean_value_loss=loss_total / seen if seen else 0.0, reinforced=reinforced,
                  discouraged=discouraged, mean_entropy=ent_total / ent_rows if ent_rows else 0.0,
                  mean_confidence=conf_total / conf_rows if conf_rows else 0.0,
                  update_applied=seen > 0 and not rejected, rejected=rejected, actor_moved=actor_moved,
                  health=health)
    return page, report
