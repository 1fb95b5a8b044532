"""The host half of the learn step (krystal_b200/learn.py) on the CPU.

plan_update + apply_update, fed per-frame readings and gradient sums computed
from the oracle's backward, must reproduce the oracle's restatement of
learnFromExperience (which updates frame after frame in f32); and the
several-rank exchange (gather of per-frame rows, all-reduce of gradient sums)
must give every rank the single-process answer (gloo, world size 2).
"""
import math
import os

import numpy as np
import pytest

from krystal_b200 import learn as L
from krystal_b200.model import BrainForwardWeights
from oracle import learn_oracle as LO
from tests.learn_cases import experiences, oracle_experiences, world

H = 128
TOL = 1e-4


def frame_readings(oracle, cfg, page, exps):
    """What kc_learn_frame_stats and kc_learn_accumulate read, from the oracle."""
    rows, grads = [], []
    for ex in oracle_experiences(exps):
        act = oracle.compile_active(ex["frame"].token_ids, ex["frame"].band_ids, ex["frame"].active_record_indices)
        q, r = act["query_records"].size, act["bank_records"].size
        bank = act["bank_records"].tolist()
        tg = np.full(q, L.NO_TARGET, np.uint32)
        for i, slot in enumerate(ex["chosen"] or []):
            if i < q and slot is not None and slot >= 0 and slot in bank:
                tg[i] = bank.index(slot)
        answered = bool((tg != L.NO_TARGET).any())
        reward = np.nan if ex["reward"] is None else ex["reward"]
        res = oracle.backward(cfg, page, ex["frame"], ex["mask"], tg if answered else None,
                              None if ex["reward"] is None else ex["reward"])
        pol, m = res["policy"], ex["mask"]
        et = er = ct = cr = 0.0
        for i in range(q):
            allowed, e = 0, 0.0
            for j in range(r):
                if m[i * r + j] <= L.NEG_INF / 2:
                    continue
                allowed += 1
                if pol[i * r + j] > 0:
                    e -= float(pol[i * r + j]) * math.log(float(pol[i * r + j]))
            if allowed > 1:
                et += e / math.log(allowed)
                er += 1
            if tg[i] != L.NO_TARGET:
                ct += float(pol[i * r + int(tg[i])])
                cr += 1
        base = float(np.sum(res["value_prediction"].astype(np.float64))) / q if q else 0.0
        rows.append([q, r, base, res["value_loss"], et, er, ct, cr, reward, float(answered)])
        grads.append((res["d_selector_wq"], res["d_selector_wk"], res["d_pool"], res["d_value_wv"]))
    return np.array(rows, np.float64), grads


def sums_of(plan, grads):
    out = np.zeros(2 * H * H + 5 * H)
    for f, (gq, gk, gp, gv) in enumerate(grads):
        out[:H * H] += plan.step[f] * gq
        out[H * H:2 * H * H] += plan.step[f] * gk
        out[2 * H * H:2 * H * H + 2 * H] += plan.step[f] * gp
        out[2 * H * H + 2 * H:] += plan.value_weight[f] * gv
    return out


@pytest.mark.parametrize("unfreeze_pool", [False, True])
def test_host_update_matches_oracle_learn(oracle, unfreeze_pool):
    cfg, w = world()
    exps = experiences(7, skip_reward=(2,), no_choice=(4,))
    opts = L.LearnOptions(unfreeze_pool=unfreeze_pool)
    want_page, want = LO.learn_from_experience(cfg, w.page, oracle_experiences(exps),
                                               LO.Options(unfreeze_pool=unfreeze_pool))
    rows, grads = frame_readings(oracle, cfg, w.page, exps)
    plan = L.plan_update(rows[:, :8], rows[:, 8], rows[:, 9] > 0, opts)
    got = BrainForwardWeights(cfg, w.page.copy())
    changes, rejected, _ = L.apply_update(got, sums_of(plan, grads), plan, opts)
    assert rejected is None and changes.value_head and changes.selector == want["actor_moved"]
    assert changes.pool == (unfreeze_pool and want["actor_moved"])
    assert np.abs(got.page.astype(np.float64) - want_page).max() <= TOL
    assert plan.seen == want["frames_seen"] and plan.reinforced == want["reinforced"]
    assert plan.discouraged == want["discouraged"]
    for k in ("mean_advantage", "mean_value_loss", "mean_entropy", "mean_confidence"):
        assert abs(getattr(plan, k) - want[k]) <= 1e-9, k


def test_rollback_restores_the_arrays(oracle):
    cfg, w = world()
    exps = experiences(5, seed=9)
    opts = L.LearnOptions(max_parameter_abs=1e-3)
    rows, grads = frame_readings(oracle, cfg, w.page, exps)
    plan = L.plan_update(rows[:, :8], rows[:, 8], rows[:, 9] > 0, opts)
    got = BrainForwardWeights(cfg, w.page.copy())
    changes, rejected, _ = L.apply_update(got, sums_of(plan, grads), plan, opts)
    assert changes is None and rejected == "parameter-limit"
    assert np.array_equal(got.page, w.page)
    _, want = LO.learn_from_experience(cfg, w.page, oracle_experiences(exps), LO.Options(max_parameter_abs=1e-3))
    assert want["rejected"] == "parameter-limit"


def test_equal_advantages_do_not_move_the_actor():
    stats = np.array([[2, 5, 0.25, 0.1, 0, 0, 0, 0]] * 3, np.float64)
    plan = L.plan_update(stats, np.array([1.0, 1.0, 1.0]), np.array([True] * 3), L.LearnOptions())
    assert not plan.actor_moved and not plan.step.any() and plan.seen == 3


def _rank(rank, world_size, port, rows, sums, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world_size)
    try:
        F = rows.shape[0]
        a, b = L.shard_bounds(F, world_size, rank)
        got_rows = L.gather_frame_rows(rows[a:b], F, None)
        total = L.all_reduce_sums(torch.from_numpy(sums[rank].copy()), None)
        q.put((rank, got_rows, total))
    finally:
        dist.destroy_process_group()


def test_two_rank_exchange_equals_one_process():
    import socket
    import torch.multiprocessing as mp
    rng = np.random.default_rng(0)
    rows = rng.normal(size=(7, 10))
    sums = rng.normal(size=(2, 2 * H * H + 5 * H))
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, rows, sums, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, got_rows, total in results:
        assert np.array_equal(got_rows, rows)
        assert np.allclose(total, sums.sum(0), rtol=0, atol=1e-12)
