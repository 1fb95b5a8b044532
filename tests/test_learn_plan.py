"""plan_update (the scalar half of learnFromExperience) against a plain loop
restatement of learn.ts:318-470, on adversarial batches: NaN rewards (skipped
experiences), zero and negative-zero statistics, infinite advantages, equal
advantages (no actor step) and magnitudes far apart. The vectorised form
must give the same bits: its sums are running sums in frame order, as the
reference's loops take them."""
import math

import numpy as np

from krystal_b200 import learn as L


def plan_loop(stats, rewards, answered, opts):
    F = rewards.size
    step = np.zeros(F)
    value_weight = np.zeros(F)
    pending = []
    seen = 0
    adv_total = loss_total = ent_total = conf_total = ent_rows = conf_rows = 0.0
    for f in range(F):
        reward = float(rewards[f])
        if math.isnan(reward) or not stats[f, 0] or not stats[f, 1]:
            continue
        advantage = reward - float(stats[f, 2])
        value_weight[f] = 1.0
        if answered[f] and math.isfinite(advantage):
            pending.append((f, advantage))
        ent_total += stats[f, 4]
        ent_rows += stats[f, 5]
        conf_total += stats[f, 6]
        conf_rows += stats[f, 7]
        adv_total += advantage
        loss_total += float(stats[f, 3])
        seen += 1
    reinforced = discouraged = 0
    moved = False
    if pending:
        mean = 0.0
        for _, a in pending:
            mean += a
        mean /= len(pending)
        var = 0.0
        for _, a in pending:
            var += (a - mean) * (a - mean)
        var /= len(pending)
        dev = math.sqrt(var)
        if dev > 1e-6:
            moved = True
            for f, a in pending:
                st = max(-opts.advantage_clip, min(opts.advantage_clip, (a - mean) / dev))
                step[f] = (opts.learning_rate * opts.policy_scale * st) / len(pending)
                reinforced += st > 0
                discouraged += st < 0
    return (step, value_weight, seen, moved, reinforced, discouraged,
            adv_total / seen if seen else 0.0, loss_total / seen if seen else 0.0,
            ent_total / ent_rows if ent_rows else 0.0, conf_total / conf_rows if conf_rows else 0.0)


def same_float(x, y):
    if math.isnan(x) and math.isnan(y):
        return True
    return x == y and math.copysign(1.0, x) == math.copysign(1.0, y)


def test_vectorised_plan_equals_the_loop():
    opts = L.LearnOptions()
    rng = np.random.default_rng(3)
    for trial in range(400):
        F = int(rng.integers(0, 200))
        stats = rng.standard_normal((F, L.STATS)) * rng.choice([1e-3, 1.0, 1e3])
        stats[rng.random((F, L.STATS)) < 0.1] = 0.0
        stats[rng.random((F, L.STATS)) < 0.03] = -0.0
        rewards = rng.standard_normal(F) * rng.choice([1e-6, 1.0, 10.0])
        rewards[rng.random(F) < 0.1] = np.nan
        if trial % 7 == 0 and F:
            rewards[:] = 1.0
            stats[:, 2] = 0.5
        if trial % 11 == 0 and F:
            stats[rng.random(F) < 0.05, 2] = np.inf
        answered = rng.random(F) < 0.8
        got = L.plan_update(stats, rewards, answered, opts)
        want = plan_loop(stats, rewards, answered, opts)
        assert np.array_equal(got.step, want[0]) and np.array_equal(got.value_weight, want[1])
        assert (got.seen, got.actor_moved, got.reinforced, got.discouraged) == want[2:6]
        for x, y in zip((got.mean_advantage, got.mean_value_loss, got.mean_entropy, got.mean_confidence), want[6:]):
            assert same_float(x, y)
