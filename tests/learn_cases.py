"""Seeded learn batches shared by the CPU and GPU learn tests: experiences
(records, chosen slots, rewards, a grammar) and the same experiences in the
form the oracle's learn restatement takes."""
import numpy as np

from krystal_b200.frame import pack_host_frame
from krystal_b200.learn import HostExperience
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights
from krystal_b200.session import selection_mask


def world(seed=3):
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 97)
    return cfg, create_brain_forward_weights(cfg, seed)


def experiences(n=6, seed=5, questions=(1, 4), bank=(3, 12), skip_reward=(), no_choice=()):
    rng = np.random.default_rng(seed)
    out = []
    for e in range(n):
        nb = int(rng.integers(bank[0], bank[1] + 1))
        nq = int(rng.integers(questions[0], questions[1] + 1))
        recs = [dict(schemaId=int(rng.integers(0, 8)), band=int(rng.choice([0, 1, 2, 3])),
                     tokens=[int(t) for t in rng.integers(1, 90, rng.integers(1, 9))]) for _ in range(nb)]
        qpos = sorted(rng.choice(nb + nq, nq, replace=False).tolist())
        for p in qpos:
            recs.insert(p, dict(query=True, tokens=[int(t) for t in rng.integers(1, 90, rng.integers(1, 5))]))
        bank_slots = [i for i in range(len(recs)) if not recs[i].get("query")]
        chosen = [int(rng.choice(bank_slots)) if rng.random() < 0.8 else -1 for _ in range(nq)]
        if e in no_choice:
            chosen = None
        k = int(rng.integers(1, 4))
        allows = (lambda kk: (lambda q, slot: (q + slot) % kk != 0))(k)
        reward = None if e in skip_reward else float(rng.normal())
        out.append(HostExperience(recs, reward, chosen, allows))
    return out


def oracle_experiences(exps):
    out = []
    for ex in exps:
        frame = pack_host_frame(ex.records)
        out.append(dict(frame=frame.gpu, chosen=ex.chosen, reward=ex.reward,
                        mask=selection_mask(frame.active, ex.allows)))
    return out
