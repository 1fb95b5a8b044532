"""Seeded demonstrations shared by the CPU and GPU teach tests, and the same
demonstrations in the form the oracle's teach restatement takes."""
import numpy as np

from krystal_b200.frame import pack_host_frame
from krystal_b200.session import selection_mask
from krystal_b200.teach import HostDemonstration


def demonstrations(n=3, seed=7, forbid=(1,), nothing=(), bank=(3, 10), questions=(1, 3)):
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
        gold = [int(rng.choice(bank_slots)) for _ in range(nq)]
        forbidden = None
        if e in forbid:  # the first question is told what not to choose instead
            forbidden = [int(rng.choice(bank_slots))] + [None] * (nq - 1)
            gold[0] = None
        if e in nothing:
            gold = [None] * nq
        k = int(rng.integers(1, 4))
        allows = (lambda kk: (lambda q, slot: (q + slot) % kk != 0))(k)
        out.append(HostDemonstration(recs, gold, forbidden, allows))
    return out


def oracle_demonstrations(demos):
    out = []
    for d in demos:
        frame = pack_host_frame(d.records)
        out.append(dict(frame=frame.gpu, gold=list(d.gold), forbidden=None if d.forbidden is None else list(d.forbidden),
                        mask=selection_mask(frame.active, d.allows)))
    return out
