"""Edge-case frames shared by the reference-run fixture generator and the
tests that check the oracle and the CUDA path against it: frames without a
bank or without a question, empty records and holes, single-token and full
records, a rule that admits nothing (the reopened row), and a question whose
every record is blocked, with sampling."""
import numpy as np

WEIGHT_SEED = 3


def token_rows():
    return np.arange(4096, dtype=np.uint32) % 64


def edge_frames():
    rng = np.random.default_rng(9)
    return [
        [dict(query=True, tokens=[5]), dict(query=True, tokens=[6, 7])],  # no bank at all
        [dict(tokens=[1, 2]), dict(tokens=[3])],  # no question
        [dict(tokens=[]), dict(tokens=[0, 0]), dict(query=True, tokens=[4]), dict(tokens=[9])],  # empty records
        [dict(tokens=[11]), dict(query=True, tokens=[12])],  # R = 1, Q = 1
        [dict(tokens=[int(t) for t in rng.integers(1, 4000, 8)]) for _ in range(30)]
        + [dict(query=True, tokens=[int(t) for t in rng.integers(1, 4000, 8)]) for _ in range(5)],  # full records
        [dict(tokens=[int(rng.integers(1, 4000))]) for _ in range(40)] + [dict(query=True, tokens=[2])],  # 1-token
        [dict(query=True, tokens=[7])] + [dict(band=int(b), schemaId=int(s), tokens=[int(s) + 1])
                                          for b, s in zip([0, 1, 2, 3, 4, 6, 7] * 3, range(21))],
        [dict(tokens=[3, 0, 5, 0, 7]), dict(query=True, tokens=[0, 9]), dict(tokens=[8, 8, 8])],  # holes
    ]


def reopen_frame():
    """12 bank records over schemas 0-3, two questions: question 0 admits schema 1 only, question 1 admits
    no schema (its row is reopened to all open). Returns (records, schema_allow u32[2*8], band_allow u32[2])."""
    recs = [dict(tokens=[i + 1], schemaId=i % 4, band=i % 3) for i in range(12)]
    recs += [dict(query=True, tokens=[40]), dict(query=True, tokens=[41])]
    schema_allow = np.zeros(16, dtype=np.uint32)
    schema_allow[0] = 0b0010
    band_allow = np.array([0xFF, 0xFF], dtype=np.uint32)
    return recs, schema_allow, band_allow


def blocked_frame():
    """9 bank records, 3 questions; an explicit mask blocking every record for question 0, and uniforms."""
    recs = [dict(tokens=[i + 1, i + 2]) for i in range(9)] + [dict(query=True, tokens=[5])] * 3
    mask = np.zeros(3 * 9, dtype=np.float32)
    mask[:9] = -1e30
    return recs, mask, np.array([0.5, 0.01, 0.97])
