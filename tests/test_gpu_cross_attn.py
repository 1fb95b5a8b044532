"""The mixer's two f32 cross-attention kernels agree bit for bit.

k_cross_attn_small (banks of at most 256 keys: one pass, the chunk's scores
for the whole bank in shared memory) and k_cross_attn_frame (any bank: keys
streamed in blocks, a max pass, then the scores again for the exponentials
and p·v) claim the same arithmetic. A batch whose banks all fit 256 keys runs
the first; the same frames with one more frame of a 300-key bank run the
second for the whole batch. The shared frames' mixer outputs, distributions
and selections must be identical, for bank lengths around the 32-key softmax
stride and the 128-key block, and for 1 to 33 questions (chunk edges).
"""
import numpy as np
import pytest

from krystal_b200 import synth
from krystal_b200.backend import CudaBrainBackend
from krystal_b200.frame import FrameBatch

pytestmark = pytest.mark.gpu

WL = synth.WORKLOADS["ragged_4096"]
CFG = synth.workload_config(WL)
W = synth.workload_weights(CFG, WL.vocab)

BANKS = [1, 2, 31, 32, 33, 63, 64, 65, 127, 128, 129, 200, 255, 256]
QUESTIONS = [1, 16, 3, 17, 8, 33, 2, 15, 9, 1, 24, 5, 16, 7]


def layout(banks, questions, seed) -> FrameBatch:
    """Frames of `banks[k]` bank records and `questions[k]` questions; frame k
    is drawn from its own generator, so a frame does not depend on the others."""
    recs, ids, schema = [], [], []
    for k, (r, q) in enumerate(zip(banks, questions)):
        rng = np.random.default_rng([seed, k])
        f = [(int(rng.integers(1, 9)), False) for _ in range(r)] + [(int(rng.integers(1, 9)), True) for _ in range(q)]
        rng.shuffle(f)
        t = rng.integers(1, WL.vocab, (len(f), 8)).astype(np.uint32)
        for i, (n, _) in enumerate(f):
            t[i, n:] = 0
        recs.append(f)
        ids.append(t)
        schema.append(rng.integers(0, WL.schemas, len(f)).astype(np.uint32))
    rec_off = np.zeros(len(recs) + 1, dtype=np.uint64)
    np.cumsum([len(f) for f in recs], out=rec_off[1:])
    flat = [r for f in recs for r in f]
    band = np.array([synth.QUERY_BAND if q else synth.BANK_BANDS[i % synth.BANK_BANDS.size]
                     for i, (_, q) in enumerate(flat)], dtype=np.uint32)
    return FrameBatch(rec_off, np.concatenate(ids).reshape(-1), np.zeros(len(flat) * 8, dtype=np.uint32),
                      np.concatenate(schema), band)


@pytest.fixture(scope="module")
def be():
    b = CudaBrainBackend(CFG, W, 0)
    b.set_precision("fast")
    yield b
    b.destroy()


def test_one_pass_and_blocked_kernels_agree(be):
    small = be.forward_batch(layout(BANKS, QUESTIONS, 3), want_query_output=True)
    big = be.forward_batch(layout(BANKS + [300], QUESTIONS + [4], 3), want_query_output=True)
    nq = sum(QUESTIONS)
    n_p = int(small["p_off"][-1])
    assert np.array_equal(small["query_output"], big["query_output"][: nq * CFG.hidden_size])
    assert np.array_equal(small["p"], big["p"][:n_p])
    np.testing.assert_array_equal(small["index"], big["index"][:nq])
