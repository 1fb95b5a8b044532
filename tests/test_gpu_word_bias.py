"""GPU parity of the same-word bias (WordBias, forward/masks.ts:145-198) on the
batch path: word ids ride beside the token ids, and the encoder's record-local
attention adds the f32 alpha between two tokens of one record that share a
valid word id. Against the oracle's restatement, on the exact path and on the
certified tensor-core path (whose exact recomputation carries the word ids)."""
import numpy as np
import pytest

from krystal_b200 import synth
from krystal_b200.backend import CudaBrainBackend

pytestmark = pytest.mark.gpu


def word_ids_for(batch, seed):
    rng = np.random.default_rng(seed)
    n = batch.token_ids.size
    w = rng.integers(0, 3, n).astype(np.uint32)
    w[rng.random(n) < 0.2] = 0xFFFFFFFF
    return w


@pytest.fixture(scope="module")
def ragged():
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    be = CudaBrainBackend(cfg, w, 0)
    yield wl, cfg, w, be
    be.destroy()


@pytest.mark.parametrize("precision", ["exact", "certified"])
@pytest.mark.parametrize("alpha", [1.5, -3.0])
def test_word_bias_matches_oracle(oracle, ragged, precision, alpha):
    wl, cfg, w, be = ragged
    be.set_precision(precision)
    try:
        batch = synth.make_batch(wl, seed=41, frames=24)
        words = word_ids_for(batch, 7)
        got = be.forward_batch(batch, word_ids=words, word_alpha=alpha)
        want = oracle.forward_batch(cfg, w.page, batch, word_ids=words, alpha=alpha)
        assert np.array_equal(got["index"], want["index"])
        assert np.abs(got["p"] - want["p"]).max() <= 1e-4
        if precision == "exact":
            assert np.mean(got["p"] == want["p"]) >= 0.9999
        plain = be.forward_batch(batch)
        assert not np.array_equal(plain["p"], got["p"])  # the bias moved the distributions
    finally:
        be.set_precision("certified")


def test_zero_alpha_and_no_words_equal_no_bias(ragged):
    wl, cfg, w, be = ragged
    batch = synth.make_batch(wl, seed=42, frames=16)
    words = word_ids_for(batch, 8)
    plain = be.forward_batch(batch)
    for res in (be.forward_batch(batch, word_ids=words, word_alpha=0.0),
                be.forward_batch(batch, word_ids=np.full_like(words, 0xFFFFFFFF), word_alpha=2.0)):
        assert np.array_equal(res["p"], plain["p"]) and np.array_equal(res["index"], plain["index"])


@pytest.mark.parametrize("precision", ["exact", "certified"])
def test_a_bias_that_blocks_a_whole_record(oracle, ragged, precision):
    """Every token of every record shares one word and alpha = -1e30: each
    in-record row is all blocked, so local attention contributes zeros
    (attentionOracle's allBlocked rule, oracle.ts:87-89)."""
    wl, cfg, w, be = ragged
    be.set_precision(precision)
    try:
        batch = synth.make_batch(wl, seed=43, frames=8)
        words = np.zeros(batch.token_ids.size, np.uint32)
        got = be.forward_batch(batch, word_ids=words, word_alpha=-1e30)
        want = oracle.forward_batch(cfg, w.page, batch, word_ids=words, alpha=-1e30)
        assert np.array_equal(got["index"], want["index"])
        assert np.abs(got["p"] - want["p"]).max() <= 1e-4
    finally:
        be.set_precision("certified")
