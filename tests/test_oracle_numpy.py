"""Cross-check: the C++ oracle against an independent numpy restatement."""
import numpy as np
import pytest

from krystal_b200 import synth
from krystal_b200.frame import pack_host_frame
from tests import numpy_forward as NF


def word_ids_for(frame_gpu, seed):
    """Per frame token: a word label shared by runs of tokens within a record
    (some tokens carry none)."""
    rng = np.random.default_rng(seed)
    n = frame_gpu.token_ids.size
    w = rng.integers(0, 3, n).astype(np.uint32)
    w[rng.random(n) < 0.2] = 0xFFFFFFFF
    return w


@pytest.mark.parametrize("frames,seed,alpha", [(3, 11, 0.0), (2, 12, 0.0), (2, 13, 1.5), (2, 14, -2.25)])
def test_oracle_agrees_with_numpy_restatement(oracle, frames, seed, alpha):
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    batch = synth.make_batch(wl, seed=seed, frames=frames)
    for f in range(frames):
        g = batch.frame(f)
        fr = pack_host_frame([dict(schemaId=int(g.schema_ids[s]), band=int(g.band_ids[s]),
                                   tokens=[int(t) for t in g.token_ids[s * 8:(s + 1) * 8] if t])
                              for s in range(g.schema_ids.size)])
        words = word_ids_for(fr.gpu, seed + f) if alpha else None
        want = NF.forward(cfg, w, fr, words, alpha)
        got = oracle.forward(cfg, w.page, fr.gpu, word_ids=words, alpha=alpha)
        for key in ("field_states", "bank_keys", "bank_values", "query_output"):
            scale = max(1.0, float(np.abs(want[key]).max()))
            assert np.abs(got[key] - want[key]).max() <= 2e-5 * scale, key
        p_np = NF.selector(want["query_output"], want["bank_keys"], None, w.selector.wq, w.selector.wk, 128)
        sel = oracle.selector(got["query_output"], got["bank_keys"], got["bank_values"], None, w.selector.wq,
                              w.selector.wk, 128)
        assert np.abs(sel["p"] - p_np).max() <= 1e-6


def test_word_bias_zero_alpha_is_no_bias_and_nonzero_moves_the_encoder(oracle):
    """compileRecordMask: alpha = 0 is bit-identical to the unbiased mask by
    construction (masks.ts:160-161); a non-zero alpha changes the encoding."""
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    g = synth.make_batch(wl, seed=21, frames=1).frame(0)
    words = word_ids_for(g, 3)
    plain = oracle.forward(cfg, w.page, g)
    zero = oracle.forward(cfg, w.page, g, word_ids=words, alpha=0.0)
    biased = oracle.forward(cfg, w.page, g, word_ids=words, alpha=2.0)
    no_words = oracle.forward(cfg, w.page, g, word_ids=np.full_like(words, 0xFFFFFFFF), alpha=2.0)
    for key in ("field_states", "query_output"):
        assert np.array_equal(zero[key], plain[key])
        assert np.array_equal(no_words[key], plain[key])
        assert not np.array_equal(biased[key], plain[key])
