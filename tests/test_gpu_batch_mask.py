"""An explicit selection mask on the batch path: a grammar that is not a
schema x band product (selectionMask over any allows(q, record) closure,
host/learn.ts:215-232) laid out like p and added to every score
(forward/oracle.ts:340-345). Certified and exact batches, the reselect of a
resident batch, and sampling under a mask, against the oracle's per-frame
forward and selector; indices exact, p within the reference's 1e-4."""
import numpy as np
import pytest

from krystal_b200 import synth
from krystal_b200.backend import CudaBrainBackend
from krystal_b200.frame import HostFrame, compile_active_frame
from krystal_b200.session import selection_mask

pytestmark = pytest.mark.gpu

P_TOL = 1e-4


def batch_mask(batch, seed):
    """Per frame, selectionMask of an arbitrary closure: (q * 7 + slot * 3 + seed) % k != 0, k per frame;
    frames whose closure admits nothing for a question get that row reopened by selectionMask."""
    rng = np.random.default_rng(seed)
    parts = []
    for f in range(batch.frames):
        g = batch.frame(f)
        act = compile_active_frame(g)
        k = int(rng.integers(1, 5))  # k = 1 blocks everything: the reopened row
        parts.append(selection_mask(act, lambda q, slot, k=k: (q * 7 + slot * 3 + seed) % k != 0))
    return np.concatenate(parts).astype(np.float32)


def oracle_select(oracle, cfg, w, batch, mask, uniforms=None):
    ps, idx = [], []
    off, qoff = 0, 0
    for f in range(batch.frames):
        g = batch.frame(f)
        enc = oracle.forward(cfg, w.page, g)
        q, r = enc["q"], enc["r"]
        u = None if uniforms is None else uniforms[qoff:qoff + q]
        sel = oracle.selector(enc["query_output"], enc["bank_keys"], enc["bank_values"], mask[off:off + q * r],
                              w.selector.wq, w.selector.wk, 128, u)
        ps.append(sel["p"])
        idx.append(sel["index"])
        off += q * r
        qoff += q
    return np.concatenate(ps), np.concatenate(idx)


@pytest.mark.parametrize("precision", ["certified", "exact"])
def test_batch_mask_matches_oracle(oracle, precision):
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    batch = synth.make_batch(wl, seed=41, frames=24)
    m1, m2 = batch_mask(batch, 1), batch_mask(batch, 2)
    nq = int((batch.band_ids == 5).sum())
    u = np.random.default_rng(9).random(nq)
    be = CudaBrainBackend(cfg, w, 0)
    be.set_precision(precision)
    try:
        got1 = be.forward_batch(batch, mask=m1)
        got2 = be.select_batch(mask=m2)             # consider once, choose again under another grammar
        got3 = be.select_batch(mask=m1, uniforms=u)  # and sample under a mask
    finally:
        be.destroy()
    for got, m, uu in ((got1, m1, None), (got2, m2, None), (got3, m1, u)):
        p, idx = oracle_select(oracle, cfg, w, batch, m, uu)
        assert np.array_equal(got["index"], idx)
        assert np.abs(got["p"] - p).max() <= P_TOL
    assert not np.array_equal(got1["index"], got2["index"])


def test_mask_and_rule_together_are_refused():
    from krystal_b200 import abi
    from krystal_b200.backend import MaskRule
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    batch = synth.make_batch(wl, seed=41, frames=4)
    be = CudaBrainBackend(cfg, w, 0)
    try:
        with pytest.raises(abi.KrystalCudaError) as e:
            be.forward_batch(batch, rule=MaskRule(*synth.make_rule(batch, seed=2)), mask=batch_mask(batch, 1))
        assert e.value.status == abi.KC_ERR_INVALID_ARG
    finally:
        be.destroy()
