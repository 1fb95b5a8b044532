"""kc_select_batch: consider once, choose many, at batch scale.

The last forward_batch's encodings stay resident; select_batch decides the
batch again under another rule and/or uniforms. Its results must equal a
fresh forward_batch under the same rule bit for bit (certified: including
which frames are recomputed exactly; exact: the oracle's arithmetic), and it
must refuse once the resident batch is gone (another call on the handle, a
weight sync) or before any batch.
"""
import numpy as np
import pytest

from krystal_b200 import abi, synth
from krystal_b200.backend import CudaBrainBackend, MaskRule
from krystal_b200.frame import QUERY_BAND, HostFrame, compile_active_frame

pytestmark = pytest.mark.gpu

WL = synth.WORKLOADS["ragged_4096"]
CFG = synth.workload_config(WL)
W = synth.workload_weights(CFG, WL.vocab)


def rule(batch, seed, density=0.5) -> MaskRule:
    sa, ba = synth.make_rule(batch, seed=seed, density=density)
    return MaskRule(sa, ba)


def uniforms(batch, seed):
    nq = int((batch.band_ids == QUERY_BAND).sum())
    return np.random.default_rng(seed).random(nq)


def same(a: dict, b: dict):
    np.testing.assert_array_equal(a["index"], b["index"])
    assert np.array_equal(a["p"], b["p"])
    assert np.array_equal(a["p_off"], b["p_off"]) and np.array_equal(a["q_off"], b["q_off"])


@pytest.fixture(scope="module")
def be():
    b = CudaBrainBackend(CFG, W, 0)
    yield b
    b.destroy()


@pytest.mark.parametrize("precision,frames", [("certified", 512), ("fast", 256), ("exact", 24)])
def test_reselect_equals_a_fresh_forward(be, precision, frames):
    be.set_precision(precision)
    batch = synth.make_batch(WL, seed=61, frames=frames)
    ra, rb, rc = rule(batch, 1), rule(batch, 2, 0.3), rule(batch, 3, 0.8)
    ub = uniforms(batch, 4)
    want_b = be.forward_batch(batch, rule=rb)
    want_c = be.forward_batch(batch, rule=rc, uniforms=ub)
    want_open = be.forward_batch(batch)
    be.forward_batch(batch, rule=ra)           # resident: encoded once
    same(be.select_batch(rule=rb), want_b)     # then chosen again, several times
    same(be.select_batch(rule=rc, uniforms=ub), want_c)
    same(be.select_batch(), want_open)
    same(be.select_batch(rule=rb), want_b)


def test_reselect_refuses_without_a_resident_batch():
    fresh = CudaBrainBackend(CFG, W, 0)
    try:
        with pytest.raises(RuntimeError):
            fresh.select_batch()
        batch = synth.make_batch(WL, seed=62, frames=32)
        fresh.forward_batch(batch)
        fresh.select_batch(rule=rule(batch, 5))
        fresh.sync(W)  # weights may have changed: the encodings are stale
        with pytest.raises(abi.KrystalCudaError, match="resident"):
            fresh.select_batch(rule=rule(batch, 5))
        fresh.forward_batch(batch)
        g = synth.make_batch(WL, seed=63, frames=1).frame(0)
        fresh.encode(HostFrame(g, compile_active_frame(g), g.schema_ids.size))  # another call on the handle
        with pytest.raises(abi.KrystalCudaError, match="resident"):
            fresh.select_batch()
    finally:
        fresh.destroy()
