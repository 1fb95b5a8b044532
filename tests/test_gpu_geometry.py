"""Geometry overrides (BrainForwardConfig, packages/krystal/src/forward/
model.ts:27-80; docs/API.md:432-451). The kernels are tiled for a 128-wide
row of four 32-wide heads, so hiddenSize / headCount / headDim stay 128 / 4 /
32 and anything else is refused by name when the backend is created. The
feed-forward width (any multiple of 128: 384 takes the fused kernel, others
the projection GEMM pair) and the encoder and mixer block counts are free;
such a brain must give the oracle's selections on both paths."""
from dataclasses import replace

import numpy as np
import pytest

from krystal_b200 import abi, synth
from krystal_b200.backend import CudaBrainBackend
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("precision", ["certified", "exact"])
@pytest.mark.parametrize("ffn,enc,mix", [(256, 1, 3), (512, 3, 1)])
def test_free_geometry_matches_oracle(oracle, precision, ffn, enc, mix):
    cfg = replace(BRAIN_FORWARD_CONFIG, ffn_size=ffn, encoder_blocks=enc, mixer_blocks=mix).with_token_rows(
        np.arange(4096, dtype=np.uint32))
    w = create_brain_forward_weights(cfg, 11)
    wl = synth.WORKLOADS["ragged_4096"]
    batch = synth.make_batch(wl, seed=13, frames=16)
    be = CudaBrainBackend(cfg, w, 0)
    try:
        be.set_precision(precision)
        got = be.forward_batch(batch)
    finally:
        be.destroy()
    want = oracle.forward_batch(cfg, w.page, batch)
    assert np.array_equal(got["index"], want["index"])
    assert np.abs(got["p"] - want["p"]).max() <= 1e-4


def test_reduced_hidden_size_is_refused_by_name():
    cfg = replace(BRAIN_FORWARD_CONFIG, hidden_size=32, head_count=1, head_dim=32, ffn_size=64, encoder_blocks=1,
                  mixer_blocks=1).with_token_rows(np.arange(64, dtype=np.uint32))
    w = create_brain_forward_weights(cfg, 1)
    with pytest.raises(abi.KrystalCudaError) as e:
        CudaBrainBackend(cfg, w, 0)
    assert e.value.status == abi.KC_ERR_CAPACITY
    assert "128/4/32" in e.value.message
