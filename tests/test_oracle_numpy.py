"""Cross-check: the C++ oracle against an independent numpy restatement."""
import numpy as np
import pytest

from krystal_b200 import synth
from krystal_b200.frame import pack_host_frame
from tests import numpy_forward as NF


@pytest.mark.parametrize("frames,seed", [(3, 11), (2, 12)])
def test_oracle_agrees_with_numpy_restatement(oracle, frames, seed):
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    batch = synth.make_batch(wl, seed=seed, frames=frames)
    for f in range(frames):
        g = batch.frame(f)
        fr = pack_host_frame([dict(schemaId=int(g.schema_ids[s]), band=int(g.band_ids[s]),
                                   tokens=[int(t) for t in g.token_ids[s * 8:(s + 1) * 8] if t])
                              for s in range(g.schema_ids.size)])
        want = NF.forward(cfg, w, fr)
        got = oracle.forward(cfg, w.page, fr.gpu)
        for key in ("field_states", "bank_keys", "bank_values", "query_output"):
            scale = max(1.0, float(np.abs(want[key]).max()))
            assert np.abs(got[key] - want[key]).max() <= 2e-5 * scale, key
        p_np = NF.selector(want["query_output"], want["bank_keys"], None, w.selector.wq, w.selector.wk, 128)
        sel = oracle.selector(got["query_output"], got["bank_keys"], got["bank_values"], None, w.selector.wq,
                              w.selector.wk, 128)
        assert np.abs(sel["p"] - p_np).max() <= 1e-6
