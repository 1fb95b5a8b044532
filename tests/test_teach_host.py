"""The host half of teach (krystal_b200/teach.py) on the CPU.

teach_from_demonstration, fed gradients by the oracle's backward through a
stand-in gradient source, must reproduce the oracle's loop restatement of
teachFromDemonstration (teach.ts:126-272) bit for bit: the capped step, the
decay, the token-by-token row writes, the rejection of a showing past the
ceiling and the report. Each showing is applied before the next is
differentiated, as the reference's contract says (:120-125).
"""
from types import SimpleNamespace

import numpy as np
import pytest

from krystal_b200.teach import TeachOptions, teach_from_demonstration
from oracle import teach_oracle as TO
from tests.learn_cases import world
from tests.teach_cases import demonstrations, oracle_demonstrations


class OracleGradients:
    """A gradient source over the oracle's backward, reading the live arrays."""

    def __init__(self, oracle, cfg, weights):
        self.oracle, self.cfg, self.weights = oracle, cfg, weights
        self.synced = 0

    def backward(self, frame, selection=None, targets=None, valence_target=None):
        r = self.oracle.backward(self.cfg, self.weights.page, frame.gpu, selection, targets, valence_target)
        return SimpleNamespace(policy=r["policy"], d_selector_wq=r["d_selector_wq"],
                               d_selector_wk=r["d_selector_wk"], d_field_states=r["d_field_states"])

    def sync(self, weights, changes=None):
        self.synced += 1


CASES = {
    "defaults": (TeachOptions(), TO.Options()),
    "frozen tables": (TeachOptions(unfreeze_tokens=False), TO.Options(unfreeze_tokens=False)),
    "capped step": (TeachOptions(max_update_abs=1e-4), TO.Options(max_update_abs=1e-4)),
    "ceiling": (TeachOptions(max_parameter_abs=0.05), TO.Options(max_parameter_abs=0.05)),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_host_teach_matches_oracle_teach(oracle, case):
    opts, oopts = CASES[case]
    cfg, w = world()
    demos = demonstrations(4, seed=3, nothing=(2,))
    page0 = w.page.copy()
    src = OracleGradients(oracle, cfg, w)
    got = teach_from_demonstration(demos, w, src, opts)
    page, want = TO.teach_from_demonstration(cfg, page0, oracle_demonstrations(demos), oopts)
    assert np.array_equal(w.page, page)
    assert (got.frames_seen, got.shown, got.rejected, got.clipped) == (
        want["frames_seen"], want["shown"], want["rejected"], want["clipped"])
    assert got.mean_agreement == want["mean_agreement"]
    assert got.max_parameter_abs == want["max_parameter_abs"]
    assert src.synced == got.frames_seen  # told after every showing kept, never after a rejected one
    if case == "ceiling":
        assert got.rejected > 0
    if case == "capped step":
        assert got.clipped > 0
