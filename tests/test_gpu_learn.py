"""GPU parity of the learn step: learn_from_experience with the CUDA backend
as the gradient source against the oracle's restatement of
learnFromExperience (host/learn.ts:280-512). Weights after the update agree
within the reference's gradient tolerance (1e-4); the report's numbers agree;
the backend thinks with the updated weights afterwards.
"""
import numpy as np
import pytest

from krystal_b200.backend import CudaBrainBackend
from krystal_b200.learn import BatchLearner, LearnOptions, learn_from_experience
from krystal_b200.model import BrainForwardWeights
from oracle import learn_oracle as LO
from tests.learn_cases import experiences, oracle_experiences, world

pytestmark = pytest.mark.gpu

TOL = 1e-4


def check_report(got, want):
    assert got.frames_seen == want["frames_seen"]
    assert got.reinforced == want["reinforced"] and got.discouraged == want["discouraged"]
    assert got.update_applied == want["update_applied"] and got.rejected == want["rejected"]
    for k in ("mean_advantage", "mean_value_loss", "mean_entropy", "mean_confidence"):
        assert abs(getattr(got, k) - want[k]) <= 1e-6, k


@pytest.mark.parametrize("precision", ["exact", "certified"])
@pytest.mark.parametrize("unfreeze_pool", [False, True])
def test_learn_matches_oracle_learn(oracle, unfreeze_pool, precision):
    cfg, w0 = world()
    w = BrainForwardWeights(cfg, w0.page.copy())
    be = CudaBrainBackend(cfg, w, 0)
    be.set_precision(precision)
    try:
        learner = BatchLearner(be, w)
        page = w0.page.copy()
        for it in range(2):  # two updates: the second runs on weights the first wrote
            exps = experiences(8, seed=11 + it, skip_reward=(3,), no_choice=(5,))
            got = learn_from_experience(exps, w, be, LearnOptions(unfreeze_pool=unfreeze_pool), learner)
            page, want = LO.learn_from_experience(cfg, page, oracle_experiences(exps),
                                                  LO.Options(unfreeze_pool=unfreeze_pool))
            check_report(got, want)
            assert np.abs(w.page.astype(np.float64) - page).max() <= TOL
            page = w.page.copy()  # continue both from the same weights
        # the backend took up what moved: its forward equals the oracle's on the new weights
        exps = experiences(1, seed=40)
        from krystal_b200.frame import pack_host_frame
        frame = pack_host_frame(exps[0].records)
        enc = be.encode(frame)
        fw = oracle.forward(cfg, w.page, frame.gpu)
        assert np.array_equal(enc.query_output, fw["query_output"])
    finally:
        be.destroy()


def test_learn_rollback_leaves_weights_and_backend(oracle):
    cfg, w0 = world()
    w = BrainForwardWeights(cfg, w0.page.copy())
    be = CudaBrainBackend(cfg, w, 0)
    try:
        exps = experiences(5, seed=9)
        got = learn_from_experience(exps, w, be, LearnOptions(max_parameter_abs=1e-3))
        _, want = LO.learn_from_experience(cfg, w0.page, oracle_experiences(exps), LO.Options(max_parameter_abs=1e-3))
        check_report(got, want)
        assert got.rejected == "parameter-limit" and not got.update_applied
        assert np.array_equal(w.page, w0.page)
    finally:
        be.destroy()


def test_learn_with_nothing_to_learn(oracle):
    cfg, w0 = world()
    w = BrainForwardWeights(cfg, w0.page.copy())
    be = CudaBrainBackend(cfg, w, 0)
    try:
        exps = experiences(3, seed=2, skip_reward=(0, 1, 2))
        got = learn_from_experience(exps, w, be)
        assert got.frames_seen == 0 and not got.update_applied
        assert np.array_equal(w.page, w0.page)
    finally:
        be.destroy()
