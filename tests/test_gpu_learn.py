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


def test_device_plan_equals_the_host_plan():
    """kc_learn_plan (one thread on the device, every sum a running sum in
    frame order) against plan_update on the host, bit for bit, on the
    adversarial batches of tests/test_learn_plan.py."""
    import torch

    from krystal_b200 import abi
    from krystal_b200 import learn as L
    from tests.test_learn_plan import same_float

    cfg, w0 = world()
    be = CudaBrainBackend(cfg, BrainForwardWeights(cfg, w0.page.copy()), 0)
    dev = torch.device("cuda", 0)
    opts = L.LearnOptions()
    copts = abi.KcLearnOptions(opts.learning_rate, opts.policy_scale, opts.advantage_clip, opts.max_parameter_abs,
                               opts.token_rate, 0, 0)
    rng = np.random.default_rng(3)
    try:
        for trial in range(200):
            F = int(rng.integers(0, 200))
            stats = rng.standard_normal((F, L.STATS)) * rng.choice([1e-3, 1.0, 1e3])
            stats[rng.random((F, L.STATS)) < 0.1] = 0.0
            stats[rng.random((F, L.STATS)) < 0.03] = -0.0
            rewards = rng.standard_normal(F) * rng.choice([1e-6, 1.0, 10.0])
            rewards[rng.random(F) < 0.1] = np.nan
            if trial % 7 == 0 and F:
                rewards[:] = 1.0
                stats[:, 2] = 0.5
            if trial % 11 == 0 and F:
                stats[rng.random(F) < 0.05, 2] = np.inf
            answered = rng.random(F) < 0.8
            want = L.plan_update(stats, rewards, answered, opts)
            rows = torch.from_numpy(np.concatenate([stats, rewards[:, None], answered[:, None].astype(np.float64)],
                                                   1).reshape(-1)).to(dev)
            plan = torch.full((3, max(F, 1)), -1.0, dtype=torch.float64, device=dev)
            report = torch.zeros(abi.KC_LEARN_REPORT, dtype=torch.float64, device=dev)
            torch.cuda.synchronize()
            be.learn_plan(rows.data_ptr(), F, copts, plan[0].data_ptr(), plan[1].data_ptr(), plan[2].data_ptr(),
                          report.data_ptr())
            be.synchronize()
            got = plan[:, :F].cpu().numpy()
            rep = report.cpu().numpy()
            assert np.array_equal(got[0], want.step) and np.array_equal(got[1], want.value_weight), trial
            assert (int(rep[0]), bool(rep[1]), int(rep[2]), int(rep[3])) == (
                want.seen, want.actor_moved, want.reinforced, want.discouraged), trial
            for x, y in zip(rep[4:8], (want.mean_advantage, want.mean_value_loss, want.mean_entropy,
                                       want.mean_confidence)):
                assert same_float(float(x), y), trial
    finally:
        be.destroy()


@pytest.mark.parametrize("precision", ["exact", "certified"])
def test_learn_with_unfrozen_tables_matches_oracle(oracle, precision):
    """unfreeze.tokens (learn.ts:298-299): the token and field rows of the
    answered frames move by step * tokenRate * dFieldStates
    (scatterEmbeddings, :242-263), over two successive updates."""
    cfg, w0 = world()
    w = BrainForwardWeights(cfg, w0.page.copy())
    be = CudaBrainBackend(cfg, w, 0)
    be.set_precision(precision)
    opts = LearnOptions(unfreeze_tokens=True, unfreeze_pool=True, token_rate=0.5)
    try:
        learner = BatchLearner(be, w)
        page = w0.page.copy()
        for it in range(2):
            exps = experiences(8, seed=21 + it, skip_reward=(2,), no_choice=(4,))
            got = learn_from_experience(exps, w, be, opts, learner)
            page, want = LO.learn_from_experience(cfg, page, oracle_experiences(exps),
                                                  LO.Options(unfreeze_pool=True, unfreeze_tokens=True,
                                                             token_rate=0.5))
            check_report(got, want)
            assert abs(got.health["semantic_embedding_max_abs"] - want["health"]["semantic_embedding_max_abs"]) <= TOL
            moved = np.flatnonzero(page != w0.page)
            assert moved.size and moved.min() < cfg.token_space * 2 * 128  # table rows moved
            assert np.abs(w.page.astype(np.float64) - page).max() <= TOL
            page = w.page.copy()
        # the device page is what the host holds: the next forward uses the moved rows
        from krystal_b200.frame import pack_host_frame
        frame = pack_host_frame(experiences(1, seed=40)[0].records)
        enc = be.encode(frame)
        fw = oracle.forward(cfg, w.page, frame.gpu)
        assert np.array_equal(enc.query_output, fw["query_output"])
    finally:
        be.destroy()


def test_rollback_restores_unfrozen_rows(oracle):
    cfg, w0 = world()
    w = BrainForwardWeights(cfg, w0.page.copy())
    be = CudaBrainBackend(cfg, w, 0)
    try:
        exps = experiences(6, seed=9)
        got = learn_from_experience(exps, w, be, LearnOptions(unfreeze_tokens=True, max_parameter_abs=1e-3))
        assert got.rejected == "parameter-limit" and not got.update_applied
        assert np.array_equal(w.page, w0.page)
        page = np.empty_like(w.page)
        be.copy_weights(0, page)
        assert np.array_equal(page, w0.page)
    finally:
        be.destroy()
