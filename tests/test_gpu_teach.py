"""GPU parity of teach: teachFromDemonstration (teach.ts:126-272) with the CUDA
backend as the gradient source — each showing differentiated by kc_backward,
applied on the host, and taken up by kc_sync before the next showing —
against the oracle's restatement. Weights agree within the reference's
gradient tolerance (1e-4) after successive showings; the report agrees; the
backend thinks with the taught weights afterwards."""
import numpy as np
import pytest

from krystal_b200.backend import CudaBrainBackend
from krystal_b200.frame import pack_host_frame
from krystal_b200.model import BrainForwardWeights
from krystal_b200.teach import TeachOptions, teach_from_demonstration
from oracle import teach_oracle as TO
from tests.learn_cases import world
from tests.teach_cases import demonstrations, oracle_demonstrations

pytestmark = pytest.mark.gpu

TOL = 1e-4


@pytest.mark.parametrize("unfreeze", [True, False])
def test_successive_showings_match_oracle_teach(oracle, unfreeze):
    cfg, w0 = world()
    w = BrainForwardWeights(cfg, w0.page.copy())
    be = CudaBrainBackend(cfg, w, 0)
    try:
        page = w0.page.copy()
        for it in range(2):  # two passes of three showings: the second meets the brain the first left
            demos = demonstrations(3, seed=50 + it)
            got = teach_from_demonstration(demos, w, be, TeachOptions(unfreeze_tokens=unfreeze))
            page, want = TO.teach_from_demonstration(cfg, page, oracle_demonstrations(demos),
                                                     TO.Options(unfreeze_tokens=unfreeze))
            assert (got.frames_seen, got.shown, got.rejected, got.clipped) == (
                want["frames_seen"], want["shown"], want["rejected"], want["clipped"])
            assert abs(got.mean_agreement - want["mean_agreement"]) <= 1e-6
            assert np.abs(w.page.astype(np.float64) - page).max() <= TOL
            page = w.page.copy()  # continue both from the same weights
        assert not np.array_equal(w.page, w0.page)
        frame = pack_host_frame(demonstrations(1, seed=99)[0].records)
        enc = be.encode(frame)
        fw = oracle.forward(cfg, w.page, frame.gpu)
        assert np.array_equal(enc.query_output, fw["query_output"])
        assert np.array_equal(enc.bank_keys, fw["bank_keys"])
    finally:
        be.destroy()


def test_session_teach_raises_agreement(oracle):
    """BrainSession.teach (session.ts:205-207): showing the same answer again
    and again moves the policy toward it (teach.ts:96-103)."""
    from krystal_b200.session import BrainSession
    cfg, _ = world()
    s = BrainSession(cfg.token_rows, seed=3)
    try:
        demo = demonstrations(1, seed=5, forbid=())
        first = s.teach(demo)
        for _ in range(8):
            last = s.teach(demo)
        assert first.frames_seen == 1 and last.frames_seen == 1
        assert last.mean_agreement > first.mean_agreement
    finally:
        s.destroy()
