"""Host-side batch helpers: FrameBatch.subset keeps frames intact (the learn
bench shards a global batch with it) and the learn workload's targets stay
inside each frame's bank."""
import numpy as np

from krystal_b200 import synth


def test_subset_slices_and_lists_keep_frames():
    b = synth.make_batch(synth.WORKLOADS["learn_1024"], seed=1, frames=10)
    for sel, idx in ((slice(3, 7), [3, 4, 5, 6]), ([0, 9, 2], [0, 9, 2])):
        s = b.subset(sel)
        assert s.frames == len(idx)
        for i, f in enumerate(idx):
            a, c = b.frame(f), s.frame(i)
            for k in ("token_ids", "field_roles", "schema_ids", "band_ids"):
                assert np.array_equal(getattr(a, k), getattr(c, k))


def test_learn_inputs_target_each_frames_bank():
    b = synth.make_batch(synth.WORKLOADS["learn_1024"], seed=2, frames=64)
    targets, rewards = synth.make_learn_inputs(b, seed=3)
    o = b.offsets()
    assert (o["q"] == 4).all()
    assert targets.size == int(o["q_off"][-1]) and rewards.size == 64
    assert (targets < np.repeat(o["r"], o["q"])).all()
