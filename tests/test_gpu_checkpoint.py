"""KRY1 straight into and out of the device weight page (kc_load_checkpoint,
kc_save_checkpoint), and BrainSession.snapshot / restore over it, after the
reference's own checkpoint cases (host/checkpoint.test.ts:26-76)."""
import numpy as np
import pytest

from krystal_b200 import synth
from krystal_b200.backend import CudaBrainBackend
from krystal_b200.checkpoint import encode_checkpoint
from krystal_b200.frame import pack_host_frame
from krystal_b200.learn import HostExperience, learn_from_experience
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights
from krystal_b200.session import BrainSession

pytestmark = pytest.mark.gpu


def rows(count=4096, offset=0):
    return (np.arange(count, dtype=np.uint32) + offset) % 64


WORLD = [dict(schemaId=1, band=3, tokens=[10, 11]), dict(schemaId=1, band=3, tokens=[20, 21]),
         dict(schemaId=9, query=True, tokens=[40, 41])]


def test_device_ingest_and_export(oracle):
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    a = synth.workload_weights(cfg, wl.vocab)
    b = synth.workload_weights(cfg, wl.vocab, seed=4242)
    be = CudaBrainBackend(cfg, a, 0)
    fresh = CudaBrainBackend(cfg, b, 0)
    try:
        ckpt = encode_checkpoint(b, cfg, cfg.token_rows)
        assert be.load_checkpoint(ckpt) is None
        assert be.save_checkpoint() == ckpt  # the device page is b, byte for byte
        frame = synth.make_batch(wl, seed=5, frames=1).frame(0)
        from krystal_b200.frame import HostFrame, compile_active_frame
        hf = HostFrame(frame, compile_active_frame(frame), frame.schema_ids.size)
        enc = be.encode(hf)
        fw = oracle.forward(cfg, b.page, frame)
        assert np.array_equal(enc.query_output, fw["query_output"])
        # the tensor-core images were rebuilt from the new page: same results as a backend built on b
        batch = synth.make_batch(wl, seed=6, frames=64)
        got, want = be.forward_batch(batch), fresh.forward_batch(batch)
        assert np.array_equal(got["index"], want["index"]) and np.array_equal(got["p"], want["p"])
        # a refusal leaves the device page as it was
        other = encode_checkpoint(a, cfg, rows(cfg.token_rows.size, 1))
        assert be.load_checkpoint(other) == "a different vocabulary"
        assert be.load_checkpoint(bytes(64)) == "not a krystal checkpoint"
        assert be.load_checkpoint(ckpt[:100]) == "truncated"
        assert be.save_checkpoint() == ckpt
    finally:
        be.destroy()
        fresh.destroy()


def test_a_restored_session_answers_exactly_as_the_one_written():
    trained = BrainSession(rows(), seed=7)
    cold = BrainSession(rows(), seed=99)
    try:
        # move it off its seed, so the test is about the checkpoint
        frame = pack_host_frame(WORLD)
        bank = frame.active.bank_records.tolist()
        report = learn_from_experience([HostExperience(WORLD, 0.5, [bank[0]])], trained.weights, trained.backend)
        assert report.update_applied
        before = trained.think(WORLD).selections[0]
        assert cold.restore(trained.snapshot()) is None
        after = cold.think(WORLD).selections[0]
        assert after.record == before.record
        assert np.array_equal(after.distribution, before.distribution)
        assert cold.backend.save_checkpoint() == trained.snapshot()
    finally:
        trained.destroy()
        cold.destroy()


def test_restore_refusals_leave_the_session_alone():
    trained = BrainSession(rows(), seed=7)
    other = BrainSession(rows(offset=1), seed=7)
    try:
        untouched = other.weights.selector.wq.copy()
        before = other.backend.save_checkpoint()
        assert other.restore(trained.snapshot()) == "a different vocabulary"
        assert np.array_equal(other.weights.selector.wq, untouched)
        assert other.backend.save_checkpoint() == before
        assert other.restore(bytes(3)) == "truncated"
    finally:
        trained.destroy()
        other.destroy()
