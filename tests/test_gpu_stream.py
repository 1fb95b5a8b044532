"""GPU tests of the streaming packer (kc_stream_*): frames queued one at a
time or in runs and batched by flushes come back with exactly the results the
one-shot batch entry point gives the same frames (a frame's results do not
depend on which frames share its batch), rules ride along per frame, a
malformed frame is refused alone, and flow control reports a full buffer.
"""
import numpy as np
import pytest

from krystal_b200 import abi, synth
from krystal_b200.backend import CudaBrainBackend, MaskRule
from krystal_b200.stream import FrameStream, clock_ms

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ragged():
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    be = CudaBrainBackend(cfg, w, 0)
    yield wl, cfg, w, be
    be.destroy()


def per_frame(res, frames):
    """Split a batch result into per-frame (p, index) pairs."""
    out = []
    for f in range(frames):
        p0, p1 = int(res["p_off"][f]), int(res["p_off"][f + 1])
        q0, q1 = int(res["q_off"][f]), int(res["q_off"][f + 1])
        out.append((res["p"][p0:p1], res["index"][q0:q1]))
    return out


def drain(st, got, want_frames):
    while len(got) < want_frames:
        b = st.poll(wait=True)
        assert b is not None, "a queued batch never finished"
        assert b.status == abi.KC_OK, b.error
        assert b.done_ms >= b.sealed_ms
        for i in range(b.frames):
            p0, p1 = int(b.p_off[i]), int(b.p_off[i + 1])
            q0, q1 = int(b.q_off[i]), int(b.q_off[i + 1])
            got[b.first_ticket + i] = (b.p[p0:p1].copy(), b.index[q0:q1].copy())


def collect(b, got):
    assert b.status == abi.KC_OK, b.error
    assert b.done_ms >= b.sealed_ms
    for i in range(b.frames):
        p0, p1 = int(b.p_off[i]), int(b.p_off[i + 1])
        q0, q1 = int(b.q_off[i]), int(b.q_off[i + 1])
        got[b.first_ticket + i] = (b.p[p0:p1].copy(), b.index[q0:q1].copy())


@pytest.mark.parametrize("precision", ["certified", "exact"])
def test_stream_results_equal_the_batch_results(ragged, precision):
    wl, cfg, w, be = ragged
    be.set_precision(precision)
    batch = synth.make_batch(wl, seed=31, frames=96)
    want = per_frame(be.forward_batch(batch), batch.frames)
    st = FrameStream(be, max_frames=40, max_records=40 * 256, depth=3)
    try:
        got = {}
        t0 = clock_ms()
        tickets = []
        for f in range(30):  # one at a time, flushing every 7 frames
            while True:
                try:
                    tickets.append(st.push(batch.frame(f)))
                    break
                except abi.KrystalCudaError as e:  # every buffer in flight: take a finished batch
                    assert e.status == abi.KC_ERR_CAPACITY and "poll first" in e.message
                    collect(st.poll(wait=True), got)
            if f % 7 == 6:
                st.flush()
        f = 30
        while f < batch.frames:  # the rest in runs of up to 9 frames
            first, n = st.push_many(batch, f, min(f + 9, batch.frames))
            if n:
                assert first == f
                f += n
            if n < 9 and f < batch.frames:  # the open buffer filled, or none was free
                st.flush()
                b = st.poll(wait=True)
                if b is not None:
                    collect(b, got)
        st.flush()
        drain(st, got, batch.frames)
        assert sorted(got) == list(range(batch.frames))
        assert tickets == list(range(30))
        for f in range(batch.frames):
            assert np.array_equal(got[f][1], want[f][1]), f
            assert np.array_equal(got[f][0], want[f][0]), f
        assert clock_ms() >= t0
    finally:
        st.close()
        be.set_precision("certified")


def test_stream_carries_each_frames_rule(ragged):
    wl, cfg, w, be = ragged
    batch = synth.make_batch(wl, seed=32, frames=24)
    sa, ba = synth.make_rule(batch, seed=5)
    want = per_frame(be.forward_batch(batch, rule=MaskRule(sa, ba)), batch.frames)
    offs = batch.offsets()
    st = FrameStream(be, max_frames=64, max_records=64 * 256, depth=2)
    try:
        for f in range(batch.frames):
            q0, q1 = int(offs["q_off"][f]), int(offs["q_off"][f + 1])
            if f % 3 == 2:  # an open frame among ruled ones: its rule admits everything
                st.push(batch.frame(f))
                want_open = per_frame(be.forward_batch(batch.subset([f])), 1)[0]
                want[f] = want_open
            else:
                st.push(batch.frame(f), sa.reshape(-1, 8)[q0:q1].reshape(-1), ba[q0:q1])
        st.flush()
        got = {}
        drain(st, got, batch.frames)
        for f in range(batch.frames):
            assert np.array_equal(got[f][1], want[f][1]), f
            assert np.array_equal(got[f][0], want[f][0]), f
    finally:
        st.close()


def test_stream_refuses_a_bad_frame_alone(ragged):
    wl, cfg, w, be = ragged
    batch = synth.make_batch(wl, seed=33, frames=3)
    st = FrameStream(be, max_frames=8, max_records=8 * 256, depth=2)
    try:
        assert st.push(batch.frame(0)) == 0
        bad = batch.frame(1)
        bad.token_ids[3] = 10 ** 9  # no entry in tokenRows
        with pytest.raises(abi.KrystalCudaError) as e:
            st.push(bad)
        assert e.value.status == abi.KC_ERR_INVALID_ARG and "tokenRows" in e.value.message
        assert st.push(batch.frame(2)) == 1
        st.flush()
        got = {}
        drain(st, got, 2)
        want = per_frame(be.forward_batch(batch.subset([0, 2])), 2)
        for t in range(2):
            assert np.array_equal(got[t][1], want[t][1])
    finally:
        st.close()


def test_stream_flow_control(ragged):
    wl, cfg, w, be = ragged
    batch = synth.make_batch(wl, seed=34, frames=12)
    st = FrameStream(be, max_frames=4, max_records=4 * 256, depth=2)
    try:
        first, n = st.push_many(batch, 0, 12)
        assert (first, n) == (0, 4)  # the open buffer holds four frames
        st.flush()
        first, n = st.push_many(batch, 4, 12)
        assert (first, n) == (4, 4)
        st.flush()
        # both buffers are sealed, running or finished: nothing is open until a poll
        assert st.push_many(batch, 8, 12)[1] == 0
        got = {}
        b = st.poll(wait=True)
        for i in range(b.frames):
            got[b.first_ticket + i] = b.index[int(b.q_off[i]):int(b.q_off[i + 1])].copy()
        b = st.poll(wait=True)  # releases the first batch's buffer
        for i in range(b.frames):
            got[b.first_ticket + i] = b.index[int(b.q_off[i]):int(b.q_off[i + 1])].copy()
        first, n = st.push_many(batch, 8, 12)
        assert (first, n) == (8, 4)
        st.flush()
        b = st.poll(wait=True)
        for i in range(b.frames):
            got[b.first_ticket + i] = b.index[int(b.q_off[i]):int(b.q_off[i + 1])].copy()
        assert st.poll(wait=True) is None  # nothing queued
        want = per_frame(be.forward_batch(batch), 12)
        assert sorted(got) == list(range(12))
        for f in range(12):
            assert np.array_equal(got[f], want[f][1])
    finally:
        st.close()


@pytest.mark.parametrize("threads", [1, 4])
def test_parallel_push_many_equals_the_batch_and_refuses_a_bad_frame_alone(ragged, threads):
    """A run large enough for the helper threads (some 50k records) is staged
    in parts; the results equal the batch path's, and a malformed frame in
    the middle is refused alone with every frame before it queued."""
    import copy
    wl, cfg, w, be = ragged
    batch = synth.make_batch(wl, seed=35, frames=400)
    want = per_frame(be.forward_batch(batch), batch.frames)
    bad = copy.deepcopy(batch)
    at = 250
    bad.token_ids[int(bad.rec_off[at]) * 8 + 3] = 10 ** 9  # no entry in tokenRows
    st = FrameStream(be, max_frames=512, max_records=512 * 256, depth=2, push_threads=threads)
    try:
        assert st.stats()["push_threads"] == threads
        with pytest.raises(abi.KrystalCudaError) as e:
            st.push_many(bad, 0, batch.frames)
        assert e.value.status == abi.KC_ERR_INVALID_ARG and "tokenRows" in e.value.message
        assert f"(frame {at})" in e.value.message
        first, n = st.push_many(bad, at + 1, batch.frames)
        assert (first, n) == (at, batch.frames - at - 1)  # tickets run on past the refused frame
        st.flush()
        got = {}
        drain(st, got, batch.frames - 1)
        kept = [f for f in range(batch.frames) if f != at]
        for t, f in enumerate(kept):
            assert np.array_equal(got[t][1], want[f][1]), f
            assert np.array_equal(got[t][0], want[f][0]), f
        s = st.stats(reset=True)
        assert s["frames_pushed"] == batch.frames - 1 and s["batches"] == 1
        assert s["bytes_staged"] == 72 * (batch.records - (int(batch.rec_off[at + 1]) - int(batch.rec_off[at])))
        assert 0 <= s["sync_wait_ms"] <= s["run_ms"]
        assert st.stats()["frames_pushed"] == 0
    finally:
        st.close()
