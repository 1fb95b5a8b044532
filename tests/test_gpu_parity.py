"""GPU parity: the CUDA path, called through the C ABI, against the oracle.

The bar: selected indices bit-exact; distributions within 1e-4 max-abs (the
reference's own tolerance, packages/webgpu/test/krystal-composed.test.ts:67-69).
The exact kernels reproduce the oracle's arithmetic, so the distributions are
also asserted bit-identical for all but a vanishing share of entries.
"""
import numpy as np
import pytest

from krystal_b200 import abi, synth
from krystal_b200.backend import CudaBrainBackend, MaskRule, WeightChanges
from krystal_b200.frame import BrainFrameGpu, FrameBatch, HostFrame, compile_active_frame, pack_host_frame
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights
from krystal_b200.session import BrainSession, selection_mask
from tests import golden_io as G

pytestmark = pytest.mark.gpu

P_TOL = 1e-4


def assert_p_close(got, want, exact_share=0.9999):
    assert got.shape == want.shape
    if got.size == 0:
        return
    assert np.abs(got - want).max() <= P_TOL
    assert np.mean(got == want) >= exact_share


def host_frame(g: BrainFrameGpu) -> HostFrame:
    return HostFrame(g, compile_active_frame(g), g.schema_ids.size)


@pytest.fixture(scope="module")
def test_records_backend():
    g, cfg, w, frame = G.test_records()
    be = CudaBrainBackend(cfg, w, 0)
    yield g, cfg, w, frame, be
    be.destroy()


def test_encode_matches_golden(test_records_backend):
    g, cfg, w, frame, be = test_records_backend
    enc = be.encode(host_frame(frame))
    assert np.array_equal(enc.query_output, g["query_output"])
    assert np.array_equal(enc.bank_keys, g["bank_keys"])
    assert np.array_equal(enc.bank_values, g["bank_values"])


def test_select_matches_golden(test_records_backend):
    g, cfg, w, frame, be = test_records_backend
    enc = be.encode(host_frame(frame))
    sel = be.select(enc, mask=g["grammar"])
    assert sel.index.tolist() == g["index"].tolist()
    assert_p_close(sel.p, g["p"], 1.0)
    assert np.abs(sel.gather - g["gather"]).max() <= 1e-6
    sel = be.select(enc)
    assert sel.index.tolist() == g["index_open"].tolist()
    assert_p_close(sel.p, g["p_open"], 1.0)


MODES = ["exact", "certified"]


def check_batch(res, want, mode, exact_share=0.9999):
    """Indices exact in every mode; p bit-identical (but for a vanishing share)
    on the exact path, within the parity tolerance on the certified path."""
    assert np.array_equal(res["index"], want["index"])
    if mode == "exact":
        assert_p_close(res["p"], want["p"], exact_share)
    else:
        assert res["p"].shape == want["p"].shape
        if res["p"].size:
            assert np.abs(res["p"] - want["p"]).max() <= P_TOL


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", G.BATCHES)
def test_batch_matches_golden(name, mode):
    g, cfg, w, b, rule, u = G.batch(name)
    be = CudaBrainBackend(cfg, w, 0)
    try:
        be.set_precision(mode)
        res = be.forward_batch(b, rule=MaskRule(*rule) if rule else None, uniforms=u, want_query_output=True)
    finally:
        be.destroy()
    assert np.array_equal(res["p_off"], g["p_off"]) and np.array_equal(res["q_off"], g["q_off"])
    check_batch(res, g, mode)
    assert np.abs(res["query_output"] - g["query_output"]).max() <= (1e-5 if mode == "exact" else 1e-4)


def _backend_for(workload: str):
    wl = synth.WORKLOADS[workload]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    return wl, cfg, w, CudaBrainBackend(cfg, w, 0)


@pytest.mark.parametrize("mode", MODES)
def test_ragged_batch_with_rule_matches_live_oracle(oracle, mode):
    wl, cfg, w, be = _backend_for("ragged_4096")
    try:
        be.set_precision(mode)
        batch = synth.make_batch(wl, seed=77, frames=48)
        rule = synth.make_rule(batch, seed=78)
        res = be.forward_batch(batch, rule=MaskRule(*rule))
    finally:
        be.destroy()
    want = oracle.forward_batch(cfg, w.page, batch, rule=rule)
    check_batch(res, want, mode)


@pytest.mark.parametrize("mode", MODES)
def test_long_bank_frame_matches_live_oracle(oracle, mode):
    wl, cfg, w, be = _backend_for("long_bank_1024")
    try:
        be.set_precision(mode)
        batch = synth.make_batch(wl, seed=5, frames=1)
        res = be.forward_batch(batch)
    finally:
        be.destroy()
    want = oracle.forward_batch(cfg, w.page, batch)
    assert res["index"].size == 64 and res["p"].size == 64 * 4096
    check_batch(res, want, mode)


def test_certifying_everything_reproduces_the_exact_path():
    """With an enormous margin every frame is recomputed exactly: the certified
    batch must then equal the exact batch bit for bit (fallback plumbing)."""
    wl, cfg, w, be = _backend_for("ragged_4096")
    try:
        batch = synth.make_batch(wl, seed=91, frames=40)
        rule = synth.make_rule(batch, seed=92)
        u = np.random.default_rng(93).random(int((batch.band_ids == 5).sum()))
        be.set_precision("exact")
        want = be.forward_batch(batch, rule=MaskRule(*rule), uniforms=u)
        be.set_precision("certified", tau=1e9)
        be.profile_read(reset=True)
        got = be.forward_batch(batch, rule=MaskRule(*rule), uniforms=u)
        st = be.profile_read(reset=True)
    finally:
        be.destroy()
    assert st["fallback_frames"] == batch.frames
    assert np.array_equal(got["index"], want["index"])
    assert np.array_equal(got["p"], want["p"])


def test_fast_path_accuracy_and_certification_rate(oracle):
    """The raw tensor-core path: p within 1e-5 of the oracle; the certified path
    recomputes only a small share of frames and then matches exactly."""
    wl, cfg, w, be = _backend_for("ragged_4096")
    try:
        batch = synth.make_batch(wl, seed=101, frames=96)
        be.set_precision("fast")
        raw = be.forward_batch(batch)
        be.set_precision("certified")
        be.profile_read(reset=True)
        cert = be.forward_batch(batch)
        st = be.profile_read(reset=True)
    finally:
        be.destroy()
    want = oracle.forward_batch(cfg, w.page, batch)
    err = float(np.abs(raw["p"] - want["p"]).max())
    rel = float(np.max(np.abs(raw["p"] - want["p"]) / np.maximum(want["p"], 1e-30)))
    mism = int((raw["index"] != want["index"]).sum())
    print(f"fast path: max |dp| = {err:.3g}, max rel dp = {rel:.3g}, index mismatches {mism} / {raw['index'].size}, "
          f"frames recomputed by certification {st['fallback_frames']} / {batch.frames}")
    assert err <= 1e-5
    assert st["fallback_frames"] <= batch.frames // 4
    check_batch(cert, want, "certified")


def test_split_overflow_falls_back_to_exact(oracle):
    """Activations too large for the fp16 split raise the overflow word: the batch
    is recomputed exactly, and later batches split at a smaller scale."""
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    w = create_brain_forward_weights(cfg, 13)
    w.embeddings[:64 * 128] *= np.float32(4000.0)  # token rows of ids 0..63: activations in the hundreds
    be = CudaBrainBackend(cfg, w, 0)
    try:
        frames = [[dict(tokens=[int(t) for t in np.random.default_rng(i).integers(1, 64, 3)]) for _ in range(12)]
                  + [dict(query=True, tokens=[5])] for i in range(6)]
        batch = _records_batch(frames)
        be.profile_read(reset=True)
        got = be.forward_batch(batch)
        st = be.profile_read(reset=True)
        again = be.forward_batch(batch)
    finally:
        be.destroy()
    want = oracle.forward_batch(cfg, w.page, batch)
    assert st["fallback_frames"] == batch.frames
    assert np.array_equal(got["index"], want["index"])
    check_batch(again, want, "certified")


def _records_batch(frames):
    from krystal_b200.frame import pack_frame_batch
    return pack_frame_batch(frames)


@pytest.fixture(scope="module")
def small_backend():
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    w = create_brain_forward_weights(cfg, 3)
    be = CudaBrainBackend(cfg, w, 0)
    yield cfg, w, be
    be.destroy()


@pytest.mark.parametrize("mode", MODES)
def test_edge_frames_match_oracle(oracle, small_backend, mode):
    cfg, w, be = small_backend
    be.set_precision(mode)
    rng = np.random.default_rng(9)
    frames = [
        [dict(query=True, tokens=[5]), dict(query=True, tokens=[6, 7])],  # no bank at all
        [dict(tokens=[1, 2]), dict(tokens=[3])],  # no question
        [dict(tokens=[]), dict(tokens=[0, 0]), dict(query=True, tokens=[4]), dict(tokens=[9])],  # empty records
        [dict(tokens=[11]), dict(query=True, tokens=[12])],  # R = 1, Q = 1
        [dict(tokens=[int(t) for t in rng.integers(1, 4000, 8)]) for _ in range(30)]
        + [dict(query=True, tokens=[int(t) for t in rng.integers(1, 4000, 8)]) for _ in range(5)],  # full records
        [dict(tokens=[int(rng.integers(1, 4000))]) for _ in range(40)] + [dict(query=True, tokens=[2])],  # 1-token
        [dict(query=True, tokens=[7])] + [dict(band=int(b), schemaId=int(s), tokens=[int(s) + 1])
                                          for b, s in zip([0, 1, 2, 3, 4, 6, 7] * 3, range(21))],
        [dict(tokens=[3, 0, 5, 0, 7]), dict(query=True, tokens=[0, 9]), dict(tokens=[8, 8, 8])],  # holes
    ]
    batch = _records_batch(frames)
    res = be.forward_batch(batch, want_query_output=True)
    want = oracle.forward_batch(cfg, w.page, batch, want_query_output=True)
    be.set_precision("certified")
    assert np.array_equal(res["q_off"], want["q_off"]) and np.array_equal(res["p_off"], want["p_off"])
    check_batch(res, want, mode, 1.0)
    assert res["index"][0] == abi.KC_NO_SELECTION and res["index"][1] == abi.KC_NO_SELECTION
    # questions of frames with an empty bank carry no query output in the oracle; skip them
    q0 = int(res["q_off"][1])
    tol = 0.0 if mode == "exact" else 1e-4
    assert np.abs(res["query_output"][q0 * 128:] - want["query_output"][q0 * 128:]).max() <= tol


@pytest.mark.parametrize("mode", MODES)
def test_batch_without_token_rows_matches_oracle(oracle, small_backend, mode):
    """Every record rowless (all PAD): no encoder rows at all, every pooled key
    and value zero."""
    cfg, w, be = small_backend
    be.set_precision(mode)
    frames = [[dict(tokens=[]), dict(tokens=[0, 0]), dict(query=True, tokens=[])],
              [dict(query=True, tokens=[0]), dict(tokens=[])]]
    batch = _records_batch(frames)
    res = be.forward_batch(batch, want_query_output=True)
    want = oracle.forward_batch(cfg, w.page, batch, want_query_output=True)
    be.set_precision("certified")
    assert res["total_t"] == 0
    check_batch(res, want, mode, 1.0)
    assert np.abs(res["query_output"] - want["query_output"]).max() <= (0.0 if mode == "exact" else 1e-4)


@pytest.mark.parametrize("mode", MODES)
def test_rule_that_admits_nothing_reopens_the_row(oracle, small_backend, mode):
    cfg, w, be = small_backend
    be.set_precision(mode)
    frames = [[dict(tokens=[i + 1], schemaId=i % 4, band=i % 3) for i in range(12)]
              + [dict(query=True, tokens=[40]), dict(query=True, tokens=[41])]]
    batch = _records_batch(frames)
    schema_allow = np.zeros(16, dtype=np.uint32)
    schema_allow[0] = 0b0010  # question 0: schema 1 only
    band_allow = np.array([0xFF, 0xFF], dtype=np.uint32)  # question 1 admits no schema at all -> reopened
    res = be.forward_batch(batch, rule=MaskRule(schema_allow, band_allow))
    want = oracle.forward_batch(cfg, w.page, batch, rule=(schema_allow, band_allow))
    be.set_precision("certified")
    check_batch(res, want, mode, 1.0)
    p = res["p"].reshape(2, 12)
    assert abs(float(p[1].sum()) - 1) < 1e-5
    assert (p[0][np.arange(12) % 4 != 1] == 0).all()


def test_select_all_blocked_and_sampling(oracle, small_backend):
    cfg, w, be = small_backend
    frame = pack_host_frame([dict(tokens=[i + 1, i + 2]) for i in range(9)] + [dict(query=True, tokens=[5])] * 3)
    enc = be.encode(frame)
    want = oracle.forward(cfg, w.page, frame.gpu)
    assert np.array_equal(enc.query_output, want["query_output"])
    mask = np.zeros(3 * 9, dtype=np.float32)
    mask[:9] = -1e30  # question 0: everything blocked (an explicit mask, not selectionMask)
    u = np.array([0.5, 0.01, 0.97])
    sel = be.select(enc, mask=mask, uniforms=u)
    ref = oracle.selector(want["query_output"], want["bank_keys"], want["bank_values"], mask, w.selector.wq,
                          w.selector.wk, 128, uniforms=u)
    assert sel.index.tolist() == ref["index"].tolist()
    assert sel.index[0] == abi.KC_NO_SELECTION and not sel.p[:9].any()
    assert_p_close(sel.p, ref["p"], 1.0)


def test_errors_are_refused_by_name(small_backend):
    cfg, w, be = small_backend
    with pytest.raises(abi.KrystalCudaError, match="at least one query record"):
        be.encode(pack_host_frame([dict(tokens=[1])]))
    bad = _records_batch([[dict(tokens=[5000]), dict(query=True, tokens=[1])]])  # id beyond tokenRows
    with pytest.raises(abi.KrystalCudaError, match="tokenRows"):
        be.forward_batch(bad)
    bad = _records_batch([[dict(tokens=[5], band=9), dict(query=True, tokens=[1])]])
    with pytest.raises(abi.KrystalCudaError, match="band"):
        be.forward_batch(bad)
    big = _records_batch([[dict(tokens=[1])] * (abi.KC_MAX_BANK + 1) + [dict(query=True, tokens=[2])]])
    with pytest.raises(abi.KrystalCudaError) as e:
        be.forward_batch(big)
    assert e.value.status == abi.KC_ERR_CAPACITY
    empty = FrameBatch(np.array([0, 1, 1], dtype=np.uint64), np.array([1, 0, 0, 0, 0, 0, 0, 0], dtype=np.uint32),
                       np.zeros(8, dtype=np.uint32), np.zeros(1, dtype=np.uint32), np.full(1, 5, dtype=np.uint32))
    with pytest.raises(abi.KrystalCudaError, match="no records"):
        be.forward_batch(empty)
    # the handle is still usable after refusals
    ok = be.encode(pack_host_frame([dict(tokens=[1]), dict(query=True, tokens=[2])]))
    assert ok.query_output.size == 128


def test_active_record_list_ends_at_first_invalid(oracle, small_backend):
    cfg, w, be = small_backend
    frame = pack_host_frame([dict(tokens=[1, 2]), dict(query=True, tokens=[3]), dict(tokens=[4]),
                             dict(tokens=[5, 6, 7])])
    frame.gpu.active_record_indices[2] = 0xFFFFFFFF  # records 2 and 3 are an unoccupied tail
    hf = host_frame(frame.gpu)
    enc = be.encode(hf)
    want = oracle.forward(cfg, w.page, frame.gpu)
    assert want["r"] == 1 and enc.bank_keys.size == 128
    assert np.array_equal(enc.query_output, want["query_output"])
    assert np.array_equal(enc.bank_keys, want["bank_keys"])


def test_sync_takes_up_changed_weights(oracle):
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    w = create_brain_forward_weights(cfg, 11)
    be = CudaBrainBackend(cfg, w, 0)
    try:
        frame = pack_host_frame([dict(tokens=[10, 11]), dict(tokens=[12]), dict(query=True, tokens=[13])])
        rng = np.random.default_rng(0)
        # move the selector and the token row of id 12 (row 12), then tell the backend only that
        w.selector.wq[:] = rng.normal(0, 0.2, w.selector.wq.size).astype(np.float32)
        w.embeddings[12 * 128:13 * 128] += np.float32(0.5)
        be.sync(w, WeightChanges(selector=True, embedding_rows=[12 * 128]))
        enc = be.encode(frame)
        want = oracle.forward(cfg, w.page, frame.gpu)
        assert np.array_equal(enc.bank_keys, want["bank_keys"])
        sel = be.select(enc)
        ref = oracle.selector(want["query_output"], want["bank_keys"], want["bank_values"], None, w.selector.wq,
                              w.selector.wk, 128)
        assert sel.index.tolist() == ref["index"].tolist()
        assert_p_close(sel.p, ref["p"], 1.0)
        # a full sync (restore) after changing the blocks
        w.enc[0].w1[:] *= np.float32(0.5)
        be.sync(w)
        enc = be.encode(frame)
        want = oracle.forward(cfg, w.page, frame.gpu)
        assert np.array_equal(enc.query_output, want["query_output"])
    finally:
        be.destroy()


def test_session_think_matches_oracle_session(oracle):
    rows = np.arange(4096, dtype=np.uint32) % 64
    session = BrainSession(rows, seed=7)
    try:
        world = [dict(schemaId=1, band=3, tokens=[10, 11, 12]), dict(schemaId=1, band=3, tokens=[10, 13]),
                 dict(schemaId=2, band=2, tokens=[20, 21]), dict(schemaId=9, query=True, tokens=[30])]
        res = session.think(world)
        assert len(res.selections) == 1 and res.selections[0].record in (0, 1, 2)
        frame = pack_host_frame(world)
        out = oracle.forward(session.config, session.weights.page, frame.gpu)
        ref = oracle.selector(out["query_output"], out["bank_keys"], out["bank_values"], None,
                              session.weights.selector.wq, session.weights.selector.wk, 128)
        assert res.selections[0].record == int(frame.active.bank_records[ref["index"][0]])
        forbidden = session.think(world, allows=lambda q, rec: rec == 2)
        assert forbidden.selections[0].record == 2
        assert abs(forbidden.selections[0].distribution[0]) < 1e-6
        reopened = session.think(world, allows=lambda q, rec: False)
        assert abs(float(reopened.selections[0].distribution.sum()) - 1) < 1e-5
        assert session.think([dict(tokens=[10])]).selections == []
        mask = selection_mask(frame.active, lambda q, rec: rec != 0)
        assert mask[0] == np.float32(-1e30)
    finally:
        session.destroy()


class _DevArray:
    """A library-owned device array, exposed to torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 2}


def test_device_resident_batch_equals_host_batch():
    torch = pytest.importorskip("torch")
    wl, cfg, w, be = _backend_for("ragged_4096")
    try:
        batch = synth.make_batch(wl, seed=3, frames=32)
        host = be.forward_batch(batch)
        dev = {k: torch.from_numpy(np.ascontiguousarray(getattr(batch, k)).view(np.int32)).cuda()
               for k in ("token_ids", "field_roles", "schema_ids", "band_ids")}
        rec_off = torch.from_numpy(batch.rec_off.astype(np.int64)).cuda()
        torch.cuda.synchronize()
        r = be.forward_batch_device(batch.frames, batch.records, rec_off.data_ptr(), dev["token_ids"].data_ptr(),
                                    dev["field_roles"].data_ptr(), dev["schema_ids"].data_ptr(),
                                    dev["band_ids"].data_ptr())
        be.synchronize()
        p = torch.as_tensor(_DevArray(r.p, r.total_p, "<f4"), device="cuda").cpu().numpy()
        idx = torch.as_tensor(_DevArray(r.index, r.total_q, "<i4"), device="cuda").cpu().numpy().view(np.uint32)
        assert np.array_equal(idx, host["index"])
        assert np.array_equal(p, host["p"])
    finally:
        be.destroy()
