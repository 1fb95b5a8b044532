"""GPU parity of the backward (forward/backward.ts:751-982 as host/gradients.ts:
30-66 requests it): the CUDA path through the C ABI against the oracle's
restatement, which test_oracle_backward.py pins by finite differences.

The bar is the reference's own gradient tolerance, max-abs 1e-4
(packages/webgpu/test/krystal-composed.test.ts:149-157). The device backward
follows the oracle's arithmetic (f64 accumulation in its order, f32 stores), so
nearly every value is expected to be bit-identical as well.
"""
import numpy as np
import pytest

from krystal_b200 import abi, synth
from krystal_b200.backend import CudaBrainBackend
from krystal_b200.frame import BrainFrameGpu, HostFrame, QUERY_BAND, compile_active_frame, pack_host_frame
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights
from krystal_b200.session import selection_mask

pytestmark = pytest.mark.gpu

TOL = 1e-4
FIELDS = ("policy", "value_prediction", "d_selector_wq", "d_selector_wk", "d_pool", "d_field_states", "d_value_wv")
NO, AWAY = abi.KC_NO_TARGET, abi.KC_AWAY_TARGET


def host_frame(g: BrainFrameGpu) -> HostFrame:
    return HostFrame(g, compile_active_frame(g), g.schema_ids.size)


def compare(got: dict, want: dict, exact_share: float = 0.99) -> None:
    for k in FIELDS:
        a, b = np.asarray(got[k], np.float32), np.asarray(want[k], np.float32)
        assert a.shape == b.shape, k
        if a.size == 0:
            continue
        err = float(np.abs(a.astype(np.float64) - b).max())
        assert err <= TOL, f"{k}: max abs {err}"
        assert np.mean(a == b) >= exact_share, f"{k}: {np.mean(a == b)} bit-identical"
    assert abs(got["value_loss"] - want["value_loss"]) <= TOL * max(1.0, abs(want["value_loss"]))


def as_dict(r) -> dict:
    return {k: getattr(r, k) for k in FIELDS + ("value_loss",)}


def small_world(seed=7):
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    w = create_brain_forward_weights(cfg, seed)
    rng = np.random.default_rng(seed)
    recs = [dict(schemaId=int(rng.integers(0, 8)), band=int(rng.choice([0, 1, 2, 3])),
                 tokens=[int(t) for t in rng.integers(1, 60, rng.integers(1, 9))]) for _ in range(9)]
    recs += [dict(query=True, tokens=[int(t) for t in rng.integers(1, 60, 3)]) for _ in range(3)]
    frame = pack_host_frame(recs)
    mask = selection_mask(frame.active, lambda q, slot: (q + slot) % 4 != 0)
    return cfg, w, frame, mask


@pytest.fixture(scope="module")
def small():
    cfg, w, frame, mask = small_world()
    be = CudaBrainBackend(cfg, w, 0)
    yield cfg, w, frame, mask, be
    be.destroy()


@pytest.mark.parametrize("targets", [None, [1, NO, 4], [AWAY | 2, 4, NO], [NO, NO, NO]])
@pytest.mark.parametrize("valence", [None, 0.3, -1.7])
def test_backward_matches_oracle(oracle, small, targets, valence):
    cfg, w, frame, mask, be = small
    tg = None if targets is None else np.array(targets, np.uint32)
    got = be.backward(frame, mask, tg, valence)
    want = oracle.backward(cfg, w.page, frame.gpu, mask, tg, valence)
    compare(as_dict(got), want)
    if valence is None:
        assert got.value_loss == 0.0 and not np.any(got.d_value_wv)


def test_backward_open_selection_equals_zero_mask(small):
    cfg, w, frame, mask, be = small
    q, r = frame.active.query_records.size, frame.active.bank_records.size
    a = be.backward(frame, None, np.array([0, 1, 2], np.uint32), 0.5)
    b = be.backward(frame, np.zeros(q * r, np.float32), np.array([0, 1, 2], np.uint32), 0.5)
    for k in FIELDS:
        assert np.array_equal(getattr(a, k), getattr(b, k)), k


def test_backward_fully_blocked_row(oracle, small):
    """A question whose every bank record is blocked: p = 0 and no offered mean."""
    cfg, w, frame, mask, be = small
    m = mask.copy().reshape(3, -1)
    m[1, :] = np.float32(-1e30)
    m = m.reshape(-1)
    tg = np.array([AWAY | 0, 3, NO], np.uint32)
    got = be.backward(frame, m, tg, 0.25)
    want = oracle.backward(cfg, w.page, frame.gpu, m, tg, 0.25)
    compare(as_dict(got), want)
    assert not np.any(got.policy.reshape(3, -1)[1])


def test_backward_after_sync(oracle, small):
    """The backward multiplies by transposed weight copies: a sync must refresh them."""
    cfg, w, frame, mask, be = small
    w2 = create_brain_forward_weights(cfg, 99)
    try:
        be.sync(w2)
        tg = np.array([2, NO, 0], np.uint32)
        compare(as_dict(be.backward(frame, mask, tg, 1.0)), oracle.backward(cfg, w2.page, frame.gpu, mask, tg, 1.0))
    finally:
        be.sync(w)


def test_backward_refuses_a_frame_without_questions(small):
    cfg, w, frame, mask, be = small
    g = pack_host_frame([dict(tokens=[3, 4]), dict(tokens=[5])])
    with pytest.raises(abi.KrystalCudaError) as e:
        be.backward(g, None, None, 0.1)
    assert e.value.status == abi.KC_ERR_INVALID_ARG


def _targets(rng, q, r):
    t = rng.integers(0, r, q).astype(np.uint32)
    kind = rng.integers(0, 4, q)
    t[kind == 0] = NO
    t[kind == 1] |= AWAY
    return t


@pytest.fixture(scope="module")
def ragged():
    wl = synth.WORKLOADS["ragged_4096"]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    be = CudaBrainBackend(cfg, w, 0)
    yield wl, cfg, w, be
    be.destroy()


def test_backward_single_frame_is_exact_at_any_precision(oracle, ragged):
    """kc_backward (the per-frame seam) always computes in the oracle's arithmetic."""
    wl, cfg, w, be = ragged
    g = synth.make_batch(wl, seed=12, frames=1).frame(0)
    frame = host_frame(g)
    q, r = frame.active.query_records.size, frame.active.bank_records.size
    tg = _targets(np.random.default_rng(1), q, r)
    be.set_precision("certified")
    a = be.backward(frame, None, tg, 0.4)
    be.set_precision("exact")
    b = be.backward(frame, None, tg, 0.4)
    be.set_precision("certified")
    for k in FIELDS:
        assert np.array_equal(getattr(a, k), getattr(b, k)), k


def test_backward_ragged_frames_match_oracle(oracle, ragged):
    wl, cfg, w, be = ragged
    batch = synth.make_batch(wl, seed=11, frames=4)
    rng = np.random.default_rng(5)
    for f in range(batch.frames):
        g = batch.frame(f)
        frame = host_frame(g)
        q, r = frame.active.query_records.size, frame.active.bank_records.size
        mask = selection_mask(frame.active, lambda i, slot: (i * 7 + slot) % 3 != 0)
        tg = _targets(rng, q, r)
        val = float(rng.normal())
        compare(as_dict(be.backward(frame, mask, tg, val)), oracle.backward(cfg, w.page, g, mask, tg, val))


def test_backward_long_bank_matches_oracle(oracle, ragged):
    """A 1024-record bank: the selector and mixer backward walk long rows."""
    wl, cfg, w, be = ragged
    long = synth.Workload("long", 1, (1032, 1032), (8, 8), wl.vocab, 64, bank=1024)
    g = synth.make_batch(long, seed=4).frame(0)
    frame = host_frame(g)
    rng = np.random.default_rng(9)
    tg = _targets(rng, 8, 1024)
    mask = selection_mask(frame.active, lambda i, slot: slot % 5 != i % 5)
    compare(as_dict(be.backward(frame, mask, tg, 0.7)), oracle.backward(cfg, w.page, g, mask, tg, 0.7))


class _DevArray:
    """A library-owned device array, exposed to torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 2}


def _rule_mask(batch, f, schema_allow, band_allow, q0):
    """selectionMask (host/learn.ts:215-232) for the device rule of frame f."""
    g = batch.frame(f)
    act = compile_active_frame(g)
    sa = schema_allow.reshape(-1, 8)

    def allows(i, slot):
        s, b = int(g.schema_ids[slot]), int(g.band_ids[slot])
        return bool((sa[q0 + i][s >> 5] >> (s & 31)) & 1) and bool((band_allow[q0 + i] >> b) & 1)

    return selection_mask(act, allows)


@pytest.mark.parametrize("precision", ["exact", "certified"])
@pytest.mark.parametrize("use_rule", [False, True])
def test_backward_batch_device_matches_oracle(oracle, ragged, use_rule, precision):
    """The batch backward: on the FP64 path (exact) nearly every value is
    bit-identical; on the tensor cores (the handle's default) within 1e-4."""
    torch = pytest.importorskip("torch")
    wl, cfg, w, be = ragged
    be.set_precision(precision)
    batch = synth.make_batch(wl, seed=21, frames=6)
    F = batch.frames
    rng = np.random.default_rng(3)
    frames = [batch.frame(f) for f in range(F)]
    acts = [compile_active_frame(g) for g in frames]
    qs = [a.query_records.size for a in acts]
    rs = [a.bank_records.size for a in acts]
    q_off = np.concatenate([[0], np.cumsum(qs)]).astype(np.int64)
    schema_allow, band_allow = synth.make_rule(batch, seed=8)
    masks = []
    for f in range(F):
        if use_rule:
            masks.append(_rule_mask(batch, f, schema_allow, band_allow, int(q_off[f])))
        else:
            masks.append(selection_mask(acts[f], lambda i, slot: (i + 2 * slot) % 5 != 1))
    targets = [_targets(rng, qs[f], rs[f]) for f in range(F)]
    valence = rng.normal(size=F)
    valence[2] = np.nan  # no value target for frame 2
    dev = {k: torch.from_numpy(np.ascontiguousarray(getattr(batch, k)).view(np.int32)).cuda()
           for k in ("token_ids", "field_roles", "schema_ids", "band_ids")}
    rec_off = torch.from_numpy(batch.rec_off.astype(np.int64)).cuda()
    sel = torch.from_numpy(np.concatenate(masks).astype(np.float32)).cuda()
    tg = torch.from_numpy(np.concatenate(targets).view(np.int32)).cuda()
    val = torch.from_numpy(valence).cuda()
    sa = torch.from_numpy(schema_allow.view(np.int32)).cuda()
    ba = torch.from_numpy(band_allow.view(np.int32)).cuda()
    torch.cuda.synchronize()
    res = be.backward_batch_device(F, batch.records, rec_off.data_ptr(), dev["token_ids"].data_ptr(),
                                   dev["field_roles"].data_ptr(), dev["schema_ids"].data_ptr(),
                                   dev["band_ids"].data_ptr(), None if use_rule else sel.data_ptr(),
                                   tg.data_ptr(), val.data_ptr(), sa.data_ptr() if use_rule else None,
                                   ba.data_ptr() if use_rule else None)
    be.synchronize()
    H = cfg.hidden_size

    def get(ptr, n, t="<f4"):
        return torch.as_tensor(_DevArray(ptr, n, t), device="cuda").cpu().numpy()

    offs = {k: get(getattr(res, k), F + 1, "<i8") for k in ("p_off", "q_off", "t_off")}
    policy = get(res.policy, res.total_p)
    pred = get(res.value_prediction, res.total_q)
    loss = get(res.value_loss, F, "<f8")
    dwq, dwk = get(res.d_selector_wq, F * H * H), get(res.d_selector_wk, F * H * H)
    dpool, dwv = get(res.d_pool, F * 2 * H), get(res.d_value_wv, F * 3 * H)
    dfs = get(res.d_field_states, res.total_t * H)
    for f in range(F):
        v = None if np.isnan(valence[f]) else float(valence[f])
        want = oracle.backward(cfg, w.page, frames[f], masks[f], targets[f], v)
        po, qo, to = (int(offs[k][f]) for k in ("p_off", "q_off", "t_off"))
        got = {"policy": policy[po:po + qs[f] * rs[f]], "value_prediction": pred[qo:qo + qs[f]],
               "value_loss": float(loss[f]), "d_selector_wq": dwq[f * H * H:(f + 1) * H * H],
               "d_selector_wk": dwk[f * H * H:(f + 1) * H * H], "d_pool": dpool[f * 2 * H:(f + 1) * 2 * H],
               "d_value_wv": dwv[f * 3 * H:(f + 1) * 3 * H],
               "d_field_states": dfs[to * H:(to + acts[f].active_tokens.size) * H]}
        compare(got, want, 0.99 if precision == "exact" else 0.0)
    be.set_precision("certified")
