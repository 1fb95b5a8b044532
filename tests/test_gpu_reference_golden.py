"""The CUDA path, through the C ABI, against outputs of the reference's own
TypeScript code (tests/golden/reference_*.npz, made by executing the
reference's source files on these inputs; tests/test_reference_golden.py
pins the oracle to the same fixtures).

The bar is the one the reference's composed test sets
(packages/webgpu/test/krystal-composed.test.ts:67-69): selected indices
exact, distributions within 1e-4; on the exact path the distributions are
also bit-identical for all but a vanishing share of entries."""
import numpy as np
import pytest

from krystal_b200.backend import CudaBrainBackend, MaskRule
from krystal_b200.frame import HostFrame, compile_active_frame
from tests import golden_io as G
from tests.test_reference_golden import REFERENCE_BATCHES

pytestmark = pytest.mark.gpu

P_TOL = 1e-4
MODES = ["exact", "certified"]


def ref(name: str) -> dict:
    return G.load(f"reference_{name}")


def check(got_p, got_index, want_p, want_index, mode):
    assert np.array_equal(got_index, want_index)
    assert got_p.shape == want_p.shape
    if got_p.size:
        assert np.abs(got_p - want_p).max() <= P_TOL
        if mode == "exact":
            assert np.mean(got_p == want_p) >= 0.9999


def test_composed_frame_matches_reference():
    """The composed test's frame: encode and select (under its grammar, and open) against the reference's run."""
    r = ref("test_records")
    g, cfg, w, frame = G.test_records()
    be = CudaBrainBackend(cfg, w, 0)
    try:
        enc = be.encode(HostFrame(frame, compile_active_frame(frame), frame.schema_ids.size))
        assert np.array_equal(enc.query_output, r["query_output"])
        assert np.array_equal(enc.bank_keys, r["bank_keys"])
        assert np.array_equal(enc.bank_values, r["bank_values"])
        for tag, mask in (("", r["grammar"]), ("_open", None)):
            sel = be.select(enc, mask=mask)
            check(sel.p, sel.index, r["p" + tag], r["index" + tag], "exact")
            assert np.abs(sel.gather - r["gather" + tag]).max() <= 1e-6
    finally:
        be.destroy()


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", REFERENCE_BATCHES)
def test_batch_matches_reference(name, mode):
    """Every frame of a batch fixture, with its schema x band rule and sampler where it has them."""
    r = ref(name)
    g, cfg, w, b, rule, u = G.batch(name)
    be = CudaBrainBackend(cfg, w, 0)
    try:
        be.set_precision(mode)
        res = be.forward_batch(b, rule=MaskRule(*rule) if rule else None, uniforms=u, want_query_output=True)
    finally:
        be.destroy()
    check(res["p"], res["index"], r["p"], r["index"], mode)
    assert np.abs(res["query_output"] - r["query_output"]).max() <= (1e-5 if mode == "exact" else 1e-4)


@pytest.mark.parametrize("mode", MODES)
def test_word_bias_matches_reference(mode):
    """compileRecordMask's same-word bias on the 64-record frame, alpha 1.5 and -3.0."""
    r = ref("word_bias_64")
    g, cfg, w, b, _, _ = G.batch("single_frame_64")
    be = CudaBrainBackend(cfg, w, 0)
    try:
        be.set_precision(mode)
        for tag in ("pos", "neg"):
            res = be.forward_batch(b, word_ids=r["word_ids"], word_alpha=float(r[f"{tag}_alpha"]),
                                   want_query_output=True)
            check(res["p"], res["index"], r[f"{tag}_p"], r[f"{tag}_index"], mode)
            assert np.abs(res["query_output"] - r[f"{tag}_query_output"]).max() <= 1e-4
    finally:
        be.destroy()


@pytest.mark.parametrize("mode", MODES)
def test_long_bank_frame_matches_reference(mode):
    """A 4096-record bank with 64 questions: selected open and under a schema x band rule."""
    from tests.test_reference_golden import long_bank_frame
    r, cfg, w, b = long_bank_frame()
    be = CudaBrainBackend(cfg, w, 0)
    try:
        be.set_precision(mode)
        for tag, rule in (("open", None), ("rule", MaskRule(r["schema_allow"], r["band_allow"]))):
            res = be.forward_batch(b, rule=rule, want_query_output=True)
            check(res["p"], res["index"], r[f"p_{tag}"], r[f"index_{tag}"], mode)
            assert np.abs(res["query_output"] - r["query_output"]).max() <= (1e-5 if mode == "exact" else 1e-4)
    finally:
        be.destroy()


@pytest.mark.parametrize("mode", MODES)
def test_edge_frames_match_reference(mode):
    """Frames without a bank or a question, empty records, holes, 1-token and full records; the rule that
    admits nothing (reopened row); a question whose every record is blocked, with sampling."""
    from krystal_b200 import abi
    from krystal_b200.frame import pack_frame_batch, pack_host_frame
    from tests.test_reference_golden import edge_world
    r = ref("edges")
    E, cfg, w = edge_world()
    be = CudaBrainBackend(cfg, w, 0)
    try:
        be.set_precision(mode)
        batch = pack_frame_batch(E.edge_frames())
        res = be.forward_batch(batch, want_query_output=True)
        check(res["p"], res["index"], r["p"], r["index"], mode)
        offs = batch.offsets()  # frames without bank records define no query output (session.ts:133)
        rows = np.repeat(np.repeat(offs["r"] > 0, offs["q"].astype(np.int64)), 128)
        assert np.abs(res["query_output"][rows] - r["query_output"][rows]).max() <= (0.0 if mode == "exact" else 1e-4)
        recs, schema_allow, band_allow = E.reopen_frame()
        res = be.forward_batch(pack_frame_batch([recs]), rule=MaskRule(schema_allow, band_allow))
        check(res["p"], res["index"], r["reopen_p"], r["reopen_index"], mode)
        recs, mask, uniforms = E.blocked_frame()
        enc = be.encode(pack_host_frame(recs))
        sel = be.select(enc, mask=mask, uniforms=uniforms)
        check(sel.p, sel.index, r["blocked_p"], r["blocked_index"], "exact")
        assert sel.index[0] == abi.KC_NO_SELECTION
        assert np.abs(sel.gather - r["blocked_gather"]).max() <= 1e-6
    finally:
        be.destroy()
