"""Pins the C++ oracle against every known answer the reference's tests hold.

Sources (reference project paths):
  matmulOracle layout KAT      packages/webgpu/test/krystal-forward.test.ts:265-270
  sampleRow KATs               packages/krystal/src/forward/sampling.test.ts:5-23
  packing / active-frame facts packages/krystal/src/host/session.test.ts:16-47
  thinking facts               packages/krystal/src/host/session.test.ts:50-82
  composed fixture sizes       packages/webgpu/test/krystal-composed.test.ts:43-50
  parameter count              docs/ENGINE.md:392-401 (1 773 952 floats, 1 149 184 in the embeddings page)
"""
import numpy as np
import pytest

from krystal_b200.frame import HostFrameError, QUERY_BAND, pack_host_frame, record_ranges
from krystal_b200.model import BRAIN_FORWARD_CONFIG, RECORD_WIDTH, create_brain_forward_weights, \
    embeddings_page_elements, mulberry32_draws, weight_layout
from krystal_b200.session import selection_mask


def rows(count):
    return np.arange(count, dtype=np.uint32) % 64


def world():
    return [
        dict(schemaId=1, band=3, tokens=[10, 11, 12]),  # an apple
        dict(schemaId=1, band=3, tokens=[10, 13]),  # a stone
        dict(schemaId=2, band=2, tokens=[20, 21]),  # a comfort
        dict(schemaId=9, query=True, tokens=[30]),  # what next?
    ]


def test_matmul_layout_kat(oracle):
    out = oracle.matmul(np.array([1, 2, 3, 4]), np.array([1, 0, 0, 1, 2, 2]), 3, 2)
    assert out.tolist() == [1, 2, 6, 3, 4, 14]


def test_sample_row_kats(oracle):
    p = np.array([0.2, 0.5, 0.3], dtype=np.float32)
    assert oracle.sample_row(p, 0.1) == 0
    assert oracle.sample_row(p, 0.6) == 1
    assert oracle.sample_row(p, 0.95) == 2
    assert oracle.sample_row(np.array([0.5, 0.49, 0], dtype=np.float32), 0.999) == 1
    assert oracle.sample_row(np.full(3, np.nan, dtype=np.float32), 0.5) == -1
    assert oracle.sample_row(np.array([np.nan, 0.4, np.nan], dtype=np.float32), 0.9) == 1


def test_parameter_count_and_page_size(oracle):
    lay = weight_layout(BRAIN_FORWARD_CONFIG)
    assert lay.total == 1_773_952
    assert embeddings_page_elements(BRAIN_FORWARD_CONFIG) == 1_149_184
    assert oracle.weight_count(BRAIN_FORWARD_CONFIG) == 1_773_952


def test_mulberry32_matches_vectorised_stream(oracle):
    a = oracle.mulberry32(1337, 4096)
    b = mulberry32_draws(1337, 0, 4096)
    assert np.array_equal(a, b)
    # regression values of the first draws for seed 1
    assert np.allclose(oracle.mulberry32(1, 3), [0.6270739405881613, 0.002735721180215478, 0.5274470399599522])


@pytest.mark.parametrize("seed", [7, 1337])
def test_weight_init_matches_numpy_restatement(oracle, seed):
    a = oracle.create_weights(BRAIN_FORWARD_CONFIG, seed)
    b = create_brain_forward_weights(BRAIN_FORWARD_CONFIG, seed).page
    # libm differences could move an f32 by one ulp in rare cases; none expected
    diff = np.nonzero(a != b)[0]
    assert diff.size <= 2
    if diff.size:
        assert np.max(np.abs(a[diff].view(np.int32) - b[diff].view(np.int32))) <= 1
    # Xavier limits and the N(0, 0.02) embedding scale
    lay = weight_layout(BRAIN_FORWARD_CONFIG)
    enc_wq = a[lay.enc:lay.enc + 128 * 128]
    assert np.abs(enc_wq).max() <= np.sqrt(6 / 256) + 1e-7
    assert abs(a[:lay.enc].std() - 0.02) < 1e-3


def test_packing_is_sized_to_what_it_was_given():
    frame = pack_host_frame(world())
    assert frame.slots == 4
    assert frame.gpu.token_ids.size == 4 * RECORD_WIDTH
    assert frame.active.active_tokens.size == 3 + 2 + 2 + 1


def test_query_record_is_a_question_rest_is_bank(oracle):
    frame = pack_host_frame(world())
    assert frame.active.query_records.tolist() == [3]
    assert frame.active.bank_records.tolist() == [0, 1, 2]
    assert frame.gpu.band_ids[3] == QUERY_BAND
    act = oracle.compile_active(frame.gpu.token_ids, frame.gpu.band_ids, frame.gpu.active_record_indices)
    assert act["query_records"].tolist() == [3]
    assert act["bank_records"].tolist() == [0, 1, 2]
    assert act["active_tokens"].tolist() == frame.active.active_tokens.tolist()


def test_no_token_attends_across_a_record_boundary():
    frame = pack_host_frame([dict(tokens=[1, 2]), dict(tokens=[3])])
    start, count = record_ranges(frame.active)
    assert [start[0], count[0]] == [0, 2]
    assert [start[1], count[1]] == [0, 2]
    assert [start[2], count[2]] == [2, 1]


def test_refusals():
    with pytest.raises(HostFrameError):
        pack_host_frame([dict(tokens=[1, 2, 3, 4, 5, 6, 7, 8, 9])])
    with pytest.raises(HostFrameError):
        pack_host_frame([])
    with pytest.raises(HostFrameError):
        pack_host_frame([dict(tokens=[-1])])


def test_pad_token_is_a_hole_not_a_token(oracle):
    frame = pack_host_frame([dict(tokens=[5, 0, 7]), dict(query=True, tokens=[9])])
    assert frame.active.active_tokens.tolist() == [0, 2, 8]
    act = oracle.compile_active(frame.gpu.token_ids, frame.gpu.band_ids, frame.gpu.active_record_indices)
    assert act["active_tokens"].tolist() == [0, 2, 8]


def _think(oracle, allows=None, seed=7, records=None):
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(rows(4096))
    w = create_brain_forward_weights(cfg, seed)
    frame = pack_host_frame(records or world())
    out = oracle.forward(cfg, w.page, frame.gpu)
    mask = selection_mask(frame.active, allows)
    sel = oracle.selector(out["query_output"], out["bank_keys"], out["bank_values"], mask, w.selector.wq,
                          w.selector.wk, 128)
    return frame, out, sel


def test_composed_fixture_sizes(oracle):
    _, out, _ = _think(oracle)
    assert [out["t"], out["r"], out["q"]] == [8, 3, 1]


def test_every_question_gets_one_choice_from_the_bank(oracle):
    frame, out, sel = _think(oracle)
    assert sel["index"].size == 1 and sel["index"][0] in (0, 1, 2)
    assert sel["p"].size == 3
    assert abs(float(sel["p"].sum()) - 1) < 1e-6


def test_same_weights_same_frame_same_answer(oracle):
    a = _think(oracle)[2]
    b = _think(oracle)[2]
    assert a["index"].tolist() == b["index"].tolist()
    assert np.array_equal(a["p"], b["p"])


def test_forbidden_record_never_chosen_and_carries_no_probability(oracle):
    frame, _, sel = _think(oracle, allows=lambda q, rec: rec == 2)
    assert frame.active.bank_records[sel["index"][0]] == 2
    assert abs(sel["p"][0]) < 1e-6 and abs(sel["p"][1]) < 1e-6


def test_question_nothing_admits_is_reopened(oracle):
    _, _, sel = _think(oracle, allows=lambda q, rec: False)
    assert abs(float(sel["p"].sum()) - 1) < 1e-5


def test_all_blocked_row_selects_nothing(oracle):
    # an explicit mask (not selectionMask) that blocks everything: p = 0, index = NO_SELECTION
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(rows(4096))
    w = create_brain_forward_weights(cfg, 7)
    frame = pack_host_frame(world())
    out = oracle.forward(cfg, w.page, frame.gpu)
    sel = oracle.selector(out["query_output"], out["bank_keys"], out["bank_values"],
                          np.full(3, -1e30, dtype=np.float32), w.selector.wq, w.selector.wk, 128)
    assert sel["index"][0] == 0xFFFFFFFF
    assert not sel["p"].any()


def test_sampling_draws_by_inverse_cdf(oracle):
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(rows(4096))
    w = create_brain_forward_weights(cfg, 7)
    frame = pack_host_frame(world())
    out = oracle.forward(cfg, w.page, frame.gpu)
    args = (out["query_output"], out["bank_keys"], out["bank_values"], None, w.selector.wq, w.selector.wk, 128)
    p = oracle.selector(*args)["p"]
    cum = np.cumsum(p.astype(np.float64))
    for u, want in ((0.0, 0), (float(cum[0]) + 1e-6, 1), (0.999999, 2)):
        assert oracle.selector(*args, uniforms=np.array([u]))["index"][0] == want


def test_selection_mask_rule_equals_closure_mask(oracle):
    rng = np.random.default_rng(5)
    recs = [dict(schemaId=int(rng.integers(0, 16)), band=int(rng.choice([0, 1, 2, 3, 4, 6, 7])),
                 tokens=[int(t) for t in rng.integers(1, 50, rng.integers(1, 9))]) for _ in range(20)]
    recs += [dict(query=True, tokens=[3]) for _ in range(4)]
    frame = pack_host_frame(recs)
    schema_allow = rng.integers(0, 2 ** 32, 4 * 8, dtype=np.uint64).astype(np.uint32)
    band_allow = np.array([0b11010011, 0, 0xFF, 0b1], dtype=np.uint32)

    def allows(q, slot):
        s, b = int(frame.gpu.schema_ids[slot]), int(frame.gpu.band_ids[slot])
        return bool((schema_allow[q * 8 + (s >> 5)] >> (s & 31)) & 1) and bool((band_allow[q] >> b) & 1)

    want = selection_mask(frame.active, allows)
    got = oracle.selection_mask_rule(frame.active.bank_records, frame.gpu.schema_ids, frame.gpu.band_ids,
                                     schema_allow, band_allow, 4)
    assert np.array_equal(got, want)
