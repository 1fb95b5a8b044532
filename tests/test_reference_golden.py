"""The oracle against outputs of the reference's own TypeScript code.

The reference_*.npz fixtures were made by tests/golden/make_reference_golden.py,
which executes the reference's source files (createBrainForwardWeights,
packHostFrame, compileActiveFrame, brainForwardOracle, selectionMask,
selectorOracle with its sampler, compileRecordMask, cpuGradients ->
brainBackwardOracle, learnFromExperience, teachFromDemonstration) under
JavaScript's number semantics on the inputs of the other golden fixtures and
of the learn/teach tests. Here the C++ oracle, the oracle's learn and teach
restatements, the weight generator and the host packing must reproduce them
bit for bit, so the oracle every GPU test is checked against is pinned to the
reference itself."""
import numpy as np
import pytest

from krystal_b200.frame import compile_active_frame, pack_host_frame
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights, weight_layout
from tests import golden_io as G
from tests.golden.make_golden import TEST_RECORDS


def ref(name: str) -> dict:
    return G.load(f"reference_{name}")


def bits_equal(a, b) -> bool:
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_weight_pages_match_reference(oracle):
    """createBrainForwardWeights (model.ts:233-265): the vectorised generator and the oracle's, every float."""
    r = ref("weights")
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    for seed in (7, 1337, 3):
        assert G.sha(create_brain_forward_weights(cfg, seed).page) == str(r[f"sha_{seed}"]), seed
        assert G.sha(oracle.create_weights(cfg, seed)) == str(r[f"sha_{seed}"]), seed


def test_host_packing_matches_reference():
    """packHostFrame (frame.ts:72-115) and compileActiveFrame (masks.ts:65-101) on the composed test's records."""
    r = ref("test_records")
    hf = pack_host_frame(TEST_RECORDS)
    assert np.array_equal(hf.gpu.token_ids, r["token_ids"])
    assert np.array_equal(hf.gpu.schema_ids, r["schema_ids"])
    assert np.array_equal(hf.gpu.band_ids, r["band_ids"])
    assert np.array_equal(hf.gpu.active_record_indices, r["active_record_indices"])
    act = compile_active_frame(hf.gpu)
    assert np.array_equal(act.active_tokens, r["active_tokens"])
    assert np.array_equal(act.bank_records, r["bank_records"])
    assert np.array_equal(act.query_records, r["query_records"])


def test_composed_forward_matches_reference(oracle):
    """brainForwardOracle and selectorOracle on the composed test's frame (krystal-composed.test.ts:40-60)."""
    r = ref("test_records")
    g, cfg, w, frame = G.test_records()
    assert G.sha(w.page) == str(r["weights_sha"])
    out = oracle.forward(cfg, w.page, frame)
    for k in ("field_states", "bank_keys", "bank_values", "query_keys", "query_output"):
        assert bits_equal(out[k], r[k]), k
    # brainForwardOracle runs its mixer on the pooled queryValues array in place (`let query = queryValues`,
    # oracle.ts:289-296), so the result's queryValues is the mixed output; the oracle keeps the pooled rows
    assert bits_equal(r["query_values"], r["query_output"])
    for tag, mask in (("", r["grammar"]), ("_open", None)):
        sel = oracle.selector(out["query_output"], out["bank_keys"], out["bank_values"], mask, w.selector.wq,
                              w.selector.wk, 128)
        assert bits_equal(sel["p"], r["p" + tag]) and np.array_equal(sel["index"], r["index" + tag]), tag
        assert bits_equal(sel["gather"], r["gather" + tag]), tag
    # the committed oracle fixture the GPU tests use holds the same numbers
    for k in ("field_states", "bank_keys", "bank_values", "query_output", "p", "index", "gather"):
        assert np.array_equal(g[k], r[k]), k


@pytest.mark.parametrize("name,targets,valence,open_selection", [
    ("toward", [1], 0.5, False),
    ("away", [0x80000000 | 1], None, False),
    ("critic", None, -0.25, True),
])
def test_backward_matches_reference(oracle, name, targets, valence, open_selection):
    """cpuGradients (host/gradients.ts:30-66) -> brainBackwardOracle (forward/backward.ts:751-982):
    the pointer loss toward a target, away from one (the AWAY bit), and the critic alone."""
    r = ref("test_records")
    g, cfg, w, frame = G.test_records()
    sel = np.zeros_like(r["grammar"]) if open_selection else r["grammar"]
    tg = None if targets is None else np.array(targets, dtype=np.uint32)
    out = oracle.backward(cfg, w.page, frame, sel, targets=tg, valence=valence)
    for k in ("policy", "value_prediction", "d_selector_wq", "d_selector_wk", "d_pool", "d_field_states",
              "d_value_wv"):
        assert bits_equal(out[k], r[f"{name}_{k}"]), k
    assert out["value_loss"] == float(r[f"{name}_value_loss"])


REFERENCE_BATCHES = G.BATCHES


@pytest.mark.parametrize("name", REFERENCE_BATCHES)
def test_batches_match_reference(oracle, name):
    """Every frame of the batch fixtures: packHostFrame, brainForwardOracle, selectionMask (learn.ts:215-232)
    under the fixture's schema x band rule, selectorOracle and sampleRow (sampling.ts:41-57)."""
    r = ref(name)
    g, cfg, w, b, rule, u = G.batch(name)
    assert G.sha(w.page) == str(r["weights_sha"])
    res = oracle.forward_batch(cfg, w.page, b, rule=rule, uniforms=u, want_query_output=True)
    assert np.array_equal(res["index"], r["index"])
    assert bits_equal(res["p"], r["p"])
    assert bits_equal(res["query_output"], r["query_output"])
    for k in ("p", "index", "query_output"):  # the committed oracle fixture the GPU tests use
        assert np.array_equal(g[k], r[k]), k


def test_word_bias_matches_reference(oracle):
    """compileRecordMask with a WordBias (masks.ts:145-198) through brainForwardOracle's local attention."""
    r = ref("word_bias_64")
    g, cfg, w, b, _, _ = G.batch("single_frame_64")
    assert G.sha(w.page) == str(r["weights_sha"])
    frame = b.frame(0)
    for tag in ("pos", "neg"):
        out = oracle.forward(cfg, w.page, frame, word_ids=r["word_ids"], alpha=float(r[f"{tag}_alpha"]))
        assert bits_equal(out["query_output"], r[f"{tag}_query_output"]), tag
        sel = oracle.selector(out["query_output"], out["bank_keys"], out["bank_values"], None, w.selector.wq,
                              w.selector.wk, 128)
        assert bits_equal(sel["p"], r[f"{tag}_p"]) and np.array_equal(sel["index"], r[f"{tag}_index"]), tag


def _page_parts(page):
    L = weight_layout(BRAIN_FORWARD_CONFIG)
    h = 128
    spans = {"embeddings": (0, L.enc), "selector_wq": (L.selector_wq, L.selector_wq + h * h),
             "selector_wk": (L.selector_wk, L.selector_wk + h * h), "value_head": (L.value_head, L.value_head + 3 * h),
             "pool": (L.pool, L.pool + 2 * h)}
    return {k: G.sha(page[a:b]) for k, (a, b) in spans.items()}


@pytest.mark.parametrize("name,kw,opts", [
    ("default", dict(n=6, seed=5, skip_reward=(2,), no_choice=(4,)), {}),
    ("unfrozen", dict(n=6, seed=9), dict(unfreeze_pool=True, unfreeze_tokens=True, learning_rate=0.1)),
    ("rejected", dict(n=5, seed=11), dict(max_parameter_abs=1e-3)),
])
def test_learn_matches_reference(name, kw, opts):
    """learnFromExperience (host/learn.ts:280-512, gradients from cpuGradients): the oracle's restatement
    leaves the same weight page, float for float, and reports the same readings."""
    from oracle import learn_oracle as LO
    from tests.learn_cases import experiences, oracle_experiences, world
    r = ref("learn")
    cfg, w = world(3)
    page, rep = LO.learn_from_experience(cfg, w.page, oracle_experiences(experiences(**kw)), LO.Options(**opts))
    for k, v in _page_parts(page).items():
        assert v == str(r[f"{name}_sha_{k}"]), k
    assert G.sha(page) == str(r[f"{name}_sha"])
    for k, js in (("frames_seen", "framesSeen"), ("mean_advantage", "meanAdvantage"),
                  ("mean_value_loss", "meanValueLoss"), ("reinforced", "reinforced"), ("discouraged", "discouraged"),
                  ("mean_entropy", "meanEntropy"), ("mean_confidence", "meanConfidence"),
                  ("update_applied", "updateApplied")):
        assert float(rep[k]) == float(r[f"{name}_{js}"]), k
    assert (rep["rejected"] or "") == str(r[f"{name}_rejected"])
    for k, js in (("semantic_embedding_max_abs", "semanticEmbeddingMaxAbs"), ("selector_max_abs", "selectorMaxAbs"),
                  ("value_max_abs", "valueMaxAbs"), ("pool_max_abs", "poolMaxAbs")):
        assert float(rep["health"][k]) == float(r[f"{name}_health_{js}"]), k


@pytest.mark.parametrize("name,kw,opts", [
    ("default", dict(n=3, seed=7, forbid=(1,)), {}),
    ("frozen", dict(n=4, seed=13, forbid=(0, 2), nothing=(3,)), dict(unfreeze_tokens=False, learning_rate=0.5)),
])
def test_teach_matches_reference(name, kw, opts):
    """teachFromDemonstration (host/teach.ts:126-272): showings applied one after another, each
    differentiated on the weights the previous one left."""
    from oracle import teach_oracle as TO
    from tests.learn_cases import world
    from tests.teach_cases import demonstrations, oracle_demonstrations
    r = ref("teach")
    cfg, w = world(3)
    page, rep = TO.teach_from_demonstration(cfg, w.page, oracle_demonstrations(demonstrations(**kw)),
                                            TO.Options(**opts))
    for k, v in _page_parts(page).items():
        assert v == str(r[f"{name}_sha_{k}"]), k
    assert G.sha(page) == str(r[f"{name}_sha"])
    for k, js in (("frames_seen", "framesSeen"), ("shown", "shown"), ("mean_agreement", "meanAgreement"),
                  ("max_parameter_abs", "maxParameterAbs"), ("rejected", "rejected"), ("clipped", "clipped")):
        assert float(rep[k]) == float(r[f"{name}_{js}"]), k


def test_reference_unit_tests_pass_under_the_runner():
    """The runner that made these fixtures, checked on the reference's own CPU unit tests
    (sampling, session, checkpoint, learn and teach test files; tests/golden/run_reference_tests.py):
    none of their assertions failed under it. A test the record lists as not run trained for longer
    than its time budget at the runner's Python speed; every file has tests that ran to completion."""
    import json
    record = json.loads((G.GOLDEN / "reference_unit_tests.json").read_text())
    assert set(record) == {"forward/sampling.test.ts", "host/session.test.ts", "host/checkpoint.test.ts",
                           "host/learn.test.ts", "host/teach.test.ts"}
    for f, tests in record.items():
        assert tests and all(t is not None for t in tests), f
        assert not [t["test"] for t in tests if t["status"] == "failed"], f
        assert sum(t["status"] == "passed" for t in tests) >= max(1, len(tests) // 2), f


def long_bank_frame():
    """The reference-run long-bank frame (4096 bank records + 64 questions, token ids over 4096 rows)."""
    from krystal_b200 import synth
    from krystal_b200.frame import FrameBatch
    r = ref("long_bank_frame")
    wl = synth.WORKLOADS["ragged_4096"]  # the same 4096-row token table and weights
    assert int(r["vocab"]) == wl.vocab
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    b = FrameBatch(r["rec_off"], r["token_ids"], r["field_roles"], r["schema_ids"], r["band_ids"])
    return r, cfg, w, b


@pytest.mark.parametrize("tag", ["open", "rule"])
def test_long_bank_frame_matches_reference(oracle, tag):
    """The pointer softmax over a 4096-record bank (oracle.ts:332-382), open and under a schema x band rule."""
    r, cfg, w, b = long_bank_frame()
    assert G.sha(w.page) == str(r["weights_sha"])
    rule = (r["schema_allow"], r["band_allow"]) if tag == "rule" else None
    res = oracle.forward_batch(cfg, w.page, b, rule=rule, want_query_output=True)
    assert np.array_equal(res["index"], r[f"index_{tag}"])
    assert bits_equal(res["p"], r[f"p_{tag}"])
    assert bits_equal(res["query_output"], r["query_output"])


def edge_world():
    from tests import edge_cases as E
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(E.token_rows())
    return E, cfg, create_brain_forward_weights(cfg, E.WEIGHT_SEED)


def test_edge_frames_match_reference(oracle):
    """Frames without a bank or a question, empty records, holes, 1-token and full records (tests/edge_cases.py)."""
    from krystal_b200.frame import pack_frame_batch
    r = ref("edges")
    E, cfg, w = edge_world()
    assert G.sha(w.page) == str(r["weights_sha"])
    batch = pack_frame_batch(E.edge_frames())
    res = oracle.forward_batch(cfg, w.page, batch, want_query_output=True)
    assert np.array_equal(res["index"], r["index"])
    assert bits_equal(res["p"], r["p"])
    # A frame without bank records has no query output to compare: the session never encodes one
    # (consider returns no selections first, session.ts:133), and the batch path defines none for it.
    offs = batch.offsets()
    has_bank = np.repeat(offs["r"] > 0, offs["q"].astype(np.int64))
    rows = np.repeat(has_bank, 128)
    assert bits_equal(res["query_output"][rows], r["query_output"][rows])


def test_reopened_and_blocked_rows_match_reference(oracle):
    """selectionMask's reopened row (learn.ts:229) and selectorOracle's all-blocked row with sampling
    (oracle.ts:356-370, sampling.ts:41-57)."""
    from krystal_b200.frame import pack_frame_batch
    r = ref("edges")
    E, cfg, w = edge_world()
    recs, schema_allow, band_allow = E.reopen_frame()
    res = oracle.forward_batch(cfg, w.page, pack_frame_batch([recs]), rule=(schema_allow, band_allow))
    assert np.array_equal(res["index"], r["reopen_index"]) and bits_equal(res["p"], r["reopen_p"])
    recs, mask, uniforms = E.blocked_frame()
    frame = pack_host_frame(recs)
    out = oracle.forward(cfg, w.page, frame.gpu)
    assert bits_equal(out["query_output"], r["blocked_query_output"])
    sel = oracle.selector(out["query_output"], out["bank_keys"], out["bank_values"], mask, w.selector.wq,
                          w.selector.wk, 128, uniforms=uniforms)
    assert np.array_equal(sel["index"], r["blocked_index"]) and bits_equal(sel["p"], r["blocked_p"])
    assert bits_equal(sel["gather"], r["blocked_gather"])


def test_learn_batch_matches_reference():
    """learnFromExperience on eight frames shaped like the learn workload (16-256 records, four questions,
    a target bank row per question, a reward per frame): the oracle's learn leaves the same page."""
    from krystal_b200 import synth
    from oracle import learn_oracle as LO
    r = ref("learn_batch")
    wl = synth.WORKLOADS["learn_1024"]
    cfg = synth.workload_config(wl)
    w0 = synth.workload_weights(cfg, wl.vocab)
    b = synth.make_batch(wl, seed=1, frames=8)
    targets, rewards = synth.make_learn_inputs(b, seed=3)
    offs = b.offsets()
    exps = []
    for f in range(b.frames):
        g = b.frame(f)
        q0, q1 = int(offs["q_off"][f]), int(offs["q_off"][f + 1])
        bank = np.flatnonzero(g.band_ids != 5)
        exps.append(dict(frame=g, chosen=[int(bank[t]) for t in targets[q0:q1]], reward=float(rewards[f]),
                         mask=np.zeros((q1 - q0) * bank.size, np.float32)))
    page, rep = LO.learn_from_experience(cfg, w0.page, exps)
    for k, v in _page_parts(page).items():
        assert v == str(r[f"sha_{k}"]), k
    assert G.sha(page) == str(r["sha"])
    for k, js in (("frames_seen", "framesSeen"), ("mean_advantage", "meanAdvantage"),
                  ("mean_value_loss", "meanValueLoss"), ("reinforced", "reinforced"), ("discouraged", "discouraged"),
                  ("mean_entropy", "meanEntropy"), ("mean_confidence", "meanConfidence"),
                  ("update_applied", "updateApplied")):
        assert float(rep[k]) == float(r[js]), k
