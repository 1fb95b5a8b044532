"""Runs the reference's own TypeScript CPU path on the inputs of the golden
fixtures in this directory and stores its outputs as reference_<name>.npz.

    python tests/golden/make_reference_golden.py [reference root] [--only step,step,...]

The reference (3ksoft/krystal) is TypeScript and this image has no
JavaScript runtime, so tsrun.py (beside this file) executes the reference's
source files themselves under JavaScript's number semantics. What runs is
the reference's code, unmodified, read from the reference tree:

  packages/krystal/src/forward/model.ts     createBrainForwardWeights (mulberry32, Xavier, Box-Muller)
  packages/krystal/src/host/frame.ts        packHostFrame
  packages/krystal/src/forward/masks.ts     compileActiveFrame, recordRanges, compileRecordMask
  packages/krystal/src/forward/oracle.ts    brainForwardOracle, selectorOracle, softmaxRow
  packages/krystal/src/forward/sampling.ts  sampleRow (through selectorOracle's sampler)
  packages/krystal/src/host/learn.ts        selectionMask, learnFromExperience
  packages/krystal/src/host/gradients.ts    cpuGradients -> forward/backward.ts brainBackwardOracle
  packages/krystal/src/host/teach.ts        teachFromDemonstration
  packages/webgpu/test/frame.ts             TEST_RECORDS, TEST_CONFIG, testFrame (the composed test's frame)

and one long-bank frame (4096 bank records, 64 questions) is made here.

The inputs are the ones the other fixtures here and the learn/teach tests
are made from (the frames and rules they store, the weights rebuilt from
their seeds); only data crosses over: records as HostRecord objects, the
token-table rows of the synthetic workloads (N(0, 1/sqrt(128)), a seeded
numpy draw), the rule as the `allows(q, slot)` closure selectionMask takes,
and the sampler's uniforms. tests/test_reference_golden.py compares the C++
oracle with these fixtures bit for bit. Only this script reads the
reference tree; the fixtures it writes are what the tests use.
"""
from __future__ import annotations

import hashlib
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

import tsrun  # noqa: E402
from tsrun import Float32Array, Uint32Array, _JSArr, _js_obj  # noqa: E402

from krystal_b200 import synth  # noqa: E402
from krystal_b200.model import BRAIN_FORWARD_CONFIG, weight_layout  # noqa: E402

QUERY_BAND = 5
H = 128


def f32(a) -> np.ndarray:
    return np.frombuffer(a, dtype=np.float32).copy() if len(a) else np.zeros(0, np.float32)


def u32(a) -> np.ndarray:
    return np.frombuffer(a, dtype=np.uint32).copy() if len(a) else np.zeros(0, np.uint32)


def digest(page: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(page, dtype=np.float32).tobytes()).hexdigest()


def page_parts(page: np.ndarray) -> dict:
    """Digests of the parts learn and teach move."""
    L = weight_layout(BRAIN_FORWARD_CONFIG)
    spans = {"embeddings": (0, L.enc), "selector_wq": (L.selector_wq, L.selector_wq + H * H),
             "selector_wk": (L.selector_wk, L.selector_wk + H * H),
             "value_head": (L.value_head, L.value_head + 3 * H), "pool": (L.pool, L.pool + 2 * H)}
    return {f"sha_{k}": digest(page[a:b]) for k, (a, b) in spans.items()}


class Reference:
    def __init__(self, ref_root: Path):
        run = tsrun.Runner()
        src = ref_root / "packages"
        self.model = run.load(src / "krystal/src/forward/model.ts")
        self.oracle = run.load(src / "krystal/src/forward/oracle.ts")
        self.masks = run.load(src / "krystal/src/forward/masks.ts")
        self.frame = run.load(src / "krystal/src/host/frame.ts")
        self.learn = run.load(src / "krystal/src/host/learn.ts")
        self.gradients = run.load(src / "krystal/src/host/gradients.ts")
        self.teach = run.load(src / "krystal/src/host/teach.ts")
        self.test_frame = run.load(src / "webgpu/test/frame.ts")

    def config(self, token_rows: np.ndarray):
        return _js_obj([(tsrun._Spread, self.model["BRAIN_FORWARD_CONFIG"]),
                        ("tokenRows", Uint32Array(token_rows.tolist()))])

    def weights(self, config, seed: int):
        return self.model["createBrainForwardWeights"](config, seed)

    def workload_weights(self, config, vocab: int):
        """createBrainForwardWeights(config, 1337) with the workload's token rows written in (input data)."""
        w = self.weights(config, 1337)
        base = self.model["embeddingTableBases"](config).token
        rows = np.random.default_rng(0x5EED).normal(0.0, 1.0 / np.sqrt(H), vocab * H).astype(np.float32)
        w.embeddings.set(Float32Array(rows.tolist()), base)
        return w

    @staticmethod
    def page(w) -> np.ndarray:
        """The weights in the flat page order of the C ABI (embeddings, encoder blocks, pool, mixer blocks,
        selector, decision head, value head)."""
        parts = [f32(w.embeddings)]
        for b in w.enc:
            parts += [f32(b.wq), f32(b.wk), f32(b.wv), f32(b.w1), f32(b.w2)]
        parts.append(f32(w.pool))
        for b in w.mixer:
            parts += [f32(b.wq), f32(b.wk), f32(b.wv), f32(b.w1), f32(b.w2)]
        parts += [f32(w.selector.wq), f32(w.selector.wk), f32(w.decisionHeadWh), f32(w.valueHeadWv)]
        return np.concatenate(parts)

    def pack(self, token_ids, schema_ids, band_ids):
        """One frame's records as HostRecord objects -> packHostFrame (frame.ts)."""
        recs = []
        tok = token_ids.reshape(-1, 8)
        for s in range(schema_ids.size):
            props = [("schemaId", int(schema_ids[s])), ("tokens", _JSArr([int(x) for x in tok[s] if x != 0]))]
            props.append(("query", True) if band_ids[s] == QUERY_BAND else ("band", int(band_ids[s])))
            recs.append(_js_obj(props))
        return self.frame["packHostFrame"](_JSArr(recs))

    def think(self, packed, weights, config, allows=None, uniforms=None, record_mask=None):
        """brainForwardOracle + selectionMask + selectorOracle, as the session's consider/choose runs them."""
        active = packed.active
        q, r = len(active.queryRecords), len(active.bankRecords)
        out = self.oracle["brainForwardOracle"](packed.gpu, active, weights, config, record_mask, Float32Array(q * r))
        mask = self.learn["selectionMask"](active, allows)
        sampler = None if uniforms is None else (lambda row, *_: float(uniforms[row]))
        sel = self.oracle["selectorOracle"](out.queryOutput, out.bankKeys, out.bankValues, mask, weights.selector,
                                            H, sampler)
        return out, sel


def rule_allows(packed, schema_allow, band_allow, q0):
    """The schema x band bitmask rule as the host closure selectionMask takes."""
    schema, band = packed.gpu.schemaIds, packed.gpu.bandIds

    def allows(q, slot, *_):
        s, b, i = int(schema[slot]), int(band[slot]), q0 + q
        return bool(s < 256 and b < 32 and (int(schema_allow[i * 8 + (s >> 5)]) >> (s & 31)) & 1
                    and (int(band_allow[i]) >> b) & 1)
    return allows


def load(name: str) -> dict:
    with np.load(HERE / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def weights(ref: Reference):
    """Digests of the reference's seeded weight pages (default geometry)."""
    cfg = ref.config(np.arange(4096, dtype=np.uint32) % 64)
    np.savez_compressed(HERE / "reference_weights.npz",
                        **{f"sha_{seed}": digest(ref.page(ref.weights(cfg, seed))) for seed in (7, 1337, 3)})


def test_records(ref: Reference):
    """The composed test's frame and weights (webgpu/test/frame.ts, krystal-composed.test.ts:40-60):
    forward, selection under the test's grammar and open, and cpuGradients for three requests."""
    tf = ref.test_frame["testFrame"]()
    cfg = ref.test_frame["TEST_CONFIG"]
    w = ref.weights(cfg, 7)
    active = tf.active
    q, r = len(active.queryRecords), len(active.bankRecords)
    out = ref.oracle["brainForwardOracle"](tf.frame, active, w, cfg, None, Float32Array(q * r))
    grammar = Float32Array(q * r)
    for i in range(q):
        for j in range(2, r):
            grammar[i * r + j] = -1e30
    sel = ref.oracle["selectorOracle"](out.queryOutput, out.bankKeys, out.bankValues, grammar, w.selector, H)
    sel_open = ref.oracle["selectorOracle"](out.queryOutput, out.bankKeys, out.bankValues, Float32Array(q * r),
                                            w.selector, H)
    packed = ref.frame["packHostFrame"](ref.test_frame["TEST_RECORDS"])
    grads = ref.gradients["cpuGradients"](w, cfg)
    requests = {
        "toward": _js_obj([("selection", grammar), ("targets", _JSArr([1])), ("valenceTarget", 0.5)]),
        "away": _js_obj([("selection", grammar), ("targets", _JSArr([0x80000000 | 1]))]),
        "critic": _js_obj([("selection", Float32Array(q * r)), ("valenceTarget", -0.25)]),
    }
    back = {}
    for name, req in requests.items():
        res = grads.backward(packed, req)
        back.update({f"{name}_policy": f32(res.policy), f"{name}_value_prediction": f32(res.valuePrediction),
                     f"{name}_value_loss": np.float64(res.valueLoss), f"{name}_d_selector_wq": f32(res.dSelectorWq),
                     f"{name}_d_selector_wk": f32(res.dSelectorWk), f"{name}_d_pool": f32(res.dPool),
                     f"{name}_d_field_states": f32(res.dFieldStates), f"{name}_d_value_wv": f32(res.dValueWv)})
    np.savez_compressed(
        HERE / "reference_test_records.npz", weights_sha=digest(ref.page(w)),
        token_ids=np.array(tf.frame.tokenIds, np.uint32), schema_ids=np.array(tf.frame.schemaIds, np.uint32),
        band_ids=np.array(tf.frame.bandIds, np.uint32),
        active_record_indices=np.array(tf.frame.activeRecordIndices, np.uint32),
        active_tokens=u32(active.activeTokens), bank_records=u32(active.bankRecords),
        query_records=u32(active.queryRecords), field_states=f32(out.fieldStates), bank_keys=f32(out.bankKeys),
        bank_values=f32(out.bankValues), query_keys=f32(out.queryKeys), query_values=f32(out.queryValues),
        query_output=f32(out.queryOutput), grammar=f32(grammar), p=f32(sel.p), index=u32(sel.index),
        gather=f32(sel.gather), p_open=f32(sel_open.p), index_open=u32(sel_open.index),
        gather_open=f32(sel_open.gather), **back)


def word_bias(ref: Reference):
    """The same-word bias (masks.ts compileRecordMask) on the single 64-record frame, two alphas."""
    g = load("single_frame_64")
    wl = synth.WORKLOADS["single_frame_64"]
    cfg = ref.config(np.arange(wl.vocab, dtype=np.uint32))
    w = ref.workload_weights(cfg, wl.vocab)
    packed = ref.pack(g["token_ids"], g["schema_ids"], g["band_ids"])
    rng = np.random.default_rng(7)
    words = rng.integers(0, 3, g["token_ids"].size).astype(np.uint32)
    words[rng.random(words.size) < 0.2] = 0xFFFFFFFF
    out = {"word_ids": words}
    for tag, alpha in (("pos", 1.5), ("neg", -3.0)):
        bias = _js_obj([("wordIds", Uint32Array(words.tolist())), ("alpha", alpha)])
        mask = ref.masks["compileRecordMask"](packed.active.activeTokens, bias).mask
        fwd, sel = ref.think(packed, w, cfg, record_mask=mask)
        out.update({f"{tag}_alpha": np.float32(alpha), f"{tag}_query_output": f32(fwd.queryOutput),
                    f"{tag}_p": f32(sel.p), f"{tag}_index": u32(sel.index)})
    np.savez_compressed(HERE / "reference_word_bias_64.npz", weights_sha=digest(ref.page(w)), **out)


def js_records(records):
    return _JSArr([_js_obj([(k, _JSArr(v) if k == "tokens" else v) for k, v in r.items()]) for r in records])


def js_options(d):
    return _js_obj([(k, js_options(v) if isinstance(v, dict) else v) for k, v in d.items()])


# name: (tests/learn_cases.experiences arguments, LearnOptions); the tests pass the same to the oracle
LEARN_CASES = {
    "default": (dict(n=6, seed=5, skip_reward=(2,), no_choice=(4,)), {}),
    "unfrozen": (dict(n=6, seed=9), {"unfreeze": {"pool": True, "tokens": True}, "learningRate": 0.1}),
    "rejected": (dict(n=5, seed=11), {"maxParameterAbs": 1e-3}),
}
# name: (tests/teach_cases.demonstrations arguments, TeachOptions)
TEACH_CASES = {
    "default": (dict(n=3, seed=7, forbid=(1,)), {}),
    "frozen": (dict(n=4, seed=13, forbid=(0, 2), nothing=(3,)), {"unfreezeTokens": False, "learningRate": 0.5}),
}
LEARN_WORLD_ROWS = np.arange(4096, dtype=np.uint32) % 97  # tests/learn_cases.world
LEARN_WORLD_SEED = 3


def learn(ref: Reference):
    """learnFromExperience (host/learn.ts:280-512), gradients from cpuGradients, on the learn tests' batches."""
    from tests.learn_cases import experiences
    out = {}
    for name, (kw, opts) in LEARN_CASES.items():
        cfg = ref.config(LEARN_WORLD_ROWS)
        w = ref.weights(cfg, LEARN_WORLD_SEED)
        exps = _JSArr([_js_obj([("records", js_records(ex.records)),
                                ("chosen", None if ex.chosen is None else _JSArr(ex.chosen)),
                                ("allows", ex.allows), ("reward", ex.reward)]) for ex in experiences(**kw)])
        rep = ref.learn["learnFromExperience"](exps, w, cfg, js_options(opts))
        page = ref.page(w)
        out[f"{name}_sha"] = digest(page)
        out.update({f"{name}_{k}": v for k, v in page_parts(page).items()})
        for k in ("framesSeen", "meanAdvantage", "meanValueLoss", "reinforced", "discouraged", "meanEntropy",
                  "meanConfidence", "updateApplied"):
            out[f"{name}_{k}"] = np.float64(getattr(rep, k))
        out[f"{name}_rejected"] = str(rep.rejected or "")
        for k in ("semanticEmbeddingMaxAbs", "selectorMaxAbs", "valueMaxAbs", "poolMaxAbs"):
            out[f"{name}_health_{k}"] = np.float64(getattr(rep.health, k))
    np.savez_compressed(HERE / "reference_learn.npz", **out)


def teach(ref: Reference):
    """teachFromDemonstration (host/teach.ts:126-272), one showing after another, on the teach tests' showings."""
    from tests.teach_cases import demonstrations
    out = {}
    for name, (kw, opts) in TEACH_CASES.items():
        cfg = ref.config(LEARN_WORLD_ROWS)
        w = ref.weights(cfg, LEARN_WORLD_SEED)
        demos = []
        for d in demonstrations(**kw):
            props = [("records", js_records(d.records)), ("gold", _JSArr(d.gold)), ("allows", d.allows)]
            if d.forbidden is not None:
                props.append(("forbidden", _JSArr(d.forbidden)))
            demos.append(_js_obj(props))
        rep = ref.teach["teachFromDemonstration"](_JSArr(demos), w, cfg, js_options(opts))
        page = ref.page(w)
        out[f"{name}_sha"] = digest(page)
        out.update({f"{name}_{k}": v for k, v in page_parts(page).items()})
        for k in ("framesSeen", "shown", "meanAgreement", "maxParameterAbs", "rejected", "clipped"):
            out[f"{name}_{k}"] = np.float64(getattr(rep, k))
    np.savez_compressed(HERE / "reference_teach.npz", **out)


def batch(ref: Reference, name: str):
    """Every frame of a batch fixture through packHostFrame, brainForwardOracle, selectionMask and selectorOracle."""
    g = load(name)
    wl = synth.WORKLOADS[str(g["workload"])]
    cfg = ref.config(np.arange(wl.vocab, dtype=np.uint32))
    if wl.vocab > cfg.tokenSpace:
        raise ValueError("a widened token table is not the reference's geometry")
    w = ref.workload_weights(cfg, wl.vocab)
    rec_off = g["rec_off"].astype(np.int64)
    rule = "schema_allow" in g
    uniforms = g.get("uniforms")
    ps, idx, qo, qs = [], [], [], 0
    for f in range(rec_off.size - 1):
        a, b = rec_off[f], rec_off[f + 1]
        packed = ref.pack(g["token_ids"][a * 8:b * 8], g["schema_ids"][a:b], g["band_ids"][a:b])
        assert np.array_equal(np.array(packed.gpu.tokenIds, np.uint32), g["token_ids"][a * 8:b * 8])
        nq = len(packed.active.queryRecords)
        allows = rule_allows(packed, g["schema_allow"], g["band_allow"], qs) if rule else None
        out, sel = ref.think(packed, w, cfg, allows=allows, uniforms=None if uniforms is None else uniforms[qs:qs + nq])
        ps.append(f32(sel.p))
        idx.append(u32(sel.index))
        qo.append(f32(out.queryOutput))
        qs += nq
    np.savez_compressed(HERE / f"reference_{name}.npz", weights_sha=digest(ref.page(w)), p=np.concatenate(ps),
                        index=np.concatenate(idx), query_output=np.concatenate(qo))


# One long-bank frame inside the reference's geometry: a 4096-record bank and 64 questions, as in the
# long-bank workload, with token ids over 4096 rows (the reference's token table holds 4352).
LONG_BANK_REF = synth.Workload("long_bank_ref", 1, (4160, 4160), (64, 64), 4096, 64, bank=4096)


def long_bank(ref: Reference):
    """The pointer softmax over a 4096-record bank: one frame, selected open and under a schema x band rule."""
    wl = LONG_BANK_REF
    b = synth.make_batch(wl, seed=51, frames=1)
    schema_allow, band_allow = synth.make_rule(b, seed=52)
    cfg = ref.config(np.arange(wl.vocab, dtype=np.uint32))
    w = ref.workload_weights(cfg, wl.vocab)
    packed = ref.pack(b.token_ids, b.schema_ids, b.band_ids)
    active = packed.active
    q, r = len(active.queryRecords), len(active.bankRecords)
    out = ref.oracle["brainForwardOracle"](packed.gpu, active, w, cfg, None, Float32Array(q * r))
    res = {}
    for tag, allows in (("open", None), ("rule", rule_allows(packed, schema_allow, band_allow, 0))):
        mask = ref.learn["selectionMask"](active, allows)
        sel = ref.oracle["selectorOracle"](out.queryOutput, out.bankKeys, out.bankValues, mask, w.selector, H)
        res.update({f"p_{tag}": f32(sel.p), f"index_{tag}": u32(sel.index)})
    np.savez_compressed(HERE / "reference_long_bank_frame.npz", weights_sha=digest(ref.page(w)), vocab=wl.vocab,
                        rec_off=b.rec_off, token_ids=b.token_ids, field_roles=b.field_roles, schema_ids=b.schema_ids,
                        band_ids=b.band_ids, schema_allow=schema_allow, band_allow=band_allow,
                        query_output=f32(out.queryOutput), **res)


def edges(ref: Reference):
    """tests/edge_cases.py: frames without a bank or a question, empty records and holes, 1-token and full
    records; the rule that admits nothing (reopened row); a blocked question with sampling."""
    from tests import edge_cases as E
    cfg = ref.config(E.token_rows())
    w = ref.weights(cfg, E.WEIGHT_SEED)
    out = {"weights_sha": digest(ref.page(w))}
    ps, idx, qo = [], [], []
    for recs in E.edge_frames():
        packed = ref.frame["packHostFrame"](js_records(recs))
        fwd, sel = ref.think(packed, w, cfg)
        ps.append(f32(sel.p))
        idx.append(u32(sel.index))
        qo.append(f32(fwd.queryOutput))
    out.update(p=np.concatenate(ps), index=np.concatenate(idx), query_output=np.concatenate(qo))
    recs, schema_allow, band_allow = E.reopen_frame()
    packed = ref.frame["packHostFrame"](js_records(recs))
    _, sel = ref.think(packed, w, cfg, allows=rule_allows(packed, schema_allow, band_allow, 0))
    out.update(reopen_p=f32(sel.p), reopen_index=u32(sel.index))
    recs, mask, uniforms = E.blocked_frame()
    packed = ref.frame["packHostFrame"](js_records(recs))
    active = packed.active
    fwd = ref.oracle["brainForwardOracle"](packed.gpu, active, w, cfg, None,
                                           Float32Array(len(active.queryRecords) * len(active.bankRecords)))
    sel = ref.oracle["selectorOracle"](fwd.queryOutput, fwd.bankKeys, fwd.bankValues, Float32Array(mask.tolist()),
                                       w.selector, H, lambda row, *_: float(uniforms[row]))
    out.update(blocked_p=f32(sel.p), blocked_index=u32(sel.index), blocked_gather=f32(sel.gather),
               blocked_query_output=f32(fwd.queryOutput))
    np.savez_compressed(HERE / "reference_edges.npz", **out)


LEARN_BATCH_FRAMES = 8


def learn_batch(ref: Reference):
    """learnFromExperience on frames shaped like the learn workload (16-256 records, four questions, a target
    bank row per question, a reward per frame; make_batch seed 1, make_learn_inputs seed 3), open grammar."""
    wl = synth.WORKLOADS["learn_1024"]
    b = synth.make_batch(wl, seed=1, frames=LEARN_BATCH_FRAMES)
    targets, rewards = synth.make_learn_inputs(b, seed=3)
    offs = b.offsets()
    cfg = ref.config(np.arange(wl.vocab, dtype=np.uint32))
    w = ref.workload_weights(cfg, wl.vocab)
    exps = []
    for f in range(b.frames):
        g = b.frame(f)
        q0, q1 = int(offs["q_off"][f]), int(offs["q_off"][f + 1])
        bank = np.flatnonzero(g.band_ids != QUERY_BAND)
        recs = _JSArr(js_records_of(g))
        exps.append(_js_obj([("records", recs), ("chosen", _JSArr([int(bank[t]) for t in targets[q0:q1]])),
                             ("reward", float(rewards[f]))]))
    rep = ref.learn["learnFromExperience"](_JSArr(exps), w, cfg, _js_obj([]))
    page = ref.page(w)
    out = {"sha": digest(page), **page_parts(page)}
    for k in ("framesSeen", "meanAdvantage", "meanValueLoss", "reinforced", "discouraged", "meanEntropy",
              "meanConfidence", "updateApplied"):
        out[k] = np.float64(getattr(rep, k))
    np.savez_compressed(HERE / "reference_learn_batch.npz", **out)


def js_records_of(g):
    """A packed frame's records back as HostRecord objects (every record active, in order)."""
    tok = g.token_ids.reshape(-1, 8)
    for s in range(g.schema_ids.size):
        props = [("schemaId", int(g.schema_ids[s])), ("tokens", _JSArr([int(x) for x in tok[s] if x != 0]))]
        props.append(("query", True) if g.band_ids[s] == QUERY_BAND else ("band", int(g.band_ids[s])))
        yield _js_obj(props)


STEPS = ("weights", "test_records", "word_bias", "learn", "teach", "single_frame_64", "ragged_16_open",
         "ragged_16_rule", "ragged_12_sample", "long_bank", "edges", "learn_batch")


def main():
    args = sys.argv[1:]
    only = set(STEPS)
    if "--only" in args:
        i = args.index("--only")
        only = set(args[i + 1].split(","))
        del args[i:i + 2]
    ref = Reference(Path(args[0]) if args else Path("/root/reference"))
    for step in STEPS:
        if step not in only:
            continue
        t0 = time.time()
        if step.startswith(("single", "ragged")):
            batch(ref, step)
        else:
            globals()[step](ref)
        print(f"{step}: {time.time() - t0:.0f} s", flush=True)


if __name__ == "__main__":
    main()
