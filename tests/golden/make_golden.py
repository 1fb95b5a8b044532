"""Generates the golden fixtures in this directory from the C++ oracle.

    python tests/golden/make_golden.py

The reference has no stored golden outputs (its parity tests compute the CPU
oracle live), so these fixtures are the oracle's outputs on seeded inputs:
they pin the oracle against regression and give the GPU tests a fixed
target. make_reference_golden.py runs the reference's own TypeScript on the
same inputs, and tests/test_reference_golden.py requires the two to agree
bit for bit. Weights are rebuilt from their seeds at
test time; each fixture stores a checksum of the weight page it was made with.
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from krystal_b200 import synth  # noqa: E402
from krystal_b200.frame import pack_host_frame  # noqa: E402
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights  # noqa: E402
from oracle import oracle as O  # noqa: E402

TEST_RECORDS = [
    dict(schemaId=1, band=3, tokens=[10, 11, 12]),  # an apple
    dict(schemaId=1, band=3, tokens=[10, 13]),  # a stone
    dict(schemaId=2, band=2, tokens=[20, 21]),  # a comfort
    dict(schemaId=9, query=True, tokens=[30]),  # what next?
]


def page_digest(page: np.ndarray) -> str:
    return hashlib.sha256(page.tobytes()).hexdigest()


def test_records_fixture():
    """TEST_RECORDS with TEST_TOKEN_ROWS = id % 64 and weight seed 7
    (packages/webgpu/test/frame.ts:16-33, krystal-composed.test.ts:43)."""
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    w = create_brain_forward_weights(cfg, 7)
    frame = pack_host_frame(TEST_RECORDS)
    out = O.forward(cfg, w.page, frame.gpu)
    grammar = np.zeros(3, dtype=np.float32)
    grammar[2:] = -1e30  # krystal-composed.test.ts:31-36: only the first two records
    sel = O.selector(out["query_output"], out["bank_keys"], out["bank_values"], grammar, w.selector.wq,
                     w.selector.wk, 128)
    sel_open = O.selector(out["query_output"], out["bank_keys"], out["bank_values"], None, w.selector.wq,
                          w.selector.wk, 128)
    np.savez_compressed(
        HERE / "test_records.npz", token_ids=frame.gpu.token_ids, field_roles=frame.gpu.field_roles,
        schema_ids=frame.gpu.schema_ids, band_ids=frame.gpu.band_ids,
        active_record_indices=frame.gpu.active_record_indices, weights_sha=page_digest(w.page),
        field_states=out["field_states"], bank_keys=out["bank_keys"], bank_values=out["bank_values"],
        query_output=out["query_output"], grammar=grammar, p=sel["p"], index=sel["index"], gather=sel["gather"],
        p_open=sel_open["p"], index_open=sel_open["index"], gather_open=sel_open["gather"])


def batch_fixture(name: str, workload: str, frames: int, seed: int, rule: bool, uniforms: bool = False):
    wl = synth.WORKLOADS[workload]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    batch = synth.make_batch(wl, seed=seed, frames=frames)
    r = synth.make_rule(batch, seed=seed + 1) if rule else None
    nq = int((batch.band_ids == 5).sum())
    u = np.random.default_rng(seed + 2).random(nq) if uniforms else None
    res = O.forward_batch(cfg, w.page, batch, rule=r, uniforms=u, want_query_output=True)
    extra = {}
    if r is not None:
        extra.update(schema_allow=r[0], band_allow=r[1])
    if u is not None:
        extra.update(uniforms=u)
    np.savez_compressed(
        HERE / f"{name}.npz", workload=workload, rec_off=batch.rec_off, token_ids=batch.token_ids,
        field_roles=batch.field_roles, schema_ids=batch.schema_ids, band_ids=batch.band_ids,
        weights_sha=page_digest(w.page), p=res["p"], index=res["index"], p_off=res["p_off"], q_off=res["q_off"],
        query_output=res["query_output"], **extra)


def main():
    test_records_fixture()
    batch_fixture("single_frame_64", "single_frame_64", 1, seed=1, rule=False)
    batch_fixture("ragged_16_open", "ragged_4096", 16, seed=21, rule=False)
    batch_fixture("ragged_16_rule", "ragged_4096", 16, seed=31, rule=True)
    batch_fixture("ragged_12_sample", "ragged_4096", 12, seed=41, rule=True, uniforms=True)
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
