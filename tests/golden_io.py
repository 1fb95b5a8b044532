"""Loads the golden fixtures and rebuilds the config and weights they were made with."""
import hashlib
from pathlib import Path

import numpy as np

from krystal_b200 import synth
from krystal_b200.frame import BrainFrameGpu, FrameBatch
from krystal_b200.model import BRAIN_FORWARD_CONFIG, create_brain_forward_weights

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def sha(page: np.ndarray) -> str:
    return hashlib.sha256(page.tobytes()).hexdigest()


def test_records():
    g = load("test_records")
    cfg = BRAIN_FORWARD_CONFIG.with_token_rows(np.arange(4096, dtype=np.uint32) % 64)
    w = create_brain_forward_weights(cfg, 7)
    frame = BrainFrameGpu(g["token_ids"], g["field_roles"], g["schema_ids"], g["band_ids"],
                          g["active_record_indices"])
    return g, cfg, w, frame


def batch(name: str):
    g = load(name)
    wl = synth.WORKLOADS[str(g["workload"])]
    cfg = synth.workload_config(wl)
    w = synth.workload_weights(cfg, wl.vocab)
    b = FrameBatch(g["rec_off"], g["token_ids"], g["field_roles"], g["schema_ids"], g["band_ids"])
    rule = (g["schema_allow"], g["band_allow"]) if "schema_allow" in g else None
    uniforms = g.get("uniforms")
    return g, cfg, w, b, rule, uniforms


BATCHES = ["single_frame_64", "ragged_16_open", "ragged_16_rule", "ragged_12_sample"]
