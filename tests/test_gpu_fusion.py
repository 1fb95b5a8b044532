"""The fused encoder kernels against the unfused sequence, bit for bit.

k_tc_attn (q|k|v projection + record-local attention + residual) and
k_tc_ffn (W1 + ReLU + W2 + residual) claim the exact arithmetic of
k_tc_gemm<Store> + k_local_attn_fast and k_tc_gemm<Relu> + k_tc_gemm<Resid>.
A handle created with KC_NO_FUSION=1 runs the unfused sequence; both handles
see the same batches, and every output (p, index, the mixer's query output)
must agree exactly, on ragged batches and on layouts that put record and
tile edges where the fused kernel's record-aligned 128-row tiles are most
likely to go wrong: a single token, totals of 120, 127, 128, 129 and 240
rows, and frames of full 8-token records only.
"""
import os

import numpy as np
import pytest

from krystal_b200 import synth
from krystal_b200.backend import CudaBrainBackend
from krystal_b200.frame import FrameBatch

pytestmark = pytest.mark.gpu

WL = synth.WORKLOADS["ragged_4096"]
CFG = synth.workload_config(WL)
W = synth.workload_weights(CFG, WL.vocab)


def make_backend(fused: bool) -> CudaBrainBackend:
    old = os.environ.pop("KC_NO_FUSION", None)
    if not fused:
        os.environ["KC_NO_FUSION"] = "1"
    try:
        return CudaBrainBackend(CFG, W, 0)
    finally:
        os.environ.pop("KC_NO_FUSION", None)
        if old is not None:
            os.environ["KC_NO_FUSION"] = old


@pytest.fixture(scope="module")
def pair():
    fused, unfused = make_backend(True), make_backend(False)
    yield fused, unfused
    fused.destroy()
    unfused.destroy()


def layout_batch(frames: list[list[tuple[int, bool]]], seed: int) -> FrameBatch:
    """Frames as lists of (tokens in the record, is a question)."""
    rng = np.random.default_rng(seed)
    counts = [len(f) for f in frames]
    rec_off = np.zeros(len(frames) + 1, dtype=np.uint64)
    np.cumsum(counts, out=rec_off[1:])
    recs = [r for f in frames for r in f]
    n = len(recs)
    ids = rng.integers(1, WL.vocab, (n, 8)).astype(np.uint32)
    for i, (t, _) in enumerate(recs):
        ids[i, t:] = 0
    band = np.array([synth.QUERY_BAND if q else synth.BANK_BANDS[i % synth.BANK_BANDS.size]
                     for i, (_, q) in enumerate(recs)], dtype=np.uint32)
    schema = rng.integers(0, WL.schemas, n).astype(np.uint32)
    return FrameBatch(rec_off, ids.reshape(-1), np.zeros(n * 8, dtype=np.uint32), schema, band)


def frame_of_rows(rows: int, question_every: int = 5) -> list[tuple[int, bool]]:
    """Records of 8 tokens (the last one shorter) totalling `rows` tokens."""
    recs, i = [], 0
    while rows > 0:
        t = min(8, rows)
        recs.append((t, i % question_every == 1))
        rows -= t
        i += 1
    if not any(q for _, q in recs):
        recs.append((1, True))
    if all(q for _, q in recs):
        recs.append((3, False))
    return recs


def assert_same(a: dict, b: dict):
    assert a["total_t"] == b["total_t"] and a["total_r"] == b["total_r"]
    np.testing.assert_array_equal(a["index"], b["index"])
    assert np.array_equal(a["p"], b["p"]), "p differs between the fused and unfused encoders"
    assert np.array_equal(a["query_output"], b["query_output"])


def run(be: CudaBrainBackend, batch: FrameBatch, precision: str, **kw) -> dict:
    be.set_precision(precision)
    return be.forward_batch(batch, want_query_output=True, **kw)


@pytest.mark.parametrize("precision", ["fast", "certified"])
def test_ragged_batch_fused_equals_unfused(pair, precision):
    fused, unfused = pair
    batch = synth.make_batch(WL, seed=31, frames=384)
    assert_same(run(fused, batch, precision), run(unfused, batch, precision))


@pytest.mark.parametrize("rows", [1, 120, 127, 128, 129, 240])
def test_tile_edges_fused_equals_unfused(pair, rows):
    fused, unfused = pair
    frames = [frame_of_rows(rows)] if rows > 1 else [[(1, True), (1, False)]]
    batch = layout_batch(frames, seed=rows)
    assert_same(run(fused, batch, "fast"), run(unfused, batch, "fast"))


def test_full_records_many_frames_fused_equals_unfused(pair):
    fused, unfused = pair
    frames = [frame_of_rows(8 * (7 + (f % 23)), question_every=4) for f in range(97)]
    batch = layout_batch(frames, seed=5)
    assert_same(run(fused, batch, "fast"), run(unfused, batch, "fast"))


def test_word_bias_fused_equals_unfused(pair):
    fused, unfused = pair
    batch = synth.make_batch(WL, seed=41, frames=128)
    rng = np.random.default_rng(9)
    words = rng.integers(0, 3, batch.records * 8).astype(np.uint32)
    words[rng.random(words.size) < 0.2] = 0xFFFFFFFF
    kw = dict(word_ids=words, word_alpha=1.5)
    assert_same(run(fused, batch, "fast", **kw), run(unfused, batch, "fast", **kw))


def test_caller_output_buffers(pair):
    """forward_batch(out=...) fills caller-owned arrays (reused across calls)
    with exactly what fresh arrays receive; too small a p buffer is refused."""
    fused, _ = pair
    fused.set_precision("certified")
    batch = synth.make_batch(WL, seed=47, frames=64)
    want = fused.forward_batch(batch)
    offs = batch.offsets()
    out = {"p": np.full(int(offs["p_off"][-1]) + 7, -1.0, np.float32),
           "index": np.zeros(int(offs["q_off"][-1]), np.uint32),
           "p_off": np.zeros(batch.frames + 1, np.uint64), "q_off": np.zeros(batch.frames + 1, np.uint64)}
    for _ in range(2):
        got = fused.forward_batch(batch, out=out)
        assert np.array_equal(got["p"], want["p"]) and np.array_equal(got["index"], want["index"])
        assert np.array_equal(out["p_off"], want["p_off"]) and np.array_equal(out["q_off"], want["q_off"])
    small = dict(out, p=np.empty(int(offs["p_off"][-1]) - 1, np.float32))
    with pytest.raises(Exception):
        fused.forward_batch(batch, out=small)


def test_empty_records_at_tile_edges_fused_equals_unfused(pair):
    """Records without tokens (all PAD) at a batch's first row, where a tile
    starts (row 120) and at frame ends: the record-aligned tiles of the fused
    attention must step over them as the unfused sequence does (their pooled
    key and value are zero)."""
    fused, unfused = pair
    frames = [[(0, False)] + frame_of_rows(120) + [(0, True), (0, False)],
              frame_of_rows(7) + [(0, False)],
              [(0, True)] + frame_of_rows(129),
              frame_of_rows(240) + [(0, False)] * 3]
    batch = layout_batch(frames, seed=77)
    for precision in ("fast", "certified"):
        assert_same(run(fused, batch, precision), run(unfused, batch, precision))


def test_planes_products_equal_separate_products():
    """The bank-side projections as one planes product per input (bk through
    the selector's and every mixer block's Wk, bv through every block's Wv)
    give the bits of one product per matrix (a handle created with
    KC_NO_PLANES=1)."""
    old = os.environ.pop("KC_NO_PLANES", None)
    try:
        with_planes = CudaBrainBackend(CFG, W, 0)
        os.environ["KC_NO_PLANES"] = "1"
        without = CudaBrainBackend(CFG, W, 0)
    finally:
        os.environ.pop("KC_NO_PLANES", None)
        if old is not None:
            os.environ["KC_NO_PLANES"] = old
    try:
        batch = synth.make_batch(WL, seed=53, frames=256)
        for precision in ("fast", "certified"):
            assert_same(run(with_planes, batch, precision), run(without, batch, precision))
    finally:
        with_planes.destroy()
        without.destroy()
