"""Seeded synthetic workloads with the shapes of the benchmark configurations.

There is no dataset on this path: frames are records of token ids. Each
workload draws its frames from a seeded generator with the distributions the
configuration names:

* tokens per record uniform 1..8, token ids uniform in [1, V) (0 is PAD);
* ``token_rows`` is the identity over V ids, so the token table has V rows;
* field roles 0 (the session default, which maps to row 0);
* question records carry band 5 (the query band); bank records draw their
  band uniformly from {0,1,2,3,4,6,7} — band 5 would make them questions;
* question slots are a random subset of the frame's positions;
* weights = createBrainForwardWeights(config, 1337), then token-table rows
  0..V-1 overwritten with N(0, 1/sqrt(H)) draws from a separate stream;
* optional selection rule: per question a random 256-bit schema mask and
  8-bit band mask (about half the bits set).
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np

from .frame import QUERY_BAND, FrameBatch
from .model import RECORD_WIDTH, BRAIN_FORWARD_CONFIG, BrainForwardConfig, BrainForwardWeights, \
    create_brain_forward_weights, embedding_table_bases

BANK_BANDS = np.array([0, 1, 2, 3, 4, 6, 7], dtype=np.uint32)


@dataclass(frozen=True)
class Workload:
    name: str
    frames: int
    records: tuple[int, int]  # uniform range of records per frame (inclusive); ignored when bank is fixed
    questions: tuple[int, int]  # uniform range of questions per frame (inclusive)
    vocab: int  # V
    schemas: int  # schema ids uniform in [0, schemas)
    bank: int | None = None  # fixed bank size (records = bank + questions)


WORKLOADS = {
    # one frame of 64 records (56 bank + 8 questions), V=1024, schema 0-15
    "single_frame_64": Workload("single_frame_64", 1, (64, 64), (8, 8), 1024, 16, bank=56),
    # 4096 frames, records 16-256 with 1-16 questions, V=4096, schema 0-63
    "ragged_4096": Workload("ragged_4096", 4096, (16, 256), (1, 16), 4096, 64),
    # 1024 frames, 4096-record bank + 64 questions, V=16384
    "long_bank_1024": Workload("long_bank_1024", 1024, (4160, 4160), (64, 64), 16384, 64, bank=4096),
    # learn step: 1024 frames, records 16-256 with 4 questions each, V=4096, schema 0-63
    "learn_1024": Workload("learn_1024", 1024, (16, 256), (4, 4), 4096, 64),
    # interactive stream: 100k frames, records 8-512 with 1-32 questions, V=4096, schema 0-63
    "stream_100k": Workload("stream_100k", 100000, (8, 512), (1, 32), 4096, 64),
}


def poisson_arrivals(frames: int, rate_per_s: float, seed: int = 4) -> np.ndarray:
    """Arrival times (ms from 0) of a Poisson process at rate_per_s."""
    rng = np.random.default_rng(seed)
    return np.cumsum(rng.exponential(1e3 / rate_per_s, frames))


def workload_config(w: Workload, base: BrainForwardConfig = BRAIN_FORWARD_CONFIG) -> BrainForwardConfig:
    """Geometry for a workload: the default profile, with the token and field
    tables widened when V exceeds the reference's fixed 4352 rows."""
    cfg = base
    if w.vocab > cfg.token_space:
        cfg = replace(cfg, token_space=w.vocab, field_space=w.vocab)
    return cfg.with_token_rows(np.arange(w.vocab, dtype=np.uint32))


def workload_weights(config: BrainForwardConfig, vocab: int, seed: int = 1337,
                     token_seed: int = 0x5EED) -> BrainForwardWeights:
    w = create_brain_forward_weights(config, seed)
    h = config.hidden_size
    base = embedding_table_bases(config).token
    rng = np.random.default_rng(token_seed)
    w.embeddings[base:base + vocab * h] = rng.normal(0.0, 1.0 / np.sqrt(h), vocab * h).astype(np.float32)
    return w


def make_batch(w: Workload, seed: int = 1, frames: int | None = None) -> FrameBatch:
    """Draw a packed ragged batch for workload ``w``."""
    rng = np.random.default_rng(seed)
    F = w.frames if frames is None else frames
    q = rng.integers(w.questions[0], w.questions[1] + 1, F)
    if w.bank is not None:
        n = q + w.bank
    else:
        n = rng.integers(w.records[0], w.records[1] + 1, F)
        n = np.maximum(n, q + 1)
    rec_off = np.zeros(F + 1, dtype=np.uint64)
    np.cumsum(n, out=rec_off[1:])
    N = int(rec_off[-1])
    frame_of = np.repeat(np.arange(F), n)
    # question slots: the q_f records of smallest random key within each frame
    key = rng.random(N)
    order = np.lexsort((key, frame_of))
    rank = np.empty(N, dtype=np.int64)
    rank[order] = np.arange(N) - np.repeat(rec_off[:-1].astype(np.int64), n)
    is_q = rank < q[frame_of]
    band = np.where(is_q, QUERY_BAND, BANK_BANDS[rng.integers(0, BANK_BANDS.size, N)]).astype(np.uint32)
    schema = rng.integers(0, w.schemas, N).astype(np.uint32)
    ntok = rng.integers(1, RECORD_WIDTH + 1, N)
    ids = rng.integers(1, w.vocab, (N, RECORD_WIDTH)).astype(np.uint32)
    ids[np.arange(RECORD_WIDTH)[None, :] >= ntok[:, None]] = 0
    return FrameBatch(rec_off, ids.reshape(-1), np.zeros(N * RECORD_WIDTH, dtype=np.uint32), schema, band)


def make_learn_inputs(batch: FrameBatch, seed: int = 3) -> tuple[np.ndarray, np.ndarray]:
    """A learn batch's outcome: per question a target bank row drawn uniformly
    from its frame's bank (u32 [Q]), and per frame a reward ~ N(0, 1) (f64 [F])."""
    rng = np.random.default_rng(seed)
    offs = batch.offsets()
    q, r = offs["q"].astype(np.int64), offs["r"].astype(np.int64)
    bank_of_q = np.repeat(r, q)
    targets = np.floor(rng.random(bank_of_q.size) * bank_of_q).astype(np.uint32)
    return targets, rng.normal(size=batch.frames)


def make_rule(batch: FrameBatch, seed: int = 2, density: float = 0.5) -> tuple[np.ndarray, np.ndarray]:
    """Per-question selection rule: schema_allow u32[Q*8] (256 bits), band_allow u32[Q]."""
    rng = np.random.default_rng(seed)
    nq = int((batch.band_ids == QUERY_BAND).sum())
    bits = rng.random((nq, 256)) < density
    schema_allow = np.packbits(bits, axis=1, bitorder="little").view(np.uint32).reshape(nq, 8).copy()
    band_bits = rng.random((nq, 8)) < density
    band_allow = np.packbits(band_bits, axis=1, bitorder="little").astype(np.uint32).reshape(nq)
    return schema_allow.reshape(-1), band_allow
