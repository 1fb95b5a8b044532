"""Model geometry, weight page layout and seeded initialisation.

Mirrors packages/krystal/src/forward/model.ts of the reference:
``BrainForwardConfig`` (model.ts:27-53), ``BRAIN_FORWARD_CONFIG`` (:55-80),
``embeddingTableBases`` (:102-124), ``createBrainForwardWeights`` (:233-265)
and ``validateBrainForwardWeights`` (:271-315).

The weights live in ONE contiguous float32 page laid out in generation order
(embeddings, enc blocks, pool, mixer blocks, selector, decision head, value
head); ``BrainForwardWeights`` exposes named views into it, the way the
reference session hands separate ``Float32Array`` s to a backend. One page
means one host→device copy on a full sync.

Unlike the reference, whose ``EMBEDDING_TABLES`` row counts are frozen at
module load from the default profile (model.ts:92-99), the six table sizes
come from the config, so a 16384-row token table is expressible. With the
default config the layout is identical to the reference's.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace

import numpy as np

# ABI constants (packages/schema/src/krystal-engine-schema.ts)
SEMANTIC_EMBEDDING_ROWS = 0x1000  # :45
REF_EMBEDDING_ROWS = 0x100  # :43
RECORD_WIDTH = 8  # BRAIN_LIMITS.recordWidth (:97)
FRAME_BANDS = 8  # BRAIN_LIMITS.frameBands
MAX_RECORD_SCHEMAS = 0x100
STREAM_RECORD = 0  # model.ts:268
STREAM_QUERY = 1  # model.ts:269


@dataclass(frozen=True)
class BrainForwardConfig:
    """BrainForwardConfig (model.ts:27-53) with the default profile's values."""

    hidden_size: int = 128
    head_count: int = 4
    head_dim: int = 32
    ffn_size: int = 384
    encoder_blocks: int = 2
    mixer_blocks: int = 2
    token_space: int = SEMANTIC_EMBEDDING_ROWS + REF_EMBEDDING_ROWS
    field_space: int = SEMANTIC_EMBEDDING_ROWS + REF_EMBEDDING_ROWS
    schema_space: int = MAX_RECORD_SCHEMAS
    band_space: int = FRAME_BANDS
    stream_space: int = 2
    pos_space: int = RECORD_WIDTH
    route_kind_count: int = 4
    # token id -> embedding row (the session supplies it; empty by default,
    # deliberately unusable, as in model.ts:75-79)
    token_rows: np.ndarray = field(default_factory=lambda: np.zeros(0, dtype=np.uint32), compare=False)

    def with_token_rows(self, token_rows) -> "BrainForwardConfig":
        return replace(self, token_rows=np.ascontiguousarray(token_rows, dtype=np.uint32))

    def table_rows(self) -> tuple[int, ...]:
        return (self.token_space, self.field_space, self.schema_space, self.band_space, self.stream_space,
                self.pos_space)


BRAIN_FORWARD_CONFIG = BrainForwardConfig()


@dataclass(frozen=True)
class EmbeddingBases:
    token: int
    field: int
    schema: int
    band: int
    stream: int
    pos: int


def embedding_table_bases(config: BrainForwardConfig) -> EmbeddingBases:
    """Word offset of each table in the embeddings page (model.ts:102-124)."""
    bases = []
    cursor = 0
    for rows in config.table_rows():
        bases.append(cursor)
        cursor += rows * config.hidden_size
    return EmbeddingBases(*bases)


def embeddings_page_elements(config: BrainForwardConfig) -> int:
    return sum(config.table_rows()) * config.hidden_size


@dataclass(frozen=True)
class WeightLayout:
    """Element offsets of every array in the flat weight page."""

    embeddings: int
    enc: int
    pool: int
    mixer: int
    selector_wq: int
    selector_wk: int
    decision_head: int
    value_head: int
    total: int
    block: int  # floats per encoder/mixer block: wq, wk, wv [H,H], w1 [F,H], w2 [H,F]


def weight_layout(config: BrainForwardConfig) -> WeightLayout:
    h, f = config.hidden_size, config.ffn_size
    block = 3 * h * h + 2 * f * h
    cursor = embeddings_page_elements(config)
    enc = cursor
    cursor += block * config.encoder_blocks
    pool = cursor
    cursor += 2 * h
    mixer = cursor
    cursor += block * config.mixer_blocks
    swq = cursor
    cursor += h * h
    swk = cursor
    cursor += h * h
    dec = cursor
    cursor += config.route_kind_count * 3 * h
    val = cursor
    cursor += 3 * h
    return WeightLayout(0, enc, pool, mixer, swq, swk, dec, val, cursor, block)


@dataclass
class BlockWeights:
    wq: np.ndarray
    wk: np.ndarray
    wv: np.ndarray
    w1: np.ndarray
    w2: np.ndarray


@dataclass
class SelectorWeights:
    wq: np.ndarray
    wk: np.ndarray


class BrainForwardWeights:
    """Named views into one flat float32 page (BrainForwardWeights, model.ts:145-183).

    Writing through a view writes the page, so the session's in-place
    updates are seen by whoever holds the page.
    """

    def __init__(self, config: BrainForwardConfig, page: np.ndarray):
        lay = weight_layout(config)
        if page.dtype != np.float32 or page.ndim != 1 or page.size != lay.total:
            raise ValueError(f"BrainForwardWeights: page must be float32[{lay.total}]")
        self.config = config
        self.page = page
        self.layout = lay
        h, f = config.hidden_size, config.ffn_size

        def blk(base: int) -> BlockWeights:
            o = base
            wq = page[o:o + h * h]; o += h * h
            wk = page[o:o + h * h]; o += h * h
            wv = page[o:o + h * h]; o += h * h
            w1 = page[o:o + f * h]; o += f * h
            w2 = page[o:o + h * f]
            return BlockWeights(wq, wk, wv, w1, w2)

        self.embeddings = page[lay.embeddings:lay.enc]
        self.enc = [blk(lay.enc + b * lay.block) for b in range(config.encoder_blocks)]
        self.pool = page[lay.pool:lay.pool + 2 * h]
        self.mixer = [blk(lay.mixer + b * lay.block) for b in range(config.mixer_blocks)]
        self.selector = SelectorWeights(page[lay.selector_wq:lay.selector_wq + h * h],
                                        page[lay.selector_wk:lay.selector_wk + h * h])
        self.decision_head_wh = page[lay.decision_head:lay.value_head]
        self.value_head_wv = page[lay.value_head:lay.total]


def mulberry32_draws(seed: int, start: int, count: int) -> np.ndarray:
    """Draws start..start+count-1 of mulberry32(seed) (model.ts:186-195), as f64.

    The generator's state after k calls is seed + k·0x6d2b79f5 (mod 2^32), so
    every draw is a pure function of its position and the stream vectorises.
    """
    k = np.arange(start + 1, start + count + 1, dtype=np.uint64)
    a = ((np.uint64(seed & 0xFFFFFFFF) + k * np.uint64(0x6D2B79F5)) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    with np.errstate(over="ignore"):
        t = (a ^ (a >> np.uint32(15))) * (np.uint32(1) | a)
        t = (t + (t ^ (t >> np.uint32(7))) * (np.uint32(61) | t)) ^ t
        out = (t ^ (t >> np.uint32(14))).astype(np.float64) / 4294967296.0
    return out


def _xavier(out: int, inp: int, draws: np.ndarray) -> np.ndarray:
    limit = np.sqrt(6.0 / (out + inp))
    return ((draws * 2 - 1) * limit).astype(np.float32)


def _normal(n: int, draws: np.ndarray, std: float) -> np.ndarray:
    # Box–Muller over consecutive (u1, u2) pairs (model.ts:204-215)
    u1 = np.maximum(draws[0::2], 1e-12)
    u2 = draws[1::2]
    r = np.sqrt(-2 * np.log(u1))
    ang = 2 * np.pi * u2
    vals = np.empty(2 * u1.size, dtype=np.float64)
    vals[0::2] = r * np.cos(ang) * std
    vals[1::2] = r * np.sin(ang) * std
    return vals[:n].astype(np.float32)


def create_brain_forward_weights(config: BrainForwardConfig = BRAIN_FORWARD_CONFIG,
                                 seed: int = 1337) -> BrainForwardWeights:
    """createBrainForwardWeights (model.ts:233-265): one mulberry32 stream."""
    lay = weight_layout(config)
    h, f = config.hidden_size, config.ffn_size
    page = np.empty(lay.total, dtype=np.float32)
    cursor = 0  # position in the page
    draw = 0  # position in the PRNG stream

    def take(n: int) -> np.ndarray:
        nonlocal draw
        d = mulberry32_draws(seed, draw, n)
        draw += n
        return d

    for rows in config.table_rows():
        n = rows * h
        page[cursor:cursor + n] = _normal(n, take(n + (n & 1)), 0.02)
        cursor += n

    def block(base: int) -> None:
        o = base
        for out, inp in ((h, h), (h, h), (h, h), (f, h), (h, f)):
            page[o:o + out * inp] = _xavier(out, inp, take(out * inp))
            o += out * inp

    for b in range(config.encoder_blocks):
        block(lay.enc + b * lay.block)
    page[lay.pool:lay.pool + 2 * h] = _normal(2 * h, take(2 * h), 0.02)
    for b in range(config.mixer_blocks):
        block(lay.mixer + b * lay.block)
    page[lay.selector_wq:lay.selector_wq + h * h] = _xavier(h, h, take(h * h))
    page[lay.selector_wk:lay.selector_wk + h * h] = _xavier(h, h, take(h * h))
    page[lay.decision_head:lay.value_head] = _xavier(config.route_kind_count, 3 * h,
                                                     take(config.route_kind_count * 3 * h))
    page[lay.value_head:lay.total] = _xavier(1, 3 * h, take(3 * h))
    return BrainForwardWeights(config, page)


def validate_brain_forward_weights(config: BrainForwardConfig, weights: BrainForwardWeights) -> None:
    """validateBrainForwardWeights (model.ts:271-315), on the page form."""
    lay = weight_layout(config)
    if weights.page.size != lay.total:
        raise ValueError("BrainForwardWeights: weight page size")
    if weights.embeddings.size != embeddings_page_elements(config):
        raise ValueError("BrainForwardWeights: embeddings page size")
    if len(weights.enc) != config.encoder_blocks:
        raise ValueError("BrainForwardWeights: encoder block count")
    if len(weights.mixer) != config.mixer_blocks:
        raise ValueError("BrainForwardWeights: mixer block count")
