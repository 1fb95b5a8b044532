"""KRY1 checkpoints (packages/krystal/src/host/checkpoint.ts:17-116).

A brain written down: an 11-word header (magic "KRY1", version, the seven
geometry numbers, the tokenRows length, the weight element count), the
tokenRows the weights learned their meanings under, then every weight array
in createBrainForwardWeights order, all little-endian. Geometry and
vocabulary are checked on the way in, and a mismatch is refused by name
rather than coerced. The weight page of ``BrainForwardWeights`` is already in
that order, so encoding and decoding are one contiguous copy each; the CUDA
backend takes the same bytes straight into its device page
(``CudaBrainBackend.load_checkpoint``).
"""
from __future__ import annotations

import numpy as np

from .model import BrainForwardConfig, BrainForwardWeights

MAGIC = 0x4B525931  # "KRY1"
VERSION = 1
HEADER_WORDS = 11


def geometry_of(config: BrainForwardConfig) -> list[int]:
    """checkpoint.ts:34-42."""
    return [config.hidden_size, config.ffn_size, config.encoder_blocks, config.mixer_blocks, config.head_count,
            config.head_dim, config.route_kind_count]


def encode_checkpoint(weights: BrainForwardWeights, config: BrainForwardConfig, token_rows) -> bytes:
    """encodeCheckpoint (checkpoint.ts:51-69)."""
    rows = np.ascontiguousarray(token_rows, dtype="<u4")
    page = np.ascontiguousarray(weights.page, dtype="<f4")
    header = np.array([MAGIC, VERSION, *geometry_of(config), rows.size, page.size], dtype="<u4")
    return header.tobytes() + rows.tobytes() + page.tobytes()


def decode_checkpoint(data, weights: BrainForwardWeights, config: BrainForwardConfig, token_rows) -> str | None:
    """decodeCheckpoint (checkpoint.ts:78-116): into the weights in place;
    None when taken up, else the refusal. `data` may start anywhere."""
    buf = memoryview(data).cast("B")
    if buf.nbytes < HEADER_WORDS * 4:
        return "truncated"
    header = np.frombuffer(buf[:HEADER_WORDS * 4], dtype="<u4")
    if header[0] != MAGIC:
        return "not a krystal checkpoint"
    if header[1] > VERSION:
        return "a later checkpoint format"
    if list(header[2:9]) != geometry_of(config):
        return "a different geometry"
    rows = np.ascontiguousarray(token_rows, dtype=np.uint32)
    count, elements = int(header[9]), int(header[10])
    if count != rows.size:
        return "a different vocabulary"
    if buf.nbytes < (HEADER_WORDS + count + elements) * 4:
        return "truncated"
    got = np.frombuffer(buf[HEADER_WORDS * 4:(HEADER_WORDS + count) * 4], dtype="<u4")
    if not np.array_equal(got, rows):
        return "a different vocabulary"
    if weights.page.size != elements:
        return "a different geometry"
    start = (HEADER_WORDS + count) * 4
    weights.page[:] = np.frombuffer(buf[start:start + elements * 4], dtype="<f4")
    return None
