"""KRY1 checkpoints on the host (host/checkpoint.ts), after the reference's
own cases (host/checkpoint.test.ts:26-76): a round trip is exact, another
vocabulary or geometry is refused and leaves the weights untouched, non-
checkpoints and short buffers say so, and an unaligned buffer still loads."""
from dataclasses import replace

import numpy as np

from krystal_b200.checkpoint import MAGIC, decode_checkpoint, encode_checkpoint
from krystal_b200.model import BRAIN_FORWARD_CONFIG, BrainForwardWeights, create_brain_forward_weights

SMALL = replace(BRAIN_FORWARD_CONFIG, hidden_size=32, head_count=1, head_dim=32, ffn_size=64, encoder_blocks=1,
                mixer_blocks=1)


def rows(count=4096, offset=0):
    return (np.arange(count, dtype=np.uint32) + offset) % 64


def test_header_layout():
    w = create_brain_forward_weights(SMALL, 7)
    b = encode_checkpoint(w, SMALL, rows())
    assert b[:4] == b"1YRK"  # 0x4b525931 little-endian
    h = np.frombuffer(b[:44], dtype="<u4")
    assert h[0] == MAGIC and h[1] == 1
    assert list(h[2:9]) == [32, 64, 1, 1, 1, 32, SMALL.route_kind_count]
    assert h[9] == 4096 and h[10] == w.page.size
    assert len(b) == 4 * (11 + 4096 + w.page.size)
    assert np.array_equal(np.frombuffer(b[44:44 + 4 * 4096], dtype="<u4"), rows())


def test_round_trip_is_exact():
    trained = create_brain_forward_weights(SMALL, 7)
    trained.page[::7] += np.float32(0.125)  # off its seed
    cold = create_brain_forward_weights(SMALL, 99)
    assert decode_checkpoint(encode_checkpoint(trained, SMALL, rows()), cold, SMALL, rows()) is None
    assert np.array_equal(cold.page, trained.page)


def test_another_vocabulary_is_refused_not_coerced():
    trained = create_brain_forward_weights(SMALL, 7)
    other = create_brain_forward_weights(SMALL, 8)
    untouched = other.page.copy()
    assert decode_checkpoint(encode_checkpoint(trained, SMALL, rows()), other, SMALL, rows(offset=1)) == \
        "a different vocabulary"
    assert decode_checkpoint(encode_checkpoint(trained, SMALL, rows()), other, SMALL, rows(4000)) == \
        "a different vocabulary"
    assert np.array_equal(other.page, untouched)


def test_another_geometry_is_refused():
    trained = create_brain_forward_weights(SMALL, 7)
    wide_cfg = replace(SMALL, hidden_size=64, head_dim=64)
    wider = create_brain_forward_weights(wide_cfg, 7)
    assert decode_checkpoint(encode_checkpoint(trained, SMALL, rows()), wider, wide_cfg, rows()) == \
        "a different geometry"
    # same seven numbers, different table sizes: the element count gives it away
    tables = replace(SMALL, token_space=SMALL.token_space + 1)
    t = create_brain_forward_weights(tables, 7)
    assert decode_checkpoint(encode_checkpoint(trained, SMALL, rows()), t, tables, rows()) == \
        "a different geometry"


def test_not_a_checkpoint_and_short_buffers():
    w = create_brain_forward_weights(SMALL, 7)
    assert decode_checkpoint(bytes(64), w, SMALL, rows()) == "not a krystal checkpoint"
    assert decode_checkpoint(bytes(3), w, SMALL, rows()) == "truncated"
    b = encode_checkpoint(w, SMALL, rows())
    assert decode_checkpoint(b[:-4], w, SMALL, rows()) == "truncated"
    later = bytearray(b)
    later[4:8] = np.array([2], dtype="<u4").tobytes()
    assert decode_checkpoint(bytes(later), w, SMALL, rows()) == "a later checkpoint format"


def test_an_unaligned_buffer_still_loads():
    trained = create_brain_forward_weights(SMALL, 7)
    b = encode_checkpoint(trained, SMALL, rows())
    shifted = bytearray(len(b) + 1)
    shifted[1:] = b
    cold = BrainForwardWeights(SMALL, create_brain_forward_weights(SMALL, 99).page.copy())
    assert decode_checkpoint(memoryview(shifted)[1:], cold, SMALL, rows()) is None
    assert np.array_equal(cold.page, trained.page)
