"""The split-KV chunk policy of the decode launches (engine.cu att_chunk), checked on the CPU.

The attention partial buffer holds kMaxChunks = 32 chunks per (row, kv head); a launch's chunk length
must keep every row's chunk count within it for any context up to the model's capacity, be a multiple of
the 16-position attention tile, and, while the context allows, give about one item per CTA.
"""

from __future__ import annotations

import pytest

MAX_CHUNKS, TILE, CTAS = 32, 16, 148


def att_chunk(rows: int, max_ctx: int, units: int, limit: int = MAX_CHUNKS) -> int:
    """engine.cu att_chunk."""
    target = max(1, min(limit, CTAS // max(1, rows * units)))
    ch = max(-(-max_ctx // target), -(-max_ctx // MAX_CHUNKS))
    ch = -(-ch // TILE) * TILE
    return max(ch, TILE)


@pytest.mark.parametrize("rows", [1, 2, 4, 5, 8])
@pytest.mark.parametrize("units", [1, 2, 4, 8, 16, 32])
def test_chunks_fit_the_partial_buffer(rows: int, units: int) -> None:
    for ctx in list(range(1, 600)) + [1023, 1024, 4097, 8192, 8300, 32768, 131072]:
        ch = att_chunk(rows, ctx, units)
        assert ch % TILE == 0 and ch >= TILE
        assert -(-ctx // ch) <= MAX_CHUNKS, (rows, units, ctx, ch)
        for limit in (8, 16):  # the chunk-count knob
            assert -(-ctx // att_chunk(rows, ctx, units, limit)) <= MAX_CHUNKS


def test_batch1_gemma3_1b_items() -> None:
    # per-q-head items (4 units) at position 640: chunks of 32 positions, 4 x 21 = 84 items for 148 CTAs
    ch = att_chunk(1, 641, 4)
    assert ch == 32 and 4 * -(-641 // ch) == 84
