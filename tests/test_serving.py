"""Continuous batching of concurrent streams (serving.BatchScheduler) on a fake
row-wise core: admission into free rows, per-row positions, the reference's
stopping rules (EOS, empty piece, max_tokens), cancellation, more streams than
rows, and the async API on top.  CPU only; the device path is in
test_gpu_serving.py."""

from __future__ import annotations

import asyncio

import numpy as np
import pytest

from mogemma_b200.serving import BatchScheduler


class RowCore:
    """Each row's next token is a fixed function of (its last token, its position):
    a stream's tokens do not depend on which row or batch it runs in."""

    def __init__(self, rows: int, vocab: int = 50) -> None:
        self.pos = [0] * rows
        self.vocab = vocab
        self.calls: list[tuple[str, object]] = []

    @staticmethod
    def next_token(tok: int, pos: int, vocab: int) -> int:
        return (tok * 7 + pos * 3 + 1) % vocab

    def set_row_pos(self, llm, row, pos):
        self.pos[row] = pos
        self.calls.append(("set_pos", (row, pos)))

    def row_positions(self, llm):
        return list(self.pos)

    def prefill_rows(self, llm, rows):
        for r, toks in enumerate(rows):
            self.pos[r] += len(toks)
        self.calls.append(("prefill", [len(t) for t in rows]))

    def step_rows(self, llm, ids, *, logits=True, sampling=None, uniforms=None):
        out = np.array([self.next_token(int(t), self.pos[r], self.vocab) for r, t in enumerate(ids)], np.int32)
        for r in range(len(ids)):
            self.pos[r] += 1
        self.calls.append(("step", len(ids)))
        return None, out


def solo(prompt: list[int], max_tokens: int, eos: int, vocab: int = 50) -> list[int]:
    """The same stream decoded alone (the reference's control flow)."""
    pos, cur, out = len(prompt) - 1, prompt[-1], []
    for _ in range(max_tokens):
        tok = RowCore.next_token(cur, pos, vocab)
        pos += 1
        if tok == eos:
            break
        out.append(tok)
        cur = tok
    return out


def _sched(core: RowCore, rows: int, *, eos: int = 0, max_tokens: int = 6) -> BatchScheduler:
    return BatchScheduler(core=core, llm={}, rows=rows, decode=lambda t: f"<{t}>", eos=eos, max_tokens=max_tokens,
                          sampling=(0.0, 0, 1.0), capacity=10_000)


async def _collect(sched: BatchScheduler, prompt: list[int]) -> list[int]:
    return [int(p[1:-1]) async for p in sched.stream(prompt)]


def test_concurrent_streams_equal_their_solo_runs() -> None:
    core = RowCore(rows=4)
    sched = _sched(core, 4, eos=49, max_tokens=9)
    prompts = [[2, 5, 9], [2, 11], [2, 3, 4, 5, 6, 7], [2, 8, 8], [2, 1], [2, 30, 31, 32]]

    async def main():
        return await asyncio.gather(*[_collect(sched, p) for p in prompts])

    got = asyncio.run(main())
    sched.close()
    for p, g in zip(prompts, got):
        assert g == solo(p, 9, 49), p
    assert sched.max_live == 4  # six streams over four rows: the extra two waited for free rows
    assert any(c[0] == "step" and c[1] > 1 for c in core.calls)  # rows decoded together


def test_eos_and_empty_piece_and_max_tokens() -> None:
    core = RowCore(rows=2)
    prompt = [2, 5]
    full = solo(prompt, 50, eos=-1)
    eos = full[3]
    sched = _sched(core, 2, eos=eos, max_tokens=50)
    assert asyncio.run(_collect(sched, prompt)) == full[:3]
    sched.close()
    sched = BatchScheduler(core=RowCore(2), llm={}, rows=2, decode=lambda t: "" if t == full[1] else f"<{t}>",
                           eos=-1, max_tokens=50, sampling=(0.0, 0, 1.0), capacity=10_000)
    assert asyncio.run(_collect(sched, prompt)) == full[:1]
    sched.close()


def test_cancelled_stream_frees_its_row() -> None:
    core = RowCore(rows=1)
    sched = _sched(core, 1, eos=-1, max_tokens=1000)

    async def main():
        gen = sched.stream([2, 5])
        first = await gen.__anext__()
        await gen.aclose()  # the consumer goes away mid-stream
        rest = await _collect(sched, [2, 7])  # the only row must be reusable
        return first, rest

    first, rest = asyncio.run(main())
    sched.close()
    assert first == f"<{solo([2, 5], 1, -1)[0]}>"
    assert rest == solo([2, 7], 1000, -1)
    assert ("set_pos", (0, 0)) in core.calls


def test_non_string_piece_is_type_error() -> None:
    sched = BatchScheduler(core=RowCore(1), llm={}, rows=1, decode=lambda t: b"x", eos=-1, max_tokens=3,
                           sampling=(0.0, 0, 1.0), capacity=10_000)
    with pytest.raises(TypeError, match="non-string"):
        asyncio.run(_collect(sched, [2, 3]))
    sched.close()


def test_backend_error_reaches_the_stream() -> None:
    class Broken(RowCore):
        def step_rows(self, *a, **k):
            raise RuntimeError("device step failed")

    sched = _sched(Broken(2), 2)
    with pytest.raises(RuntimeError, match="device step failed"):
        asyncio.run(_collect(sched, [2, 3]))
    sched.close()
