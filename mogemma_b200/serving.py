"""Continuous batching of concurrent generation streams onto one device model.

The reference's ``AsyncGemmaModel.generate_stream`` (src/py/mogemma/model.py:
379-420) runs one stream at a time through a shared synchronous model.  Here
concurrent streams share the device instead: every stream owns a row of a
model created with several rows (the decode kernel's batch), and one worker
thread advances all live rows together -- one decode launch per step for every
admitted stream, each row at its own position.

Scheduling, per iteration of the worker:

1. admit waiting streams into free rows (lowest row first): the row's position
   is reset to 0 and its prompt prefix ``tokens[:-1]`` is prefilled into that
   row alone (other rows are untouched);
2. one batched step over rows ``0 .. highest live row`` draws every live row's
   next token on the device (rows in that range without a stream decode a
   placeholder token; their positions are reset before they could reach the
   capacity, and a new stream re-prefills its row from position 0);
3. each live row's token goes through the reference's stopping rules -- EOS,
   an empty decoded piece, ``max_tokens`` -- and its piece is handed to the
   stream's asyncio queue; finished or cancelled streams release their rows.

Every stream sees the arithmetic of its own batch-1 run (per-row GEMV sums in
the same order; the draw rules of ``_sample_next_token``), so a greedy stream
is the same whether it runs alone or next to others.
"""

from __future__ import annotations

import asyncio
import threading
from collections import deque
from collections.abc import AsyncIterator, Callable, Sequence
from dataclasses import dataclass, field
from typing import Any


@dataclass
class _Stream:
    prompt: list[int]
    loop: asyncio.AbstractEventLoop
    queue: asyncio.Queue
    row: int = -1
    cur: int = 0
    produced: int = 0
    cancelled: bool = False
    done: bool = False
    variates: Callable[[int], float] | None = None  # step -> uniform variate (tests); None: device Philox


_END = object()


@dataclass
class BatchScheduler:
    """Runs admitted streams of one model together; see the module docstring.

    ``core`` is the ``_core`` module (or an object with ``set_row_pos``,
    ``prefill_rows`` and ``step_rows`` of the same meaning); ``decode`` maps a
    token id to its text piece; ``eos`` is the end-of-sequence id; ``sampling``
    is (temperature, top_k, top_p) shared by every stream of the model."""

    core: Any
    llm: Any
    rows: int
    decode: Callable[[int], str]
    eos: int
    max_tokens: int
    sampling: tuple[float, int, float]
    capacity: int
    _pending: deque = field(default_factory=deque)
    _live: dict = field(default_factory=dict)  # row -> _Stream
    _cv: threading.Condition = field(default_factory=threading.Condition)
    _thread: threading.Thread | None = None
    _closed: bool = False
    steps: int = 0  # batched decode steps run (for tests and monitoring)
    max_live: int = 0

    # ------------------------------------------------------------------ public
    async def stream(self, prompt: Sequence[int], variates: Callable[[int], float] | None = None) -> AsyncIterator[str]:
        """Pieces of one stream, as the reference's generate_stream yields them."""
        s = _Stream(list(prompt), asyncio.get_running_loop(), asyncio.Queue(), variates=variates)
        with self._cv:
            if self._closed:
                msg = "the batch scheduler is closed"
                raise RuntimeError(msg)
            self._pending.append(s)
            self._start()
            self._cv.notify()
        try:
            while True:
                item = await s.queue.get()
                if item is _END:
                    return
                if isinstance(item, BaseException):
                    raise item
                yield item
        finally:
            with self._cv:
                s.cancelled = True
                self._cv.notify()

    def close(self) -> None:
        with self._cv:
            self._closed = True
            self._cv.notify()
        if self._thread is not None:
            self._thread.join(timeout=30)

    # ------------------------------------------------------------------ worker
    def _start(self) -> None:
        if self._thread is None:
            self._thread = threading.Thread(target=self._run, name="mogemma-b200-batcher", daemon=True)
            self._thread.start()

    def _emit(self, s: _Stream, item: object) -> None:
        s.loop.call_soon_threadsafe(s.queue.put_nowait, item)

    def _finish(self, s: _Stream, item: object = _END) -> None:
        if not s.done:
            s.done = True
            self._emit(s, item)

    def _run(self) -> None:
        while True:
            with self._cv:
                while not self._closed and not self._pending and not self._live:
                    self._cv.wait()
                if self._closed:
                    for s in list(self._pending) + list(self._live.values()):
                        self._finish(s, RuntimeError("the batch scheduler is closed"))
                    return
                for row, s in list(self._live.items()):  # streams whose consumer went away
                    if s.cancelled:
                        del self._live[row]
                admit = []
                free = [r for r in range(self.rows) if r not in self._live]
                while self._pending and free:
                    s = self._pending.popleft()
                    if s.cancelled:
                        continue
                    s.row = free.pop(0)
                    self._live[s.row] = s
                    admit.append(s)
                live = dict(self._live)
            try:
                for s in admit:
                    self._admit(s)
                live = {r: s for r, s in live.items() if not s.done}
                if live:
                    self._step(live)
            except Exception as exc:  # noqa: BLE001 -- delivered to every waiting stream
                with self._cv:
                    for s in list(self._live.values()):
                        self._finish(s, exc)
                    self._live.clear()
            with self._cv:
                for row, s in list(self._live.items()):
                    if s.done:
                        del self._live[row]

    def _admit(self, s: _Stream) -> None:
        self.core.set_row_pos(self.llm, s.row, 0)
        prefix = s.prompt[:-1]
        if prefix:
            rows: list[list[int]] = [[] for _ in range(s.row + 1)]
            rows[s.row] = prefix
            self.core.prefill_rows(self.llm, rows)
        s.cur = int(s.prompt[-1])

    def _step(self, live: dict[int, _Stream]) -> None:
        n = max(live) + 1
        self.max_live = max(self.max_live, len(live))
        positions = self.core.row_positions(self.llm)
        for r in range(n):
            if r not in live and positions[r] >= self.capacity - 1:
                self.core.set_row_pos(self.llm, r, 0)
        ids = [live[r].cur if r in live else 0 for r in range(n)]
        uniforms = None
        if any(s.variates is not None for s in live.values()):
            uniforms = [live[r].variates(live[r].produced) if r in live and live[r].variates else 0.5
                        for r in range(n)]
        for r, s in live.items():
            if positions[r] >= self.capacity:
                self._finish(s, RuntimeError("Sequence length exceeded"))
        live = {r: s for r, s in live.items() if not s.done}
        if not live:
            return
        _, drawn = self.core.step_rows(self.llm, ids, logits=False, sampling=self.sampling, uniforms=uniforms)
        self.steps += 1
        for r, s in live.items():
            if s.cancelled:
                s.done = True
                continue
            tok = int(drawn[r])
            if tok == self.eos:
                self._finish(s)
                continue
            piece = self.decode(tok)
            if not isinstance(piece, str):
                self._finish(s, TypeError("tokenizer.decode returned non-string output"))
                continue
            if not piece:
                self._finish(s)
                continue
            self._emit(s, piece)
            s.cur = tok
            s.produced += 1
            if s.produced >= self.max_tokens:
                self._finish(s)
