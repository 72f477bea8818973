"""The drop-in API end to end on the device: a synthetic checkpoint written as
safetensors, read back by the loader, run by SyncGemmaModel and by the batching
AsyncGemmaModel (a stub tokenizer maps text "a b c" to ids [a, b, c] and id t
back to "<t>").

* SyncGemmaModel.generate_stream (greedy) equals the oracle's stream under the
  reference's control flow (BOS, prefill of tokens[:-1], EOS).
* Concurrent AsyncGemmaModel.generate_stream calls -- more streams than rows --
  are decoded together and each equals its own batch-1 run.
* Sampled streams (T 0.7, top-k 64) with given uniform variates equal the
  batch-1 device draw with the same variates, stream by stream.
"""

from __future__ import annotations

import asyncio
from pathlib import Path
from unittest import mock

import numpy as np
import pytest

import mogemma_b200.model as api
import oracle
from mogemma_b200 import GenerationConfig, SyncGemmaModel, _core, synth
from mogemma_b200.model import AsyncGemmaModel
from mogemma_b200.serving import BatchScheduler

pytestmark = pytest.mark.gpu

DIMS = synth.tiny(vocab=3000)
PROMPTS = ["5 9 13", "2 100 7 7", "44", "2 8 9 10 11 12 13", "300 301", "2 17 18"]


class _Tok:
    def encode(self, text):
        return mock.MagicMock(ids=[int(x) for x in text.split()])

    def decode(self, ids):
        return f"<{ids[0]}>"

    def token_to_id(self, token):
        return None  # no EOS alias: id 0 ends a stream

    def enable_truncation(self, **_):
        return None

    def enable_padding(self, **_):
        return None


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory) -> tuple[Path, dict]:
    d = tmp_path_factory.mktemp("tiny-ckpt")
    w = synth.make_weights(DIMS, seed=21)
    synth.write_safetensors(w, d)
    (d / "tokenizer.model").touch()
    return d, w


@pytest.fixture(autouse=True)
def stub_tokenizer():
    with mock.patch.object(api, "_Tokenizer", lambda *_a, **_k: _Tok()):
        yield


def _oracle_stream(w: dict, ids: list[int], n: int) -> list[int]:
    toks = ids if ids and ids[0] == 2 else [2, *ids]
    ref = oracle.RefModel(w, max_seq_len=512)
    for t in toks[:-1]:
        ref.step_no_logits(t)
    cur, out = toks[-1], []
    for _ in range(n):
        cur = int(np.argmax(ref.step(cur)))
        if cur == 0:
            break
        out.append(cur)
    return out


def test_loader_to_sync_model_greedy_equals_oracle(ckpt) -> None:
    d, w = ckpt
    model = SyncGemmaModel(GenerationConfig(model_path=d, max_tokens=20, temperature=0.0))
    for text in PROMPTS[:3]:
        got = [int(p[1:-1]) for p in model.generate_stream(text)]
        assert got == _oracle_stream(w, [int(x) for x in text.split()], 20), text


def test_async_streams_batched_and_equal_to_batch1(ckpt) -> None:
    d, _w = ckpt
    cfg = GenerationConfig(model_path=d, max_tokens=24, temperature=0.0)
    solo = SyncGemmaModel(cfg)
    want = [[int(p[1:-1]) for p in solo.generate_stream(t)] for t in PROMPTS]
    model = AsyncGemmaModel(cfg, max_concurrent=4)

    async def run(text):
        return [int(p[1:-1]) async for p in model.generate_stream(text)]

    async def main():
        return await asyncio.gather(*[run(t) for t in PROMPTS])

    got = asyncio.run(main())
    sched = model._scheduler  # noqa: SLF001
    assert sched is not None and sched.max_live >= 2, "streams were not decoded together"
    model.close()
    assert got == want


def test_sampled_streams_with_shared_variates(ckpt) -> None:
    d, w = ckpt
    rows = 3
    llm = _core.init_model(synth.metadata_of(w), max_batch=rows, capacity=256)
    rng = np.random.default_rng(4)
    prompts = [[2, *[int(x) for x in t.split()]] for t in PROMPTS[:5]]
    us = [rng.random(16) for _ in prompts]
    sched = BatchScheduler(core=_core, llm=llm, rows=rows, decode=lambda t: f"<{t}>", eos=-1, max_tokens=16,
                           sampling=(0.7, 64, 1.0), capacity=256)

    async def run(i):
        return [int(p[1:-1]) async for p in sched.stream(prompts[i], variates=lambda k, i=i: float(us[i][k]))]

    async def main():
        return await asyncio.gather(*[run(i) for i in range(len(prompts))])

    got = asyncio.run(main())
    sched.close()
    llm["_handle"].close()
    one = _core.init_model(synth.metadata_of(w), capacity=256)
    for i, p in enumerate(prompts):
        one["_handle"].set_pos(0)
        one["pos"] = 0
        _core.prefill(one, p[:-1])
        cur, want = p[-1], []
        for k in range(16):
            cur = _core.step_sample(one, cur, 0.7, 64, 1.0, uniform=float(us[i][k]))
            want.append(cur)
        assert got[i] == want, i
