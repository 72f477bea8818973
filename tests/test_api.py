"""The drop-in Python API (SyncGemmaModel, AsyncGemmaModel, EmbeddingModel) on
stub backends, with the control-flow contracts the reference's own tests pin:

* src/py/tests/test_gemma_model.py:161-198 -- the exact sequence of ``step``
  calls (BOS inserted, prefill of tokens[:-1], decode from the last prompt
  token) and the decoded output;  :201-229 -- stop on EOS;  :232-255 -- a
  non-string decode is a TypeError;  :258-280 -- missing/failing core;
  :283-333 -- instruction templates for ``-it`` models.
* src/py/tests/test_contracts_integration.py:121-171 -- error contracts.
* src/py/tests/test_async.py:56-100 -- async generate / stream / EOS.
* src/py/tests/test_embeddings.py:118-230 -- embedding row and dtype contracts.

A backend that offers only the reference trio (init_model / step /
generate_embeddings) is driven exactly as the reference drives its ``_core``;
temperature > 0 draws go to the CUDA sampler, replaced here by a recording stub.
No GPU is used.
"""

from __future__ import annotations

import asyncio
import json
import struct
from pathlib import Path
from unittest import mock

import numpy as np
import pytest

import mogemma_b200.model as api
from mogemma_b200 import EmbeddingConfig, EmbeddingModel, GenerationConfig, SyncGemmaModel
from mogemma_b200.hub import HubManager
from mogemma_b200.model import AsyncGemmaModel


def _write_empty_checkpoint(d: Path) -> Path:
    d.mkdir(parents=True, exist_ok=True)
    header = b"{}"
    (d / "model.safetensors").write_bytes(struct.pack("<Q", len(header)) + header)
    (d / "tokenizer.model").touch()
    return d


@pytest.fixture
def ckpt(tmp_path: Path) -> Path:
    return _write_empty_checkpoint(tmp_path / "tiny-model")


@pytest.fixture
def tok():
    """A tokenizer double: prompt ids [1, 2, 3], every token decodes to "<id>"."""
    with mock.patch.object(api, "_Tokenizer") as cls:
        t = mock.MagicMock()
        t.encode.return_value = mock.MagicMock(ids=[1, 2, 3])
        t.encode_batch.side_effect = lambda texts, **_: [mock.MagicMock(ids=[1, 2, 3]) for _ in texts]
        t.decode.side_effect = lambda ids: f"<{ids[0]}>"
        t.token_to_id.return_value = 999  # EOS id that no stub produces unless a test says so
        cls.return_value = t
        yield t


class ScriptedCore:
    """Reference-trio backend: returns the logits rows of `script` in turn
    (the last row repeats) and records every call."""

    def __init__(self, script: list[list[float]]) -> None:
        self.script = [np.asarray(r, np.float32) for r in script]
        self.calls: list[tuple[int, float, int, float]] = []

    def init_model(self, _metadata: object) -> object:
        return {}

    def step(self, llm: object, token_id: int, temperature: float, top_k: int, top_p: float) -> np.ndarray:
        del llm
        self.calls.append((token_id, temperature, top_k, top_p))
        return self.script[min(len(self.calls) - 1, len(self.script) - 1)]

    def generate_embeddings(self, llm: object, tokens: object) -> np.ndarray:
        del llm
        return np.ones((len(tokens), 768), np.float32)


class RecordingSampler:
    """Stands in for the CUDA sampler (``_core.sample``): first argmax, arguments recorded."""

    def __init__(self) -> None:
        self.seen: list[tuple[float, int, float]] = []

    def sample(self, values, temperature, top_k, top_p, **_):
        self.seen.append((temperature, top_k, top_p))
        return np.array([int(np.argmax(values))], np.int32)


@pytest.fixture(autouse=True)
def sampler(monkeypatch: pytest.MonkeyPatch) -> RecordingSampler:
    s = RecordingSampler()
    monkeypatch.setattr(api, "_device_core", s)
    return s


def _use(monkeypatch: pytest.MonkeyPatch, core: object) -> object:
    monkeypatch.setattr(api, "_core", core)
    return core


# ---------------------------------------------------------------- generation control flow
def test_step_sequence_and_output_match_reference_golden(ckpt, tok, monkeypatch) -> None:
    # calls 1-3 are the prefill of BOS + [1, 2]; call 4 decodes from token 3 and picks 2
    core = _use(monkeypatch, ScriptedCore([[4, 0, 0]] * 3 + [[0, 0, 5], [4, 0, 0]]))
    model = SyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=2, temperature=0.0, top_k=50, top_p=1.0))
    assert model.generate("Hello") == "<2><0>"
    assert core.calls == [(2, 0.0, 50, 1.0), (1, 0.0, 50, 1.0), (2, 0.0, 50, 1.0), (3, 0.0, 50, 1.0),
                          (2, 0.0, 50, 1.0)]


def test_generation_stops_on_eos(ckpt, tok, monkeypatch) -> None:
    tok.token_to_id.return_value = 0  # "<end_of_turn>" -> 0
    core = _use(monkeypatch, ScriptedCore([[0, 0, 0]] * 3 + [[5, 0, 0]]))
    model = SyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=5, temperature=0.0))
    assert model.generate("Hello") == ""
    assert len(core.calls) == 4


def test_generation_stops_on_empty_piece(ckpt, tok, monkeypatch) -> None:
    tok.decode.side_effect = None
    tok.decode.return_value = ""
    core = _use(monkeypatch, ScriptedCore([[5, 0, 0]]))
    model = SyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=5, temperature=0.0))
    assert model.generate("Hello") == ""
    assert len(core.calls) == 4


def test_bos_not_duplicated(ckpt, tok, monkeypatch) -> None:
    tok.encode.return_value = mock.MagicMock(ids=[2, 7])
    core = _use(monkeypatch, ScriptedCore([[5, 0, 0]]))
    SyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=1, temperature=0.0)).generate("x")
    assert [c[0] for c in core.calls] == [2, 7]


def test_non_string_decode_is_type_error(ckpt, tok, monkeypatch) -> None:
    tok.decode.side_effect = None
    tok.decode.return_value = b"\xff"
    _use(monkeypatch, ScriptedCore([[0, 0, 5]]))
    model = SyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=1))
    with pytest.raises(TypeError, match=r"tokenizer\.decode returned non-string output"):
        model.generate("Hello")


def test_empty_logits_is_a_value_error(ckpt, tok, monkeypatch) -> None:
    _use(monkeypatch, ScriptedCore([[]]))
    model = SyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=1, temperature=0.0))
    with pytest.raises(ValueError, match="backend returned empty logits"):
        model.generate("hello")


def test_sampled_generation_uses_device_sampler(ckpt, tok, monkeypatch, sampler) -> None:
    """temperature > 0 on host logits: the draw goes to the CUDA sampler with the config's arguments."""
    _use(monkeypatch, ScriptedCore([[5, 0, 0]]))
    out = SyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=5, temperature=0.7, top_k=10,
                                          top_p=0.9)).generate("Hello")
    assert out == "<0>" * 5
    assert sampler.seen == [(0.7, 10, 0.9)] * 5


def test_consecutive_generations_restart_at_position_zero(ckpt, tok, monkeypatch) -> None:
    class PosCore(ScriptedCore):
        def step(self, llm, token_id, temperature, top_k, top_p):
            llm["pos"] = llm.get("pos", 0) + 1
            self.positions.append(llm["pos"])
            return super().step(llm, token_id, temperature, top_k, top_p)

    core = PosCore([[5, 0, 0]])
    core.positions = []
    _use(monkeypatch, core)
    model = SyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=2, temperature=0.0))
    model.generate("a")
    model.generate("b")
    assert core.positions == [1, 2, 3, 4, 5] * 2


def test_instruction_template_for_it_models(tmp_path, tok, monkeypatch) -> None:
    d = _write_empty_checkpoint(tmp_path / "gemma3-270m-it")
    _use(monkeypatch, ScriptedCore([[5, 0, 0]]))
    tok.decode.side_effect = None
    tok.decode.return_value = ""
    SyncGemmaModel(GenerationConfig(model_path=d, max_tokens=1)).generate("What is the capital of France?")
    prompt = tok.encode.call_args.args[0]
    assert prompt.startswith("<start_of_turn>user\n") and prompt.endswith("<start_of_turn>model\n")
    templated = "<start_of_turn>user\nhi\n<end_of_turn>\n<start_of_turn>model\n"
    SyncGemmaModel(GenerationConfig(model_path=d, max_tokens=1)).generate(templated)
    assert tok.encode.call_args.args[0] == templated


# ---------------------------------------------------------------- construction contracts
def test_missing_core_and_failing_init(ckpt, tok, monkeypatch) -> None:
    monkeypatch.setattr(api, "_core", None)
    with pytest.raises(RuntimeError, match="Mojo core is unavailable"):
        SyncGemmaModel(GenerationConfig(model_path=ckpt))
    with pytest.raises(RuntimeError, match="Mojo core is unavailable"):
        EmbeddingModel(EmbeddingConfig(model_path=ckpt))

    class Failing:
        def init_model(self, _):
            raise RuntimeError("checkpoint missing or unreadable")

    monkeypatch.setattr(api, "_core", Failing())
    with pytest.raises(RuntimeError, match="generation model failed to initialize"):
        SyncGemmaModel(GenerationConfig(model_path=ckpt))
    with pytest.raises(RuntimeError, match="embedding model failed to initialize"):
        EmbeddingModel(EmbeddingConfig(model_path=ckpt))


def test_string_config_and_hub_resolution(tmp_path, tok, monkeypatch) -> None:
    _use(monkeypatch, ScriptedCore([[5, 0, 0]]))
    d = _write_empty_checkpoint(tmp_path / "google--gemma-3-4b-it")
    calls: list[tuple[str, bool, bool]] = []

    def fake_resolve(self, model_id, *, download_if_missing, strict, **_):
        calls.append((model_id, download_if_missing, strict))
        return d

    monkeypatch.setattr(HubManager, "resolve_model", fake_resolve)
    SyncGemmaModel(GenerationConfig(model_path="google/gemma-3-4b-it"))
    EmbeddingModel(EmbeddingConfig(model_path="google/gemma-3-4b-it"))
    assert calls == [("google/gemma-3-4b-it", True, True)] * 2
    monkeypatch.undo()
    _use(monkeypatch, ScriptedCore([[5, 0, 0]]))
    m = SyncGemmaModel(str(d))
    assert str(m.config.model_path) == str(d)


def test_unknown_model_id_is_not_found(tok) -> None:
    with pytest.raises(HubManager.ModelNotFoundError, match="not found in the public gemma-data bucket"):
        SyncGemmaModel(GenerationConfig(model_path="bert-base-uncased-missing"))
    with pytest.raises(HubManager.ModelNotFoundError, match="not found in the public gemma-data bucket"):
        EmbeddingModel(EmbeddingConfig(model_path="bert-base-uncased-missing"))


def test_config_validation() -> None:
    with pytest.raises(ValueError, match="temperature"):
        GenerationConfig(model_path="m", temperature=-1.0)
    with pytest.raises(ValueError, match="top_p"):
        GenerationConfig(model_path="m", top_p=1.5)
    with pytest.raises(ValueError, match="max_tokens"):
        GenerationConfig(model_path="m", max_tokens=0)
    with pytest.raises(ValueError, match="batch_size"):
        EmbeddingConfig(model_path="m", batch_size=0)
    assert EmbeddingConfig(model_path="m").device == "cpu"


# ---------------------------------------------------------------- async
def test_async_generate_stream_and_eos(ckpt, tok, monkeypatch) -> None:
    _use(monkeypatch, ScriptedCore([[0, 5, 0]]))
    model = AsyncGemmaModel(GenerationConfig(model_path=ckpt, max_tokens=5, temperature=0.0))

    async def run() -> tuple[str, list[str]]:
        full = await model.generate("Hello")
        pieces = [p async for p in model.generate_stream("Hello")]
        return full, pieces

    full, pieces = asyncio.run(run())
    assert full == "<1>" * 5 and pieces == ["<1>"] * 5
    tok.token_to_id.return_value = 1
    assert asyncio.run(_collect(model)) == []


async def _collect(model: AsyncGemmaModel) -> list[str]:
    return [p async for p in model.generate_stream("Hello")]


# ---------------------------------------------------------------- embeddings
def test_embedding_rows_and_dtype(ckpt, tok, monkeypatch) -> None:
    _use(monkeypatch, ScriptedCore([[0]]))
    model = EmbeddingModel(EmbeddingConfig(model_path=ckpt))
    one = model.embed("Hello world")
    assert one.shape == (1, 768) and one.dtype == np.float32
    assert model.embed(["a", "b"]).shape == (2, 768)
    with pytest.raises(ValueError, match="at least one value"):
        model.embed([])
    with pytest.raises(ValueError, match="at least one row"):
        model.embed_tokens(np.empty((0, 1), np.int32))
    with pytest.raises(ValueError, match="2D array"):
        model.embed_tokens(np.zeros(3, np.int32))


def test_embedding_backend_contracts(ckpt, tok, monkeypatch) -> None:
    class Flat(ScriptedCore):
        def generate_embeddings(self, llm, tokens):
            return np.zeros((768,), np.float32)

    class WrongRows(ScriptedCore):
        def generate_embeddings(self, llm, tokens):
            return np.zeros((1, 768), np.float32)

    class F64(ScriptedCore):
        def generate_embeddings(self, llm, tokens):
            return np.ones((len(tokens), 768), np.float64)

    toks = np.array([[1, 2, 3]], np.int32)
    _use(monkeypatch, Flat([[0]]))
    with pytest.raises(ValueError, match="expected 2D embeddings"):
        EmbeddingModel(EmbeddingConfig(model_path=ckpt)).embed_tokens(toks)
    _use(monkeypatch, WrongRows([[0]]))
    with pytest.raises(ValueError, match="embedding rows"):
        EmbeddingModel(EmbeddingConfig(model_path=ckpt)).embed(["first", "second"])
    _use(monkeypatch, F64([[0]]))
    out = EmbeddingModel(EmbeddingConfig(model_path=ckpt)).embed_tokens(toks)
    assert out.dtype == np.float32 and out.shape == (1, 768)


def test_pretokenized_embedding_needs_no_tokenizer(ckpt, monkeypatch) -> None:
    _use(monkeypatch, ScriptedCore([[0]]))
    monkeypatch.setattr(api, "SENTENCEPIECE_INSTALLED", False)
    model = EmbeddingModel(EmbeddingConfig(model_path=ckpt))
    assert model.embed_tokens(np.array([[1, 2, 3], [4, 5, 6]], np.int32)).shape == (2, 768)
    with pytest.raises(ModuleNotFoundError, match="embed_tokens"):
        model.embed("hello")


def test_checkpoint_header_is_read(tmp_path, tok, monkeypatch) -> None:
    """The loader hands the core {name: (pointer, shape, dtype)} from the safetensors header."""
    seen = {}

    class Recorder(ScriptedCore):
        def init_model(self, metadata):
            seen.update(metadata)
            return {}

    d = tmp_path / "m"
    d.mkdir()
    arr = np.arange(6, dtype=np.float32).reshape(2, 3)
    header = json.dumps({"w": {"dtype": "F32", "shape": [2, 3], "data_offsets": [0, arr.nbytes]}}).encode()
    (d / "model.safetensors").write_bytes(struct.pack("<Q", len(header)) + header + arr.tobytes())
    _use(monkeypatch, Recorder([[0]]))
    SyncGemmaModel(GenerationConfig(model_path=d))
    ptr, shape, dtype = seen["w"]
    assert shape == (2, 3) and dtype == "F32" and isinstance(ptr, int)
