"""Gemma 3 model classes: the drop-in Python API.

``SyncGemmaModel``, ``AsyncGemmaModel.generate_stream``, ``EmbeddingModel.embed``
and their constructors keep the reference signatures and control flow
(src/py/mogemma/model.py): BOS insertion, prompt templating for ``-it``
models, prefill of ``tokens[:-1]`` then decode from the last prompt token,
EOS aliases, stop on an empty decode, and the same error messages.

The backend is ``_core`` (the ctypes shim over the CUDA library).  When it
offers them, prefill runs without logits (``_core.prefill``) and each decode
step draws its token on the device (``_core.step_sample``), so 4 bytes cross
the bus per token instead of the 1 MB logits row.  A backend object that only
provides the reference trio (``init_model``/``step``/``generate_embeddings``)
is driven exactly like the reference drives ``mogemma._core``.
"""

from __future__ import annotations

import asyncio
import contextlib
from collections.abc import AsyncIterator, Generator, Iterator, Sequence
from pathlib import Path
from typing import Any, Protocol, cast

import numpy as np
import numpy.typing as npt

from .config import EmbeddingConfig, GenerationConfig
from .hub import HubManager
from .loader import ModelLoader, auto_loader

# Optional dependencies.  The names are module globals so that callers (and
# tests) can switch tokenization off the way the reference package allows.
try:
    from sentencepiece import SentencePieceProcessor as _SentencePiece  # type: ignore[import-untyped]
except ModuleNotFoundError:
    _SentencePiece = None
SENTENCEPIECE_INSTALLED = _SentencePiece is not None

try:
    from opentelemetry import trace as _otel
except ModuleNotFoundError:
    _otel = None


@contextlib.contextmanager
def _span(name: str, **attributes: object) -> Iterator[None]:
    """An OpenTelemetry span named ``name`` carrying ``attributes`` when the
    package is installed; otherwise nothing is recorded."""
    if _otel is None:
        yield
        return
    with _otel.get_tracer("mogemma_b200").start_as_current_span(name) as span:
        for key, value in attributes.items():
            span.set_attribute(key, value)
        yield

try:
    from . import _core
except ImportError:  # the CUDA library is not built: every model init fails loudly below
    _core = None  # type: ignore[assignment]

_device_core = _core


class _EncodedToken(Protocol):
    ids: Sequence[int]


class _Tokenizer:
    """sentencepiece wrapper with the small surface the models use."""

    def __init__(self, model_path: str) -> None:
        if _SentencePiece is None:
            raise ModuleNotFoundError("sentencepiece runtime is unavailable")
        self.sp = _SentencePiece(model_file=model_path)
        self._max_length: int | None = None

    def enable_truncation(self, *, max_length: int, **_: object) -> None:
        self._max_length = max_length

    def enable_padding(self, **_: object) -> None:
        return None

    def encode_batch(self, text: Sequence[str]) -> Sequence[_EncodedToken]:
        return [self.encode(t) for t in text]

    def encode(self, text: str) -> _EncodedToken:
        ids = list(self.sp.EncodeAsIds(text))
        if self._max_length is not None:
            ids = ids[: self._max_length]

        class _Encoded:
            def __init__(self, ids: list[int]) -> None:
                self.ids = ids

        return cast("_EncodedToken", _Encoded(ids))

    def decode(self, ids: Sequence[int]) -> str:
        return str(self.sp.DecodeIds(list(ids)))

    def token_to_id(self, token: str) -> int | None:
        tid = self.sp.piece_to_id(token)
        if tid == self.sp.unk_id() and token not in ("<unk>", " "):
            return None
        return int(tid)


_MATRIX_NDIM = 2
_BOS_TOKEN_ID = 2
_EOS_TOKEN_ID_ALIASES = ("<end_of_turn>", "</s>", "<eos>", "<|eos|>")
_TURN_START = "<start_of_turn>"
_TURN_END = "<end_of_turn>"


def _core_missing(kind: str) -> RuntimeError:
    if kind == "embedding":
        what = "embeddings", "embed()/embed_tokens()"
    else:
        what = "text generation", "generate()"
    return RuntimeError(
        f"Mojo core is unavailable for {what[0]}. "
        f"Build the B200 engine (mogemma_b200/libmogemma_cuda.so) before calling {what[1]}."
    )


def _resolve_model_path(raw_model_path: str | Path) -> Path:
    return HubManager().resolve_model(str(raw_model_path), download_if_missing=True, strict=True)


def _initialize_llm(loader: ModelLoader, *, model_type: str, rows: int = 1) -> object:
    if _core is None:
        raise _core_missing(model_type)
    try:
        if rows > 1 and hasattr(_core, "step_rows"):  # the CUDA engine: a model with several rows
            return _core.init_model(loader.get_tensor_metadata(), max_batch=rows)
        return _core.init_model(loader.get_tensor_metadata())
    except Exception as exc:
        msg = f"{model_type} model failed to initialize from '{loader.model_path}': {exc}"
        raise RuntimeError(msg) from exc


def _sample_next_token(logits: npt.ArrayLike, *, temperature: float, top_k: int, top_p: float) -> int:
    """Pick the next token from logits a backend returned to the host.

    Same rules as the reference helper (model.py:103-150); temperature <= 0 is
    the first argmax, every other setting is drawn by the CUDA sampler.
    """
    values = np.asarray(logits, dtype=np.float32).reshape(-1)
    if values.size == 0:
        raise ValueError("backend returned empty logits")
    if temperature <= 0:
        return int(np.argmax(values))
    if _device_core is None:
        msg = "sampling with temperature > 0 needs the CUDA engine (mogemma_b200/libmogemma_cuda.so)"
        raise RuntimeError(msg)
    seed = int(np.random.default_rng().integers(0, 2**63 - 1))
    return int(_device_core.sample(values, temperature, top_k, top_p, seed=seed)[0])


def _normalize_eos_token_id(tokenizer: _Tokenizer) -> int:
    for alias in _EOS_TOKEN_ID_ALIASES:
        tid = tokenizer.token_to_id(alias)
        if tid is not None:
            return int(tid)
    return 0


def _is_instruction_tuned_model(model_path: Path, config_model_path: str | Path) -> bool:
    return str(config_model_path).lower().endswith("-it") or model_path.name.lower().endswith("-it")


def _format_instruction_prompt(prompt: str) -> str:
    if _TURN_START in prompt or _TURN_END in prompt:
        return prompt
    return f"{_TURN_START}user\n{prompt}\n{_TURN_END}\n{_TURN_START}model\n"


class EmbeddingModel:
    """Mean-pooled Gemma 3 embeddings computed by the CUDA engine."""

    def __init__(self, config: EmbeddingConfig | str | None = None, tokenizer: _Tokenizer | None = None) -> None:
        if config is None:
            config = EmbeddingConfig()
        elif isinstance(config, str):
            config = EmbeddingConfig(model_path=config)
        self.config = config
        self._tokenizer = tokenizer
        self.model_path = _resolve_model_path(config.model_path)
        self._loader = auto_loader(self.model_path)
        self._llm: object | None = _initialize_llm(self._loader, model_type="embedding")

    def _ensure_tokenizer(self) -> _Tokenizer:
        if self._tokenizer is not None:
            return self._tokenizer
        if not SENTENCEPIECE_INSTALLED:
            msg = (
                "Text tokenization requires 'sentencepiece' dependency. "
                "Install with: pip install 'mogemma[llm]' or call embed_tokens(...) with pre-tokenized inputs."
            )
            raise ModuleNotFoundError(msg)
        sp_path = self.model_path / "tokenizer.model"
        if not sp_path.exists():
            msg = f"No tokenizer.model found in {self.model_path}"
            raise FileNotFoundError(msg)
        self._tokenizer = _Tokenizer(str(sp_path))
        return self._tokenizer

    def _embed_token_array(self, tokens: Sequence[Sequence[int]], input_count: int) -> npt.NDArray[np.float32]:
        if _core is None or self._llm is None:
            raise _core_missing("embedding")
        emb = np.asarray(_core.generate_embeddings(self._llm, tokens), dtype=np.float32)
        if emb.ndim != _MATRIX_NDIM:
            msg = f"expected 2D embeddings from backend, got {emb.ndim}D"
            raise ValueError(msg)
        if emb.shape[0] != input_count:
            msg = f"backend returned {emb.shape[0]} embedding rows for {input_count} inputs"
            raise ValueError(msg)
        return emb

    def embed(self, text: str | list[str]) -> npt.NDArray[np.float32]:
        """Tokenize ``text`` and return one embedding row per input."""
        texts = [text] if isinstance(text, str) else text
        if not texts:
            raise ValueError("text input must contain at least one value")
        tokenizer = self._ensure_tokenizer()
        with _span("EmbeddingModel.embed", text_count=len(texts)):
            tokenizer.enable_truncation(max_length=self.config.max_sequence_length)
            tokenizer.enable_padding()
            tokens = [e.ids for e in tokenizer.encode_batch(texts)]
            return self._embed_token_array(tokens, len(texts))

    def embed_tokens(self, tokens: Sequence[Sequence[int]] | npt.NDArray[np.int32]) -> npt.NDArray[np.float32]:
        """Embed pre-tokenized id rows."""
        if isinstance(tokens, np.ndarray):
            if tokens.ndim != _MATRIX_NDIM:
                msg = f"tokens must be a 2D array of token IDs, got shape {tokens.shape}"
                raise ValueError(msg)
            rows = tokens.tolist()
        else:
            rows = list(tokens)
        if len(rows) == 0:
            raise ValueError("tokens must contain at least one row")
        return self._embed_token_array(rows, len(rows))

    @property
    def tokenizer(self) -> _Tokenizer:
        return self._ensure_tokenizer()


class SyncGemmaModel:
    """Gemma 3 text generation on the CUDA engine."""

    def __init__(self, config: GenerationConfig | str | None = None, tokenizer: _Tokenizer | None = None, *,
                 _rows: int = 1) -> None:
        if config is None:
            config = GenerationConfig()
        elif isinstance(config, str):
            config = GenerationConfig(model_path=config)
        self.config = config
        self._tokenizer = tokenizer
        self.model_path = _resolve_model_path(config.model_path)
        self._loader = auto_loader(self.model_path)
        self._instruction_tuned = _is_instruction_tuned_model(self.model_path, config.model_path)
        self._llm: object | None = _initialize_llm(self._loader, model_type="generation", rows=_rows)

    def _ensure_tokenizer(self) -> _Tokenizer:
        if self._tokenizer is not None:
            return self._tokenizer
        if not SENTENCEPIECE_INSTALLED:
            msg = "Text generation requires 'sentencepiece' dependency. Install with: pip install 'mogemma[llm]'"
            raise ModuleNotFoundError(msg)
        sp_path = self.model_path / "tokenizer.model"
        if not sp_path.exists():
            msg = f"No tokenizer.model found in {self.model_path}"
            raise FileNotFoundError(msg)
        self._tokenizer = _Tokenizer(str(sp_path))
        return self._tokenizer

    def generate(self, prompt: str) -> str:
        """Generate text from ``prompt``."""
        return "".join(self.generate_stream(prompt))

    def _prompt_tokens(self, tokenizer: _Tokenizer, prompt: str) -> list[int]:
        text = _format_instruction_prompt(prompt) if self._instruction_tuned else prompt
        with _span("SyncGemmaModel.generate_stream", prompt_length=len(prompt)):
            tokenizer.enable_truncation(max_length=self.config.max_sequence_length)
            tokenizer.enable_padding()
            tokens = list(tokenizer.encode(text).ids)
            if not tokens or tokens[0] != _BOS_TOKEN_ID:
                tokens = [_BOS_TOKEN_ID, *tokens]
        return tokens

    def generate_stream(self, prompt: str) -> Generator[str, None, None]:
        """Yield decoded text one token at a time."""
        tokenizer = self._ensure_tokenizer()
        tokens = self._prompt_tokens(tokenizer, prompt)
        core = _core
        if core is None or self._llm is None:
            raise _core_missing("generation")
        if isinstance(self._llm, dict):
            self._llm["pos"] = 0
        cfg = self.config
        prefix = [int(t) for t in tokens[:-1]]
        if hasattr(core, "prefill"):
            core.prefill(self._llm, prefix)
        else:
            for t in prefix:
                core.step(self._llm, t, cfg.temperature, cfg.top_k, cfg.top_p)
        current = int(tokens[-1]) if tokens else int(_normalize_eos_token_id(tokenizer))
        eos = _normalize_eos_token_id(tokenizer)
        device_draw = hasattr(core, "step_sample")
        for _ in range(cfg.max_tokens):
            if device_draw:
                nxt = int(core.step_sample(self._llm, current, cfg.temperature, cfg.top_k, cfg.top_p))
            else:
                logits = core.step(self._llm, current, cfg.temperature, cfg.top_k, cfg.top_p)
                nxt = _sample_next_token(logits, temperature=cfg.temperature, top_k=cfg.top_k, top_p=cfg.top_p)
            if nxt == eos:
                return
            piece = tokenizer.decode([nxt])
            if not isinstance(piece, str):
                raise TypeError("tokenizer.decode returned non-string output")
            if not piece:
                return
            yield piece
            current = nxt

    @property
    def tokenizer(self) -> _Tokenizer:
        return self._ensure_tokenizer()


class AsyncGemmaModel:
    """asyncio front end of SyncGemmaModel.

    With the CUDA engine, concurrent ``generate_stream`` calls are batched onto
    one device model (``serving.BatchScheduler``): each stream gets a row, and
    one decode launch per step advances every live stream, each at its own
    position.  With a backend that only offers the reference trio
    (init_model / step / generate_embeddings), streams run one at a time in a
    worker thread, as the reference does (src/py/mogemma/model.py:379-420).
    """

    MAX_CONCURRENT = 8  # streams decoded together (rows of the persistent decode kernel)

    def __init__(self, config: GenerationConfig | str | None = None, *, max_concurrent: int | None = None) -> None:
        rows = self.MAX_CONCURRENT if max_concurrent is None else max(1, int(max_concurrent))
        self._model = SyncGemmaModel(config, _rows=rows)
        self._rows = rows
        self._scheduler: Any = None

    def _batcher(self) -> Any:
        """The scheduler when the backend is the CUDA engine with several rows, else None."""
        core = _core
        llm = self._model._llm  # noqa: SLF001
        if self._rows < 2 or core is None or not hasattr(core, "set_row_pos") or not isinstance(llm, dict):
            return None
        if llm.get("arch") == "nano":  # the Gemma 3n engine decodes one stream: serial, as the reference
            return None
        if self._scheduler is None:
            from .serving import BatchScheduler  # noqa: PLC0415

            tokenizer = self._model._ensure_tokenizer()  # noqa: SLF001
            cfg = self._model.config
            self._scheduler = BatchScheduler(
                core=core, llm=llm, rows=self._rows, decode=lambda t: tokenizer.decode([t]),
                eos=_normalize_eos_token_id(tokenizer), max_tokens=cfg.max_tokens,
                sampling=(cfg.temperature, cfg.top_k, cfg.top_p), capacity=int(llm["max_seq_len"]))
        return self._scheduler

    async def generate(self, prompt: str) -> str:
        if self._batcher() is not None:
            return "".join([piece async for piece in self.generate_stream(prompt)])
        return await asyncio.to_thread(self._model.generate, prompt)

    async def generate_stream(self, prompt: str) -> AsyncIterator[str]:
        batcher = self._batcher()
        if batcher is not None:
            tokens = self._model._prompt_tokens(self._model._ensure_tokenizer(), prompt)  # noqa: SLF001
            async for piece in batcher.stream(tokens):
                yield piece
            return
        gen = self._model.generate_stream(prompt)

        def pull() -> str | None:
            try:
                return next(gen)
            except StopIteration:
                return None

        try:
            while True:
                piece = await asyncio.to_thread(pull)
                if piece is None:
                    break
                yield piece
        except asyncio.CancelledError:
            gen.close()
            raise
        finally:
            with contextlib.suppress(RuntimeError):
                gen.close()

    def close(self) -> None:
        """Stop the batching worker (streams still waiting get an error)."""
        if self._scheduler is not None:
            self._scheduler.close()
            self._scheduler = None

    @property
    def tokenizer(self) -> _Tokenizer:
        return self._model.tokenizer


__all__: list[Any] = ["AsyncGemmaModel", "EmbeddingModel", "SyncGemmaModel"]
