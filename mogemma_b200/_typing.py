"""Optional runtime dependencies (sentencepiece, opentelemetry), resolved once."""

from typing import Any

_SPProcessorImpl: Any | None
trace: Any | None

try:
    import sentencepiece as _sp  # type: ignore[import-untyped]

    _SPProcessorImpl = _sp.SentencePieceProcessor
except ModuleNotFoundError:
    _SPProcessorImpl = None

try:
    from opentelemetry import trace as _trace
except ModuleNotFoundError:
    trace = None
else:
    trace = _trace

SENTENCEPIECE_INSTALLED = _SPProcessorImpl is not None
OPENTELEMETRY_INSTALLED = trace is not None

__all__ = ["OPENTELEMETRY_INSTALLED", "SENTENCEPIECE_INSTALLED", "_SPProcessorImpl", "trace"]
