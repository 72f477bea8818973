"""Runtime configuration objects.

Same frozen dataclasses, field names, defaults and validation messages as the
reference (``src/py/mogemma/config.py:13-92``): they are part of the drop-in
contract.  ``device`` is accepted and ignored there; here every model runs on
a CUDA device chosen with ``MOGEMMA_B200_DEVICE`` (default 0).
"""

from dataclasses import dataclass, field
from pathlib import Path

_BAD_PATH = "model_path must be a non-empty local path or a valid Google model id"
_BAD_SEQ = "max_sequence_length must be greater than 0"
_BAD_BATCH = "batch_size must be greater than 0"
_BAD_TOKENS = "max_tokens must be greater than 0"


def _check_path(model_path: Path | str) -> None:
    text = str(model_path)
    if not text or text in {".", ".."}:
        raise ValueError(_BAD_PATH)


@dataclass(frozen=True)
class EmbeddingConfig:
    """Configuration for Gemma 3 embedding generation."""

    model_path: Path | str = "gemma3-270m-it"
    device: str = "cpu"
    max_sequence_length: int = 512
    batch_size: int = 1
    metadata: dict[str, str] = field(default_factory=dict)

    def __post_init__(self) -> None:
        """Validate configuration."""
        _check_path(self.model_path)
        if self.max_sequence_length <= 0:
            raise ValueError(_BAD_SEQ)
        if self.batch_size <= 0:
            raise ValueError(_BAD_BATCH)


@dataclass(frozen=True)
class GenerationConfig:
    """Configuration for Gemma 3 text generation."""

    model_path: Path | str = "gemma3-270m-it"
    device: str = "cpu"
    max_sequence_length: int = 512
    max_tokens: int = 128
    temperature: float = 1.0
    top_k: int = 50
    top_p: float = 1.0

    def __post_init__(self) -> None:
        """Validate configuration."""
        if self.temperature < 0:
            raise ValueError("temperature must be non-negative")
        if self.top_k < 0:
            raise ValueError("top_k must be non-negative")
        if not (0.0 <= self.top_p <= 1.0):
            raise ValueError("top_p must be between 0.0 and 1.0")
        _check_path(self.model_path)
        if self.max_sequence_length <= 0:
            raise ValueError(_BAD_SEQ)
        if self.max_tokens <= 0:
            raise ValueError(_BAD_TOKENS)
