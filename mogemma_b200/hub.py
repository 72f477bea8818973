"""Model path resolution (local directories and the local cache only).

Keeps the reference's ``HubManager.resolve_model`` contract
(src/py/mogemma/hub.py:51-80) for local paths and cached models.  Downloading
from Google Cloud Storage is outside this engine's scope (no network on the
compute path); an unknown id raises ``ModelNotFoundError``.
"""

from __future__ import annotations

from pathlib import Path


class HubManager:
    """Resolves model ids to local directories."""

    class GCSDownloadError(ConnectionError):
        """Raised when a download fails."""

    class ModelNotFoundError(FileNotFoundError):
        """Raised when a model id cannot be resolved."""

    def __init__(self, cache_path: str | Path | None = None) -> None:
        self.cache_path = Path(cache_path) if cache_path is not None else Path.home() / ".cache" / "mogemma"

    @staticmethod
    def _clean_model_id(model_id: str) -> str:
        clean = model_id.removeprefix("google/")
        return clean.replace("gemma-", "gemma") if clean.startswith("gemma-") else clean

    @staticmethod
    def _has_safetensors(path: Path) -> bool:
        return (path / "model.safetensors").exists() or (path / "model.safetensors.index.json").exists()

    def resolve_model(self, model_id: str, *, download_if_missing: bool = False, strict: bool = False,
                      **_kwargs: object) -> Path:
        """Map ``model_id`` to a local directory."""
        local = Path(model_id)
        if local.exists() and local.is_dir():
            return local
        if local.exists():
            if strict:
                msg = f"Model path '{model_id}' exists but is not a directory."
                raise ValueError(msg)
            return local
        cached = self.cache_path / model_id.replace("/", "--")
        if cached.is_dir() and self._has_safetensors(cached):
            return cached
        if download_if_missing:
            msg = (
                f"Model '{self._clean_model_id(model_id)}' not found in the public gemma-data bucket cache at "
                f"{self.cache_path}; this engine does not download models."
            )
            raise self.ModelNotFoundError(msg)
        if strict:
            msg = (
                f"Cannot resolve model path '{model_id}'. "
                "Use an existing local directory or a valid Google model id (e.g., gemma-3-1b-it)."
            )
            raise ValueError(msg)
        return local
