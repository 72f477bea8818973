"""mogemma_b200: B200 (sm_100a) engine behind the MoGemma Python API.

Public names match the reference package ``mogemma`` (src/py/mogemma/__init__.py)
and are imported lazily.
"""

from importlib import import_module
from typing import TYPE_CHECKING

if TYPE_CHECKING:
    from .config import EmbeddingConfig, GenerationConfig
    from .hub import HubManager
    from .model import AsyncGemmaModel, EmbeddingModel, SyncGemmaModel

__all__ = ["AsyncGemmaModel", "EmbeddingConfig", "EmbeddingModel", "GenerationConfig", "HubManager", "SyncGemmaModel"]

_WHERE = {
    "AsyncGemmaModel": ".model",
    "EmbeddingConfig": ".config",
    "EmbeddingModel": ".model",
    "GenerationConfig": ".config",
    "HubManager": ".hub",
    "SyncGemmaModel": ".model",
}


def __getattr__(name: str) -> object:
    where = _WHERE.get(name)
    if where is None:
        msg = f"module 'mogemma_b200' has no attribute '{name}'"
        raise AttributeError(msg)
    value = getattr(import_module(where, __name__), name)
    globals()[name] = value
    return value
