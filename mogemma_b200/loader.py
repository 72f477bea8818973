"""Safetensors weights as zero-copy host pointers.

Produces the ``{name: (host_ptr, shape, dtype)}`` metadata that the reference
loader hands to ``_core.init_model`` (src/py/mogemma/loader.py:86-107): each
file is memory-mapped read-only and the pointers stay valid while the loader
is open.  ``init_model`` copies the tensors to HBM once, so the mapping can be
closed after the model is built.  Orbax/OCDBT checkpoints (converted by the
reference's convert.py) are outside this engine's scope.
"""

from __future__ import annotations

import json
import mmap
import struct
from pathlib import Path
from typing import Any, Protocol

import numpy as np


class SafetensorsLoader:
    """Memory-mapped safetensors files exposing raw tensor pointers."""

    def __init__(self, model_path: str | Path) -> None:
        self.model_path = Path(model_path)
        self.mmaps: dict[str, mmap.mmap] = {}
        self.file_objs: dict[str, Any] = {}
        self.tensor_file_map: dict[str, str] = {}
        self.tensor_metadata: dict[str, dict[str, Any]] = {}
        self.file_data_offsets: dict[str, int] = {}
        self._bases: dict[str, int] = {}
        self._views: dict[str, np.ndarray] = {}
        self._open_all()

    def _open_all(self) -> None:
        p = self.model_path
        if p.is_file():
            self._map(p.name, p)
            return
        index = p / "model.safetensors.index.json"
        if index.exists():
            weight_map = json.loads(index.read_text(encoding="utf-8")).get("weight_map", {})
            self.tensor_file_map = dict(weight_map)
            for fname in sorted(set(weight_map.values())):
                fpath = p / fname
                if not fpath.exists():
                    msg = f"Missing weights file: {fpath}"
                    raise FileNotFoundError(msg)
                self._map(fname, fpath)
            return
        single = p / "model.safetensors"
        if not single.exists():
            msg = f"No model.safetensors or index found in {p}"
            raise FileNotFoundError(msg)
        self._map("model.safetensors", single)

    def _map(self, fname: str, fpath: Path) -> None:
        f = fpath.open("rb")
        m = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        self.file_objs[fname] = f
        self.mmaps[fname] = m
        (hlen,) = struct.unpack("<Q", m[:8])
        header = json.loads(m[8 : 8 + hlen])
        self.file_data_offsets[fname] = 8 + hlen
        view = np.frombuffer(m, dtype=np.uint8)
        self._views[fname] = view
        self._bases[fname] = int(view.ctypes.data)
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            self.tensor_file_map[name] = fname
            self.tensor_metadata[name] = meta

    def get_tensor_metadata(self) -> dict[str, tuple[int, tuple[int, ...], str]]:
        """``{name: (data_pointer, shape, dtype)}`` for the engine."""
        out: dict[str, tuple[int, tuple[int, ...], str]] = {}
        for name, meta in self.tensor_metadata.items():
            fname = self.tensor_file_map[name]
            ptr = self._bases[fname] + self.file_data_offsets[fname] + int(meta["data_offsets"][0])
            out[name] = (ptr, tuple(int(s) for s in meta["shape"]), str(meta["dtype"]))
        return out

    def __enter__(self) -> SafetensorsLoader:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()

    @staticmethod
    def can_load(model_path: Path) -> bool:
        """True when ``model_path`` holds safetensors weights."""
        if model_path.is_file() and model_path.suffix == ".safetensors":
            return True
        if not model_path.is_dir():
            return False
        return (model_path / "model.safetensors").exists() or (model_path / "model.safetensors.index.json").exists()

    def close(self) -> None:
        """Unmap files (pointers from get_tensor_metadata become invalid)."""
        self._views.clear()
        for m in self.mmaps.values():
            try:
                m.close()
            except BufferError:
                pass
        for f in self.file_objs.values():
            f.close()
        self.mmaps.clear()
        self.file_objs.clear()
        self.tensor_file_map.clear()
        self.tensor_metadata.clear()


class ModelLoader(Protocol):
    """What the model classes need from a weights loader."""

    model_path: Path

    def get_tensor_metadata(self) -> dict[str, tuple[int, tuple[int, ...], str]]: ...

    def close(self) -> None: ...


def auto_loader(model_path: str | Path) -> ModelLoader:
    """Return a loader for ``model_path`` (safetensors only)."""
    path = Path(model_path)
    if SafetensorsLoader.can_load(path):
        return SafetensorsLoader(path)
    msg = (
        f"No supported model format found in {path}. "
        "Expected safetensors files (model.safetensors); convert Orbax/OCDBT checkpoints first."
    )
    raise FileNotFoundError(msg)
