"""Safetensors checkpoints as zero-copy host pointers.

``_core.init_model`` takes ``{name: (host_ptr, shape, dtype)}`` -- the metadata
the reference loader produces (src/py/mogemma/loader.py:86-107).  Here every
shard is memory-mapped read-only and each tensor is described by one table
entry (shard, byte range, shape, dtype), checked against the shard's size when
the header is read.  The pointers stay valid while the loader is open;
``init_model`` copies the tensors to HBM (through pinned staging buffers), so
the loader can be closed once the model is built.

Accepted layouts: a single ``.safetensors`` file, a directory holding
``model.safetensors``, or a sharded directory with
``model.safetensors.index.json``.  Orbax/OCDBT checkpoints are converted by
``mogemma_b200.convert`` first.
"""

from __future__ import annotations

import json
import mmap
import struct
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Protocol

import numpy as np

_ITEMSIZE = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "I64": 8, "I32": 4, "I16": 2, "I8": 1, "U8": 1, "BOOL": 1,
             "U16": 2, "U32": 4, "U64": 8, "F8_E4M3": 1, "F8_E5M2": 1}
_NUMPY = {"F64": np.float64, "F32": np.float32, "F16": np.float16, "I64": np.int64, "I32": np.int32,
          "I16": np.int16, "I8": np.int8, "U8": np.uint8, "BOOL": np.bool_, "U16": np.uint16, "U32": np.uint32,
          "U64": np.uint64, "BF16": np.uint16}


@dataclass(frozen=True)
class TensorEntry:
    """Where one tensor lives: shard index, absolute byte range in the shard, shape, dtype."""

    shard: int
    begin: int
    end: int
    shape: tuple[int, ...]
    dtype: str


class SafetensorsLoader:
    """Read-only memory maps of a checkpoint's shards with a tensor table."""

    def __init__(self, model_path: str | Path) -> None:
        self.model_path = Path(model_path)
        self._files: list[Any] = []
        self._maps: list[mmap.mmap] = []
        self._bytes: list[np.ndarray] = []  # uint8 views of the maps (pointer source)
        self.tensors: dict[str, TensorEntry] = {}
        try:
            for shard in self._shard_paths():
                self._open_shard(shard)
        except Exception:
            self.close()
            raise

    # ---------------------------------------------------------------- layout
    def _shard_paths(self) -> list[Path]:
        p = self.model_path
        if p.is_file():
            return [p]
        index = p / "model.safetensors.index.json"
        if index.is_file():
            weight_map = json.loads(index.read_text(encoding="utf-8")).get("weight_map", {})
            names = sorted(set(weight_map.values()))
            missing = [n for n in names if not (p / n).is_file()]
            if missing:
                msg = f"Missing weights file: {p / missing[0]}"
                raise FileNotFoundError(msg)
            return [p / n for n in names]
        if (p / "model.safetensors").is_file():
            return [p / "model.safetensors"]
        msg = f"No model.safetensors or index found in {p}"
        raise FileNotFoundError(msg)

    def _open_shard(self, path: Path) -> None:
        idx = len(self._maps)
        f = path.open("rb")
        self._files.append(f)
        size = path.stat().st_size
        if size < 8:  # noqa: PLR2004
            msg = f"{path}: not a safetensors file ({size} bytes)"
            raise ValueError(msg)
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        self._maps.append(mm)
        (hlen,) = struct.unpack("<Q", mm[:8])
        if 8 + hlen > size:
            msg = f"{path}: header of {hlen} bytes runs past the end of the file"
            raise ValueError(msg)
        header = json.loads(bytes(mm[8 : 8 + hlen]).decode("utf-8"))
        self._bytes.append(np.frombuffer(mm, dtype=np.uint8))
        data0 = 8 + hlen
        for name, meta in header.items():
            if name == "__metadata__":
                continue
            dtype = str(meta["dtype"])
            shape = tuple(int(s) for s in meta["shape"])
            lo, hi = (int(x) for x in meta["data_offsets"])
            if not (0 <= lo <= hi and data0 + hi <= size):
                msg = f"{path}: tensor '{name}' byte range [{lo}, {hi}) lies outside the file"
                raise ValueError(msg)
            if dtype in _ITEMSIZE and hi - lo != int(np.prod(shape, dtype=np.int64)) * _ITEMSIZE[dtype]:
                msg = f"{path}: tensor '{name}' holds {hi - lo} bytes, not {shape} x {dtype}"
                raise ValueError(msg)
            self.tensors[name] = TensorEntry(idx, data0 + lo, data0 + hi, shape, dtype)

    # ---------------------------------------------------------------- access
    def get_tensor_metadata(self) -> dict[str, tuple[int, tuple[int, ...], str]]:
        """``{name: (host_pointer, shape, dtype)}`` for ``_core.init_model``."""
        return {name: (int(self._bytes[e.shard].ctypes.data) + e.begin, e.shape, e.dtype)
                for name, e in self.tensors.items()}

    def array(self, name: str) -> np.ndarray:
        """A read-only NumPy view of one tensor (BF16 as its raw uint16 bits)."""
        e = self.tensors[name]
        return self._bytes[e.shard][e.begin : e.end].view(_NUMPY[e.dtype]).reshape(e.shape)

    @staticmethod
    def can_load(model_path: Path) -> bool:
        """True when ``model_path`` holds safetensors weights."""
        if model_path.is_file():
            return model_path.suffix == ".safetensors"
        return (model_path / "model.safetensors").is_file() or (model_path / "model.safetensors.index.json").is_file()

    def close(self) -> None:
        """Unmap every shard; pointers from get_tensor_metadata become invalid."""
        self._bytes.clear()
        for mm in self._maps:
            try:
                mm.close()
            except BufferError:  # a view handed out by array() is still alive
                pass
        for f in self._files:
            f.close()
        self._maps.clear()
        self._files.clear()
        self.tensors.clear()

    def __enter__(self) -> SafetensorsLoader:
        return self

    def __exit__(self, *exc: object) -> None:
        self.close()


class ModelLoader(Protocol):
    """What the model classes need from a weights loader."""

    model_path: Path

    def get_tensor_metadata(self) -> dict[str, tuple[int, tuple[int, ...], str]]: ...

    def close(self) -> None: ...


def auto_loader(model_path: str | Path) -> ModelLoader:
    """A loader for ``model_path`` (safetensors; convert Orbax checkpoints first)."""
    path = Path(model_path)
    if SafetensorsLoader.can_load(path):
        return SafetensorsLoader(path)
    msg = (
        f"No supported model format found in {path}. "
        "Expected safetensors files (model.safetensors); convert Orbax/OCDBT checkpoints first."
    )
    raise FileNotFoundError(msg)
