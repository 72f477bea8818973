"""Safetensors loader (src/py/mogemma/loader.py:59-107; its tests
src/py/tests/test_loader.py:25-74): pointers into the memory map, sharded
checkpoints, and the error contracts.  CPU only."""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

from mogemma_b200.loader import SafetensorsLoader, auto_loader

save_file = pytest.importorskip("safetensors.numpy").save_file


def _read(ptr: int, nbytes: int) -> bytes:
    return ctypes.string_at(ptr, nbytes)


def test_pointers_read_the_mapped_bytes(tmp_path: Path) -> None:
    f = tmp_path / "t.safetensors"
    u8 = np.array([42, 1, 2, 3], np.uint8)
    f32 = np.array([1.5, 2.5, 3.5], np.float32)
    save_file({"my_tensor": u8, "other_tensor": f32}, str(f))
    with SafetensorsLoader(f) as ld:
        meta = ld.get_tensor_metadata()
        ptr, shape, dtype = meta["my_tensor"]
        assert isinstance(ptr, int) and shape == (4,) and dtype == "U8"
        assert _read(ptr, 4) == u8.tobytes()
        ptr, shape, dtype = meta["other_tensor"]
        assert shape == (3,) and dtype == "F32"
        assert _read(ptr, 12) == f32.tobytes()
        np.testing.assert_array_equal(ld.array("other_tensor"), f32)


def test_sharded_directory(tmp_path: Path) -> None:
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    b = np.arange(5, dtype=np.int32)
    save_file({"a": a}, str(tmp_path / "model-00001-of-00002.safetensors"))
    save_file({"b": b}, str(tmp_path / "model-00002-of-00002.safetensors"))
    index = {"weight_map": {"a": "model-00001-of-00002.safetensors", "b": "model-00002-of-00002.safetensors"}}
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps(index))
    ld = auto_loader(tmp_path)
    meta = ld.get_tensor_metadata()
    assert set(meta) == {"a", "b"}
    assert _read(meta["a"][0], a.nbytes) == a.tobytes()
    assert _read(meta["b"][0], b.nbytes) == b.tobytes()
    ld.close()


def test_missing_shard_is_reported(tmp_path: Path) -> None:
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"a": "gone.safetensors"}}))
    with pytest.raises(FileNotFoundError, match="Missing weights file"):
        SafetensorsLoader(tmp_path)


def test_rejects_missing_path_and_empty_directory(tmp_path: Path) -> None:
    with pytest.raises(FileNotFoundError, match=r"No model.safetensors"):
        SafetensorsLoader(tmp_path / "does-not-exist")
    with pytest.raises(FileNotFoundError, match=r"No model.safetensors or index found"):
        SafetensorsLoader(tmp_path)
    with pytest.raises(FileNotFoundError, match="No supported model format"):
        auto_loader(tmp_path)


def test_rejects_byte_ranges_outside_the_file(tmp_path: Path) -> None:
    header = json.dumps({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}).encode()
    f = tmp_path / "model.safetensors"
    f.write_bytes(len(header).to_bytes(8, "little") + header + b"\0" * 8)  # 8 of the 16 bytes
    with pytest.raises(ValueError, match="outside the file"):
        SafetensorsLoader(tmp_path)
    header = json.dumps({"w": {"dtype": "F32", "shape": [3], "data_offsets": [0, 16]}}).encode()
    f.write_bytes(len(header).to_bytes(8, "little") + header + b"\0" * 16)
    with pytest.raises(ValueError, match="holds 16 bytes"):
        SafetensorsLoader(tmp_path)
