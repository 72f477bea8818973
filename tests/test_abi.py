"""The C-ABI library loads, exports every entry point include/*.h declares,
and the ctypes mirrors of its structs match the C layout (no GPU needed)."""

from __future__ import annotations

import re
import subprocess
from pathlib import Path

import pytest

from mogemma_b200 import _core

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "mogemma_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mg_[a-z_0-9]+)\s*\(", text)))


def test_header_declares_entry_points() -> None:
    names = declared_functions()
    for n in ("mg_model_create", "mg_step", "mg_prefill", "mg_generate", "mg_sample", "mg_embed",
              "mg_model_destroy", "mg_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol() -> None:
    lib = _core.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"
    assert lib.mg_abi_version() == 1


def test_struct_layout_matches_header(tmp_path: Path) -> None:
    src = tmp_path / "sizes.c"
    src.write_text(
        '#include <stdio.h>\n#include <stddef.h>\n#include "mogemma_b200.h"\n'
        "int main(void){printf(\"%zu %zu %zu %zu %zu %zu %zu %zu %zu\\n\", sizeof(mg_tensor_desc), sizeof(mg_options),"
        " sizeof(mg_model_info), sizeof(mg_sampling), offsetof(mg_options, seed), offsetof(mg_options, reserved1),"
        " offsetof(mg_sampling, uniforms_host), offsetof(mg_options, synthetic_seed), sizeof(mg_nano_info));"
        " return 0;}\n")
    exe = tmp_path / "sizes"
    try:
        subprocess.run(["gcc", "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    except (FileNotFoundError, subprocess.CalledProcessError):
        pytest.skip("no C compiler")
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    import ctypes  # noqa: PLC0415

    want = [ctypes.sizeof(_core.TensorDesc), ctypes.sizeof(_core.Options), ctypes.sizeof(_core.ModelInfo),
            ctypes.sizeof(_core.Sampling), _core.Options.seed.offset, _core.Options.reserved1.offset,
            _core.Sampling.uniforms_host.offset, _core.Options.synthetic_seed.offset, ctypes.sizeof(_core.NanoInfo)]
    assert got == want


def test_create_without_tensors_fails_cleanly() -> None:
    import ctypes  # noqa: PLC0415

    out = ctypes.c_void_p()
    st = _core.lib().mg_model_create(None, 0, None, ctypes.byref(out))
    assert st == _core.MG_ERR_INVALID
    assert b"no tensors" in _core.lib().mg_last_error()


def test_nano_create_rejects_bad_input_without_a_device() -> None:
    """mg_nano_create checks its arguments and the checkpoint kind before any CUDA call."""
    import ctypes  # noqa: PLC0415

    out = ctypes.c_void_p()
    lib = _core.lib()
    assert lib.mg_nano_create(None, 0, 0, 64, ctypes.byref(out)) == _core.MG_ERR_INVALID
    descs, _keep = _core._tensor_descs({"model.embed_tokens.weight": (1, (4, 2), "F32")})  # noqa: SLF001
    assert lib.mg_nano_create(descs, len(descs), 0, 64, ctypes.byref(out)) == _core.MG_ERR_INVALID
    assert b"not a Gemma 3n checkpoint" in lib.mg_last_error()
    assert not out.value
