"""Gemma 3 checkpoints from the Orbax layout into HuggingFace-named safetensors.

The reference's one-time conversion (src/py/mogemma/convert.py:124-149, the
standard Gemma 3 path) turns the Orbax tree that Google distributes into the
tensor names and ``[out, in]`` float32 layout its engine -- and this one --
consume.  The rules are restated here as a table: each Orbax tensor of a layer
maps to one or more HuggingFace tensors through a fixed reshape/transpose:

===========================================  ==========================================  ============================
Orbax (``transformer/layer_{n}/...``)         HuggingFace (``model.layers.{n}....``)      layout change
===========================================  ==========================================  ============================
``pre_attention_norm.scale``                  ``input_layernorm.weight``                  --
``post_attention_norm.scale``                 ``post_attention_layernorm.weight``         --
``pre_ffw_norm.scale``                        ``pre_feedforward_layernorm.weight``        --
``post_ffw_norm.scale``                       ``post_feedforward_layernorm.weight``       --
``attn/_query_norm.scale``                    ``self_attn.q_norm.weight``                 --
``attn/_key_norm.scale``                      ``self_attn.k_norm.weight``                 --
``attn/q_einsum.w`` [heads, hidden, hd]       ``self_attn.q_proj.weight`` [heads*hd, hidden]  per head transpose
``attn/kv_einsum.w`` [2, kv, hidden, hd]      ``self_attn.{k,v}_proj.weight`` [kv*hd, hidden]  split, per head transpose
``attn/attn_vec_einsum.w`` [heads, hd, hid]   ``self_attn.o_proj.weight`` [hidden, heads*hd]  flatten heads, transpose
``mlp/gating_einsum.w`` [2, inter, hidden]    ``mlp.{gate,up}_proj.weight`` [inter, hidden]   split
``mlp/linear.w`` [inter, hidden]              ``mlp.down_proj.weight`` [hidden, inter]        transpose
===========================================  ==========================================  ============================

plus ``transformer/embedder.input_embedding`` -> ``model.embed_tokens.weight``
and its tied copy ``lm_head.weight``, and ``transformer/final_norm.scale`` ->
``model.norm.weight``.  Every output is float32 (bf16 sources are widened).

The converter reads from any mapping of Orbax names to arrays and writes the
safetensors file tensor by tensor, so no more than one converted tensor is in
memory at a time.  Reading an Orbax/OCDBT directory itself needs
``tensorstore``; :func:`read_orbax` says so when it is missing.  Gemma 3n
(nano) checkpoints are not handled: the B200 engine runs the standard family.
"""

from __future__ import annotations

import json
import re
import struct
from collections.abc import Callable, Iterable, Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np

_LAYER = re.compile(r"^transformer/layer_(\d+)/(.+)$")

Array = Any  # numpy-compatible array (np.ndarray or a lazily read tensor)


@dataclass(frozen=True)
class _Rule:
    """One HuggingFace tensor of a layer: its name, Orbax source and reshaping."""

    hf: str
    src: str
    fn: Callable[[np.ndarray], np.ndarray]
    shape: Callable[[tuple[int, ...]], tuple[int, ...]]


def _heads_to_rows(a: np.ndarray) -> np.ndarray:  # [h, hidden, hd] -> [h*hd, hidden]
    return a.transpose(0, 2, 1).reshape(-1, a.shape[1])


def _rows_shape(s: tuple[int, ...]) -> tuple[int, ...]:
    return (s[0] * s[2], s[1])


_LAYER_RULES: tuple[_Rule, ...] = (
    _Rule("input_layernorm.weight", "pre_attention_norm.scale", lambda a: a, lambda s: s),
    _Rule("post_attention_layernorm.weight", "post_attention_norm.scale", lambda a: a, lambda s: s),
    _Rule("pre_feedforward_layernorm.weight", "pre_ffw_norm.scale", lambda a: a, lambda s: s),
    _Rule("post_feedforward_layernorm.weight", "post_ffw_norm.scale", lambda a: a, lambda s: s),
    _Rule("self_attn.q_norm.weight", "attn/_query_norm.scale", lambda a: a, lambda s: s),
    _Rule("self_attn.k_norm.weight", "attn/_key_norm.scale", lambda a: a, lambda s: s),
    _Rule("self_attn.q_proj.weight", "attn/q_einsum.w", _heads_to_rows, _rows_shape),
    _Rule("self_attn.k_proj.weight", "attn/kv_einsum.w", lambda a: _heads_to_rows(a[0]), lambda s: _rows_shape(s[1:])),
    _Rule("self_attn.v_proj.weight", "attn/kv_einsum.w", lambda a: _heads_to_rows(a[1]), lambda s: _rows_shape(s[1:])),
    _Rule("self_attn.o_proj.weight", "attn/attn_vec_einsum.w", lambda a: a.reshape(-1, a.shape[2]).T,
          lambda s: (s[2], s[0] * s[1])),
    _Rule("mlp.gate_proj.weight", "mlp/gating_einsum.w", lambda a: a[0], lambda s: s[1:]),
    _Rule("mlp.up_proj.weight", "mlp/gating_einsum.w", lambda a: a[1], lambda s: s[1:]),
    _Rule("mlp.down_proj.weight", "mlp/linear.w", lambda a: a.T, lambda s: (s[1], s[0])),
)
_GLOBAL_RULES: tuple[_Rule, ...] = (
    _Rule("model.embed_tokens.weight", "transformer/embedder.input_embedding", lambda a: a, lambda s: s),
    _Rule("lm_head.weight", "transformer/embedder.input_embedding", lambda a: a, lambda s: s),  # tied
    _Rule("model.norm.weight", "transformer/final_norm.scale", lambda a: a, lambda s: s),
)


def detect_family(names: Iterable[str]) -> str:
    """``"gemma3"`` for the standard family, ``"gemma3_nano"`` for Gemma 3n
    (AltUp / per-layer-mapping tensors present)."""
    for n in names:
        if "altup" in n or "per_layer_mapping" in n:
            return "gemma3_nano"
    return "gemma3"


def _layers(names: Iterable[str]) -> list[int]:
    found = set()
    for n in names:
        m = _LAYER.match(n)
        if m:
            found.add(int(m.group(1)))
    return sorted(found)


def plan(orbax: Mapping[str, Array]) -> list[tuple[str, str, _Rule]]:
    """The conversion as (HuggingFace name, Orbax name, rule) in output order.

    Raises ValueError for a Gemma 3n checkpoint and KeyError naming the first
    Orbax tensor a rule needs but the checkpoint lacks."""
    names = list(orbax.keys())
    if detect_family(names) != "gemma3":
        msg = "Gemma 3n (nano) checkpoints are not supported by the B200 engine"
        raise ValueError(msg)
    out = [(r.hf, r.src, r) for r in _GLOBAL_RULES]
    for n in _layers(names):
        out += [(f"model.layers.{n}.{r.hf}", f"transformer/layer_{n}/{r.src}", r) for r in _LAYER_RULES]
    missing = next((src for _, src, _r in out if src not in orbax), None)
    if missing is not None:
        msg = f"Key not found in Orbax checkpoint: {missing}"
        raise KeyError(msg)
    return out


def convert_tensors(orbax: Mapping[str, Array]) -> dict[str, np.ndarray]:
    """All HuggingFace tensors in memory ({name: float32 array}); the embedding
    and lm_head are the same array, as the reference's tied weights are."""
    out: dict[str, np.ndarray] = {}
    for hf, src, rule in plan(orbax):
        if hf == "lm_head.weight":
            out[hf] = out["model.embed_tokens.weight"]
            continue
        out[hf] = np.ascontiguousarray(rule.fn(np.asarray(orbax[src])), dtype=np.float32)
    return out


def write_safetensors(orbax: Mapping[str, Array], path: str | Path) -> Path:
    """Convert and write ``path`` (a ``.safetensors`` file, or a directory that
    receives ``model.safetensors``) one tensor at a time."""
    path = Path(path)
    if path.suffix != ".safetensors":
        path.mkdir(parents=True, exist_ok=True)
        path = path / "model.safetensors"
    steps = plan(orbax)
    header: dict[str, Any] = {}
    off = 0
    for hf, src, rule in steps:
        shape = rule.shape(tuple(int(x) for x in np.shape(orbax[src])))
        nbytes = int(np.prod(shape, dtype=np.int64)) * 4
        header[hf] = {"dtype": "F32", "shape": list(shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    blob = json.dumps(header, separators=(",", ":")).encode()
    blob += b" " * (-len(blob) % 8)
    with path.open("wb") as f:
        f.write(struct.pack("<Q", len(blob)))
        f.write(blob)
        for hf, src, rule in steps:
            a = np.ascontiguousarray(rule.fn(np.asarray(orbax[src])), dtype=np.float32)
            if list(a.shape) != header[hf]["shape"]:
                msg = f"{hf}: converted shape {a.shape} differs from the planned {header[hf]['shape']}"
                raise ValueError(msg)
            f.write(a.tobytes())
    return path


def read_orbax(checkpoint_dir: str | Path) -> Mapping[str, Array]:
    """Lazily read Orbax tensors of ``checkpoint_dir`` by name.

    The checkpoint keeps Zarr arrays in an OCDBT key-value store under
    ``ocdbt.process_0``; reading it needs ``tensorstore``, which this engine
    does not depend on (without it this raises ModuleNotFoundError)."""
    try:
        import tensorstore as ts  # type: ignore[import-not-found]  # noqa: PLC0415
    except ModuleNotFoundError as exc:
        msg = "reading Orbax/OCDBT checkpoints needs the 'tensorstore' package"
        raise ModuleNotFoundError(msg) from exc
    kvstore = {"driver": "ocdbt", "base": f"file://{Path(checkpoint_dir) / 'ocdbt.process_0'}"}
    keys = ts.KvStore.open(kvstore).result().list().result()
    names = sorted({k.decode().rsplit("/", 1)[0] for k in keys if k.decode().endswith("/.zarray")})
    if not names:
        msg = f"No tensors found in OCDBT checkpoint at {checkpoint_dir}"
        raise FileNotFoundError(msg)

    class _Lazy(Mapping[str, Array]):
        def __getitem__(self, name: str) -> Array:
            if name not in names:
                raise KeyError(name)
            # an open store: its shape is known without reading; np.asarray reads it
            return ts.open({"driver": "zarr", "kvstore": kvstore, "path": name}).result()

        def __iter__(self):  # noqa: ANN204
            return iter(names)

        def __len__(self) -> int:
            return len(names)

    return _Lazy()


def convert_orbax_to_safetensors(checkpoint_dir: str | Path, out_dir: str | Path | None = None) -> Path:
    """Convert the Orbax checkpoint in ``checkpoint_dir`` into
    ``out_dir/model.safetensors`` (default: the checkpoint directory)."""
    return write_safetensors(read_orbax(checkpoint_dir), Path(out_dir or checkpoint_dir))
