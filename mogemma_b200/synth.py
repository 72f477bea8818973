"""Seeded random-init Gemma 3 checkpoints in the reference weight layout.

No checkpoints or datasets are reachable offline, so benchmarks and tests use
synthetic weights: every tensor ~ N(0, std) (std 0.02) from
``numpy.random.default_rng`` with a per-tensor sub-seed derived from the
tensor name, norm weights included (so ``1 + w`` stays near 1).  Names and
``[out, in]`` row-major fp32 layout follow the reference loader
(src/mo/mogemma/core.mojo:79-104, src/py/mogemma/convert.py:92-131);
``lm_head.weight`` is the same array as ``model.embed_tokens.weight`` (tied).
For bf16 configurations the values are rounded to bf16 and kept as their
exact fp32 upcast, so the fp32 oracle sees the very numbers the bf16 device
weights hold.
"""

from __future__ import annotations

import hashlib
import json
import struct
from dataclasses import asdict, dataclass
from pathlib import Path

import numpy as np


@dataclass(frozen=True)
class Gemma3Dims:
    name: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int = 262144
    window: int = 512
    qk_norm: bool = True


CONFIGS: dict[str, Gemma3Dims] = {
    "gemma3-270m": Gemma3Dims("gemma3-270m", 640, 18, 4, 1, 256, 2048, window=512),
    "gemma3-1b": Gemma3Dims("gemma3-1b", 1152, 26, 4, 1, 256, 6912, window=512),
    "embedding-300m": Gemma3Dims("embedding-300m", 768, 24, 3, 1, 256, 1152, window=512),
    "gemma3-4b": Gemma3Dims("gemma3-4b", 2560, 34, 8, 4, 256, 10240, window=1024),
    "gemma3-27b": Gemma3Dims("gemma3-27b", 5376, 62, 32, 16, 128, 21504, window=1024),
}


def tiny(hidden: int = 256, layers: int = 2, heads: int = 4, kv_heads: int = 1, head_dim: int = 64,
         intermediate: int = 512, vocab: int = 4096, window: int = 16, qk_norm: bool = True) -> Gemma3Dims:
    """A small configuration for oracle-speed tests."""
    return Gemma3Dims("tiny", hidden, layers, heads, kv_heads, head_dim, intermediate, vocab, window, qk_norm)


def _subseed(seed: int, name: str) -> int:
    h = hashlib.blake2b(f"{seed}:{name}".encode(), digest_size=8).digest()
    return int.from_bytes(h, "little")


def round_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 (ties to even); returns fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def tensor_shapes(d: Gemma3Dims) -> dict[str, tuple[int, ...]]:
    shapes: dict[str, tuple[int, ...]] = {
        "model.embed_tokens.weight": (d.vocab, d.hidden),
        "model.norm.weight": (d.hidden,),
    }
    q, kv = d.heads * d.head_dim, d.kv_heads * d.head_dim
    for i in range(d.layers):
        p = f"model.layers.{i}."
        shapes[p + "input_layernorm.weight"] = (d.hidden,)
        shapes[p + "post_attention_layernorm.weight"] = (d.hidden,)
        shapes[p + "pre_feedforward_layernorm.weight"] = (d.hidden,)
        shapes[p + "post_feedforward_layernorm.weight"] = (d.hidden,)
        shapes[p + "self_attn.q_proj.weight"] = (q, d.hidden)
        shapes[p + "self_attn.k_proj.weight"] = (kv, d.hidden)
        shapes[p + "self_attn.v_proj.weight"] = (kv, d.hidden)
        shapes[p + "self_attn.o_proj.weight"] = (d.hidden, q)
        if d.qk_norm:
            shapes[p + "self_attn.q_norm.weight"] = (d.head_dim,)
            shapes[p + "self_attn.k_norm.weight"] = (d.head_dim,)
        shapes[p + "mlp.gate_proj.weight"] = (d.intermediate, d.hidden)
        shapes[p + "mlp.up_proj.weight"] = (d.intermediate, d.hidden)
        shapes[p + "mlp.down_proj.weight"] = (d.hidden, d.intermediate)
    return shapes


def make_weights(d: Gemma3Dims, *, seed: int = 0, std: float = 0.02, bf16: bool = False,
                 layers: int | None = None) -> dict[str, np.ndarray]:
    """``{hf_name: float32 ndarray}``; ``lm_head.weight`` aliases the embedding.

    ``layers`` keeps only the first n layers (full-width slices of big models).
    """
    out: dict[str, np.ndarray] = {}
    for name, shape in tensor_shapes(d).items():
        if layers is not None and name.startswith("model.layers."):
            if int(name.split(".")[2]) >= layers:
                continue
        rng = np.random.default_rng(_subseed(seed, name))
        a = rng.standard_normal(shape, dtype=np.float32)
        a *= np.float32(std)
        if bf16:
            a = round_to_bf16(a)
        out[name] = a
    out["lm_head.weight"] = out["model.embed_tokens.weight"]
    return out


@dataclass(frozen=True)
class NanoDims:
    """Gemma 3n ("nano") shapes.  ``kv_share_start``: layers from here on carry zero k/v projections
    and read an earlier layer's cache (src/mo/mogemma/core.mojo:261-273); ``table_layers``: the
    per-layer embedding table's layer count (defaults to ``layers``)."""

    name: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    per_layer_dim: int
    laurel_rank: int
    modalities: int = 4
    vocab: int = 262144
    kv_share_start: int | None = None
    table_layers: int | None = None


def nano_tiny(hidden: int = 64, layers: int = 12, heads: int = 4, kv_heads: int = 2, head_dim: int = 16,
              intermediate: int = 96, per_layer_dim: int = 8, laurel_rank: int = 8, vocab: int = 512,
              kv_share_start: int | None = 8, table_layers: int | None = None) -> NanoDims:
    """A small Gemma 3n configuration for oracle-speed tests (12 layers: sparse and dense MLPs, both
    attention kinds, KV sharing from layer 8)."""
    return NanoDims("nano-tiny", hidden, layers, heads, kv_heads, head_dim, intermediate, per_layer_dim, laurel_rank,
                    4, vocab, kv_share_start, table_layers)


def nano_tensor_shapes(d: NanoDims) -> dict[str, tuple[int, ...]]:
    """Tensor names and shapes the reference's nano loader reads (src/mo/mogemma/core.mojo:111-165)."""
    H, P, T, nm = d.hidden, d.per_layer_dim, d.table_layers or d.layers, d.modalities
    q, kv = d.heads * d.head_dim, d.kv_heads * d.head_dim
    shapes: dict[str, tuple[int, ...]] = {
        "model.embed_tokens.weight": (d.vocab, H),
        "model.norm.weight": (H,),
        "model.per_layer_embed.weight": (d.vocab, T, P),
        "model.per_layer_embed.projection.weight": (H, T, P),
        "model.per_layer_embed.norm.weight": (P,),
    }
    for i in range(nm - 1):
        shapes[f"model.altup.projection.{i}.weight"] = (H, H)
        shapes[f"model.altup.unembed.{i}.weight"] = (H, H)
    for i in range(d.layers):
        p = f"model.layers.{i}."
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            shapes[p + n + ".weight"] = (H,)
        shapes[p + "self_attn.q_proj.weight"] = (q, H)
        shapes[p + "self_attn.k_proj.weight"] = (kv, H)
        shapes[p + "self_attn.v_proj.weight"] = (kv, H)
        shapes[p + "self_attn.o_proj.weight"] = (H, q)
        shapes[p + "self_attn.q_norm.weight"] = (d.head_dim,)
        shapes[p + "self_attn.k_norm.weight"] = (d.head_dim,)
        shapes[p + "mlp.gate_proj.weight"] = (d.intermediate, H)
        shapes[p + "mlp.up_proj.weight"] = (d.intermediate, H)
        shapes[p + "mlp.down_proj.weight"] = (H, d.intermediate)
        shapes[p + "altup.router.weight"] = (nm, H)
        shapes[p + "altup.router_norm.weight"] = (H,)
        shapes[p + "altup.prediction_coefs"] = (nm, nm, nm)
        shapes[p + "altup.correction_coefs"] = (nm, nm)
        shapes[p + "altup.output_scale"] = (H,)
        shapes[p + "laurel.down_proj.weight"] = (d.laurel_rank, H)
        shapes[p + "laurel.up_proj.weight"] = (H, d.laurel_rank)
        shapes[p + "laurel.norm.weight"] = (H,)
        shapes[p + "per_layer_map.gate.weight"] = (P, H)
        shapes[p + "per_layer_map.projection.weight"] = (H, P)
        shapes[p + "per_layer_map.norm.weight"] = (H,)
    return shapes


def make_nano_weights(d: NanoDims, *, seed: int = 0, std: float = 0.02,
                      scales: dict[str, float] | None = None) -> dict[str, np.ndarray]:
    """Seeded Gemma 3n weights: N(0, std) matrices, norm weights and AltUp output scales 1 + N(0, std)
    (the nano norms multiply by the weight itself), k/v projections of layers from kv_share_start on
    zero; ``lm_head.weight`` aliases the embedding.  ``scales`` multiplies the noise of tensors whose
    name contains a key (e.g. larger AltUp coefficients)."""
    out: dict[str, np.ndarray] = {}
    for name, shape in nano_tensor_shapes(d).items():
        rng = np.random.default_rng(_subseed(seed, name))
        k = np.float32(std * next((v for key, v in (scales or {}).items() if key in name), 1.0))
        a = rng.standard_normal(shape, dtype=np.float32) * k
        if name.endswith("norm.weight") or name.endswith("output_scale"):
            a += np.float32(1.0)
        layer = int(name.split(".")[2]) if name.startswith("model.layers.") else -1
        if d.kv_share_start is not None and layer >= d.kv_share_start and (
                name.endswith("k_proj.weight") or name.endswith("v_proj.weight")):
            a[...] = 0.0
        out[name] = a
    out["lm_head.weight"] = out["model.embed_tokens.weight"]
    return out


def metadata_of(weights: dict[str, np.ndarray]) -> dict[str, tuple[int, tuple[int, ...], str]]:
    """Loader-style ``{name: (ptr, shape, dtype)}`` over in-memory arrays."""
    return {k: (int(v.ctypes.data), tuple(v.shape), "F32") for k, v in weights.items()}


def prompt_ids(n: int, vocab: int, *, seed: int = 1) -> np.ndarray:
    """Uniform random prompt ids in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)


def write_safetensors(weights: dict[str, np.ndarray], path: Path, *, dims: Gemma3Dims | None = None) -> Path:
    """Write fp32 safetensors (HF names) to ``path``/model.safetensors."""
    path.mkdir(parents=True, exist_ok=True)
    header: dict[str, object] = {}
    off = 0
    order = sorted(weights)
    for k in order:
        n = weights[k].nbytes
        header[k] = {"dtype": "F32", "shape": list(weights[k].shape), "data_offsets": [off, off + n]}
        off += n
    if dims is not None:
        header["__metadata__"] = {k: str(v) for k, v in asdict(dims).items()}
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with (path / "model.safetensors").open("wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for k in order:
            f.write(np.ascontiguousarray(weights[k], dtype=np.float32).tobytes())
    return path
