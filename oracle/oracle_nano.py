"""Oracle for the Gemma 3n ("nano") decode path (TEST INFRASTRUCTURE).

Drives ``ref_nano.c`` (inside ``libmg_oracle.so``), the C restatement of
``src/mo/mogemma/layers.mojo:121-171, 373-1063``.  Dimension inference and the
arch / kv_share_start keys follow ``init_model_mojo``'s nano branch
(``src/mo/mogemma/core.mojo:296-312``).  Only ``tests/`` import this module.
"""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np
import numpy.typing as npt

import oracle

_F = ctypes.POINTER(ctypes.c_float)
_I32 = ctypes.POINTER(ctypes.c_int32)

_BASE = ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm", "post_feedforward_layernorm",
         "q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj", "q_norm", "k_norm")
_ALTUP = ("router", "router_norm", "prediction_coefs", "correction_coefs", "output_scale")


class NanoLayerW(ctypes.Structure):
    _fields_ = ([(n, _F) for n in _BASE] + [(n, _F) for n in _ALTUP]
                + [("laurel_down", _F), ("laurel_up", _F), ("laurel_norm", _F), ("laurel_rank", ctypes.c_int64),
                   ("plm_gate", _F), ("plm_projection", _F), ("plm_norm", _F)])


# reference tensor name of each NanoLayerW pointer field (core.mojo:136-164)
_LAYER_NAMES = {
    "input_layernorm": "input_layernorm.weight", "post_attention_layernorm": "post_attention_layernorm.weight",
    "pre_feedforward_layernorm": "pre_feedforward_layernorm.weight",
    "post_feedforward_layernorm": "post_feedforward_layernorm.weight",
    "q_proj": "self_attn.q_proj.weight", "k_proj": "self_attn.k_proj.weight", "v_proj": "self_attn.v_proj.weight",
    "o_proj": "self_attn.o_proj.weight", "gate_proj": "mlp.gate_proj.weight", "up_proj": "mlp.up_proj.weight",
    "down_proj": "mlp.down_proj.weight", "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight",
    "router": "altup.router.weight", "router_norm": "altup.router_norm.weight",
    "prediction_coefs": "altup.prediction_coefs", "correction_coefs": "altup.correction_coefs",
    "output_scale": "altup.output_scale", "laurel_down": "laurel.down_proj.weight",
    "laurel_up": "laurel.up_proj.weight", "laurel_norm": "laurel.norm.weight",
    "plm_gate": "per_layer_map.gate.weight", "plm_projection": "per_layer_map.projection.weight",
    "plm_norm": "per_layer_map.norm.weight",
}

_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        L = oracle.lib()
        i64, i32, flt, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p
        W = ctypes.POINTER(NanoLayerW)
        L.ref_nano_laurel.argtypes = [_F, _F, _F, _F, _F, i64, i64]
        L.ref_nano_per_layer_mapping.argtypes = [_F, _F, _F, _F, _F, _F, i64, i64]
        L.ref_nano_altup_predict.argtypes = [_F, _F, W, i64, i32]
        L.ref_nano_altup_correct.argtypes = [_F, _F, _F, W, i64, i32]
        L.ref_nano_activation_sparsity.argtypes = [_F, i64, flt]
        L.ref_nano_layer.argtypes = [_F, _F, W, i32, _F, i64, i64, i64, i64, i64, i64, i64, _F, _F, _F, _F, i32, i32]
        L.ref_nano_create.restype = vp
        L.ref_nano_create.argtypes = [_F, _F, _F, _F, _F, _F, ctypes.POINTER(_F), ctypes.POINTER(_F), W, i32, i64, i64,
                                      i64, i64, i64, i64, i64, i64, i32, i64]
        L.ref_nano_destroy.argtypes = [vp]
        L.ref_nano_kv_share_start.restype = i64
        L.ref_nano_kv_share_start.argtypes = [vp]
        L.ref_nano_pos.restype = i64
        L.ref_nano_pos.argtypes = [vp]
        L.ref_nano_set_pos.argtypes = [vp, i64]
        L.ref_nano_k_cache.restype = _F
        L.ref_nano_k_cache.argtypes = [vp]
        L.ref_nano_step.restype = ctypes.c_int
        L.ref_nano_step.argtypes = [vp, i32, _F]
        L.ref_nano_embed_sequence.argtypes = [vp, _I32, i64, _F]
        _lib = L
    return _lib


def _f32(a: Any) -> npt.NDArray[np.float32]:
    return np.ascontiguousarray(a, dtype=np.float32)


def _fp(a: npt.NDArray[np.float32] | None) -> Any:
    return oracle._fp(a)  # noqa: SLF001


def layer_struct(arrays: dict[str, np.ndarray], laurel_rank: int | None = None) -> tuple[NanoLayerW, list]:
    """A NanoLayerW over ``{field: array}`` (missing fields stay NULL); returns it with the arrays it points at."""
    keep: list = []
    w = NanoLayerW()
    for field, _t in NanoLayerW._fields_:
        if field == "laurel_rank":
            continue
        a = arrays.get(field)
        if a is not None:
            a = _f32(a)
            keep.append(a)
            setattr(w, field, _fp(a))
    if laurel_rank is None and arrays.get("laurel_down") is not None:
        laurel_rank = int(np.asarray(arrays["laurel_down"]).shape[0])
    w.laurel_rank = int(laurel_rank or 0)
    return w, keep


# ---------------------------------------------------------------- components
def laurel(x: np.ndarray, down: np.ndarray, up: np.ndarray, norm: np.ndarray) -> np.ndarray:
    x, down, up, norm = map(_f32, (x, down, up, norm))
    out = np.zeros(x.shape[0], np.float32)
    lib().ref_nano_laurel(_fp(out), _fp(x), _fp(down), _fp(up), _fp(norm), x.shape[0], down.shape[0])
    return out


def per_layer_mapping(active: np.ndarray, per_layer_input: np.ndarray, gate: np.ndarray, projection: np.ndarray,
                      norm: np.ndarray) -> np.ndarray:
    active, pli, gate, projection, norm = map(_f32, (active, per_layer_input, gate, projection, norm))
    out = np.zeros(active.shape[0], np.float32)
    lib().ref_nano_per_layer_mapping(_fp(out), _fp(active), _fp(pli), _fp(gate), _fp(projection), _fp(norm),
                                     active.shape[0], gate.shape[0])
    return out


def altup_predict(streams: np.ndarray, altup: dict[str, np.ndarray]) -> np.ndarray:
    streams = _f32(streams)
    nm, h = streams.shape
    w, _keep = layer_struct(altup)
    out = np.zeros_like(streams)
    lib().ref_nano_altup_predict(_fp(out), _fp(streams), ctypes.byref(w), h, nm)
    return out


def altup_correct(predictions: np.ndarray, activated: np.ndarray, altup: dict[str, np.ndarray]) -> np.ndarray:
    predictions, activated = _f32(predictions), _f32(activated)
    nm, h = predictions.shape
    w, _keep = layer_struct(altup)
    out = np.zeros_like(predictions)
    lib().ref_nano_altup_correct(_fp(out), _fp(predictions), _fp(activated), ctypes.byref(w), h, nm)
    return out


def activation_sparsity(gate: np.ndarray, sparsity: float = 0.95) -> np.ndarray:
    g = _f32(gate).copy()
    lib().ref_nano_activation_sparsity(_fp(g), g.shape[0], sparsity)
    return g


# ---------------------------------------------------------------- the model
def _layer_count(weights: dict[str, np.ndarray]) -> int:
    n = 0
    while f"model.layers.{n}.input_layernorm.weight" in weights:  # core.mojo:131-135
        n += 1
    return n


class NanoRefModel:
    """The reference's nano ``init_model`` + ``step`` on the C oracle.

    ``info`` holds the keys ``init_model_mojo`` returns for arch "nano" (core.mojo:296-361)."""

    def __init__(self, weights: dict[str, np.ndarray], max_seq_len: int = 256) -> None:
        self._keep: list = []

        def get(name: str) -> npt.NDArray[np.float32] | None:
            a = weights.get(name)
            if a is None:
                return None
            a = _f32(a)
            self._keep.append(a)
            return a

        L = _layer_count(weights)
        if L == 0:
            raise ValueError("Invalid Nano model weights: no layers found in metadata")
        p0 = "model.layers.0."
        qn = weights.get(p0 + "self_attn.q_norm.weight")
        hd = int(qn.shape[0]) if qn is not None else 256
        embed = get("model.embed_tokens.weight")
        lm_head = get("lm_head.weight")
        assert embed is not None and lm_head is not None
        hidden = int(embed.shape[1])
        nkv = int(weights[p0 + "self_attn.k_proj.weight"].shape[0]) // hd
        nq = int(weights[p0 + "self_attn.q_proj.weight"].shape[0]) // hd
        inter = int(weights[p0 + "mlp.gate_proj.weight"].shape[0])
        vocab = int(lm_head.shape[0])
        pld = int(weights[p0 + "per_layer_map.gate.weight"].shape[0])
        if pld <= 0:
            raise ValueError("Invalid Nano model weights: per_layer_map gate dim must be > 0")
        nm = int(weights[p0 + "altup.router.weight"].shape[0])
        ple = get("model.per_layer_embed.weight")
        assert ple is not None
        table_layers = int(ple.shape[1])
        structs = (NanoLayerW * L)()
        for i in range(L):
            arrays = {f: get(f"model.layers.{i}.{n}") for f, n in _LAYER_NAMES.items()}
            w, keep = layer_struct({k: v for k, v in arrays.items() if v is not None})
            self._keep.extend(keep)
            structs[i] = w
        proj = (_F * max(1, nm - 1))()
        unemb = (_F * max(1, nm - 1))()
        for i in range(nm - 1):  # core.mojo:118-124 reads projection/unembed 0..2
            proj[i] = _fp(get(f"model.altup.projection.{i}.weight"))
            unemb[i] = _fp(get(f"model.altup.unembed.{i}.weight"))
        self._structs = structs
        self._ptr = lib().ref_nano_create(
            _fp(embed), _fp(get("model.norm.weight")), _fp(lm_head), _fp(ple),
            _fp(get("model.per_layer_embed.projection.weight")), _fp(get("model.per_layer_embed.norm.weight")),
            proj, unemb, structs, L, hidden, nq, nkv, hd, inter, vocab, pld, table_layers, nm, max_seq_len)
        if not self._ptr:
            raise ValueError("unsupported nano configuration")
        self.vocab = vocab
        self.hidden = hidden
        self.info = {"arch": "nano", "num_layers": L, "num_kv_heads": nkv, "head_dim": hd, "hidden_size": hidden,
                     "intermediate_size": inter, "vocab_size": vocab, "per_layer_dim": pld,
                     "kv_share_start": int(lib().ref_nano_kv_share_start(self._ptr)), "max_seq_len": max_seq_len}

    def __del__(self) -> None:
        if getattr(self, "_ptr", None):
            lib().ref_nano_destroy(self._ptr)
            self._ptr = None

    @property
    def pos(self) -> int:
        return int(lib().ref_nano_pos(self._ptr))

    @pos.setter
    def pos(self, v: int) -> None:
        lib().ref_nano_set_pos(self._ptr, int(v))

    def step(self, token_id: int) -> npt.NDArray[np.float32]:
        out = np.zeros(self.vocab, np.float32)
        if lib().ref_nano_step(self._ptr, int(token_id), _fp(out)) != 0:
            raise RuntimeError("Sequence length exceeded")
        return out

    def step_no_logits(self, token_id: int) -> None:
        if lib().ref_nano_step(self._ptr, int(token_id), ctypes.cast(None, _F)) != 0:
            raise RuntimeError("Sequence length exceeded")

    def embed(self, ids: list[int]) -> npt.NDArray[np.float32]:
        a = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(self.hidden, np.float32)
        lib().ref_nano_embed_sequence(self._ptr, a.ctypes.data_as(_I32), a.shape[0], _fp(out))
        return out
