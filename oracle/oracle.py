"""Oracle: CPU restatement of the MoGemma reference engine (TEST INFRASTRUCTURE).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this module, and only as the checker.  The product path
(``mogemma_b200``) never imports it.

* :class:`RefModel` drives ``libmg_oracle.so`` (``ref_cpu.c``), the C restatement
  of ``src/mo/mogemma/{ops,layers,core}.mojo``.  Dimension inference follows
  ``init_model_mojo`` (``src/mo/mogemma/core.mojo:316-325``).
* :func:`sample_next_token` restates ``_sample_next_token``
  (``src/py/mogemma/model.py:103-150``) with the uniform variate passed in,
  so the categorical draw is reproducible.  NumPy's ``Generator.choice(n, p=p)``
  draws one uniform ``u`` and returns ``searchsorted(cumsum(p)/sum, u, 'right')``.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np
import numpy.typing as npt

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "libmg_oracle.so"
_lib: ctypes.CDLL | None = None

_F = ctypes.POINTER(ctypes.c_float)
_I32 = ctypes.POINTER(ctypes.c_int32)


class _LayerW(ctypes.Structure):
    _fields_ = [
        (n, _F)
        for n in (
            "input_layernorm",
            "post_attention_layernorm",
            "q_proj",
            "k_proj",
            "v_proj",
            "o_proj",
            "gate_proj",
            "up_proj",
            "down_proj",
            "q_norm",
            "k_norm",
            "pre_feedforward_layernorm",
            "post_feedforward_layernorm",
        )
    ]


def build() -> Path:
    """Compile ``libmg_oracle.so`` from ``ref_cpu.c`` (gcc)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        i64, i32, flt = ctypes.c_int64, ctypes.c_int32, ctypes.c_float
        L.ref_geglu.argtypes = [_F, _F, _F, i64, ctypes.c_int]
        L.ref_rope_rotate.argtypes = [_F, _F, _F, i64, ctypes.c_int]
        L.ref_vec_mat_mul.argtypes = [_F, _F, _F, i64, i64, ctypes.c_int]
        L.ref_rms_norm.argtypes = [_F, _F, _F, i64, flt, ctypes.c_int]
        L.ref_softmax.argtypes = [_F, i64, ctypes.c_int]
        L.ref_rope_tables.argtypes = [_F, _F, i64, i64, flt]
        L.ref_model_create.restype = ctypes.c_void_p
        L.ref_model_create.argtypes = [_F, _F, _F, ctypes.POINTER(_LayerW), i32, i64, i64, i64, i64, i64, i64, i64,
                                       i32, i32, i32, flt, flt]
        L.ref_model_destroy.argtypes = [ctypes.c_void_p]
        L.ref_model_pos.restype = i64
        L.ref_model_pos.argtypes = [ctypes.c_void_p]
        L.ref_model_set_pos.argtypes = [ctypes.c_void_p, i64]
        L.ref_step.restype = ctypes.c_int
        L.ref_step.argtypes = [ctypes.c_void_p, i32, _F]
        L.ref_step_no_logits.restype = ctypes.c_int
        L.ref_step_no_logits.argtypes = [ctypes.c_void_p, i32]
        L.ref_embed_sequence.argtypes = [ctypes.c_void_p, _I32, i64, _F, ctypes.c_int]
        L.ref_encode_sequence.argtypes = [ctypes.c_void_p, _I32, i64, _F, i64, _F, _F]
        L.ref_encode_sequence.restype = ctypes.c_int
        L.ref_model_k_cache.restype = _F
        L.ref_model_k_cache.argtypes = [ctypes.c_void_p]
        L.ref_model_v_cache.restype = _F
        L.ref_model_v_cache.argtypes = [ctypes.c_void_p]
        L.ref_forward_attention_raw.argtypes = [_F, _F, ctypes.POINTER(_LayerW), i64, i64, i64, i64, i64, _F, _F,
                                                _F, _F, _F]
        L.ref_forward_mlp_raw.argtypes = [_F, _F, ctypes.POINTER(_LayerW), i64, i64, _F]
        L.ref_forward_layer_raw.argtypes = [_F, _F, ctypes.POINTER(_LayerW), i64, i64, i64, i64, i64, i64, _F, _F,
                                            _F, _F, _F]
        L.ref_set_threads.argtypes = [ctypes.c_int]
        L.ref_get_threads.restype = ctypes.c_int
        _lib = L
    return _lib


def _fp(a: npt.NDArray[np.float32] | None) -> ctypes._Pointer:  # type: ignore[type-arg]
    if a is None:
        return ctypes.cast(None, _F)
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], "oracle needs C-contiguous float32"
    return a.ctypes.data_as(_F)


def set_threads(n: int) -> None:
    lib().ref_set_threads(int(n))


# ---------------------------------------------------------------- op level
def vec_mat_mul(x: np.ndarray, w: np.ndarray, nelts: int = 16) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros(w.shape[0], np.float32)
    lib().ref_vec_mat_mul(_fp(out), _fp(x), _fp(w), w.shape[1], w.shape[0], nelts)
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6, nelts: int = 16) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib().ref_rms_norm(_fp(out), _fp(x), _fp(w), x.size, eps, nelts)
    return out


def softmax(x: np.ndarray, nelts: int = 16) -> np.ndarray:
    v = np.array(x, np.float32, copy=True)
    lib().ref_softmax(_fp(v), v.size, nelts)
    return v


def geglu(gate: np.ndarray, up: np.ndarray, nelts: int = 16) -> np.ndarray:
    g = np.ascontiguousarray(gate, np.float32)
    u = np.ascontiguousarray(up, np.float32)
    out = np.zeros_like(g)
    lib().ref_geglu(_fp(out), _fp(g), _fp(u), g.size, nelts)
    return out


def rope_rotate(vec: np.ndarray, cos: np.ndarray, sin: np.ndarray, nelts: int = 16) -> np.ndarray:
    v = np.array(vec, np.float32, copy=True)
    c = np.ascontiguousarray(cos, np.float32)
    s = np.ascontiguousarray(sin, np.float32)
    lib().ref_rope_rotate(_fp(v), _fp(c), _fp(s), v.size, nelts)
    return v


def rope_tables(max_seq_len: int, head_dim: int, base: float = 10000.0) -> tuple[np.ndarray, np.ndarray]:
    c = np.zeros(max_seq_len * head_dim, np.float32)
    s = np.zeros(max_seq_len * head_dim, np.float32)
    lib().ref_rope_tables(_fp(c), _fp(s), max_seq_len, head_dim, base)
    return c, s


LAYER_KEYS = (
    ("input_layernorm", "input_layernorm.weight"),
    ("post_attention_layernorm", "post_attention_layernorm.weight"),
    ("q_proj", "self_attn.q_proj.weight"),
    ("k_proj", "self_attn.k_proj.weight"),
    ("v_proj", "self_attn.v_proj.weight"),
    ("o_proj", "self_attn.o_proj.weight"),
    ("gate_proj", "mlp.gate_proj.weight"),
    ("up_proj", "mlp.up_proj.weight"),
    ("down_proj", "mlp.down_proj.weight"),
    ("q_norm", "self_attn.q_norm.weight"),
    ("k_norm", "self_attn.k_norm.weight"),
    ("pre_feedforward_layernorm", "pre_feedforward_layernorm.weight"),
    ("post_feedforward_layernorm", "post_feedforward_layernorm.weight"),
)


def layer_struct(arrs: dict[str, np.ndarray | None]) -> _LayerW:
    lw = _LayerW()
    for field, _ in LAYER_KEYS:
        setattr(lw, field, _fp(arrs.get(field)))
    return lw


def forward_attention_raw(x, w: dict, pos, hidden, nh, nkv, hd, cos_t, sin_t, k_cache, v_cache) -> np.ndarray:
    out = np.zeros(hidden, np.float32)
    scratch = np.zeros(hidden * 64 + 4 * nh * hd + 4 * nkv * hd + pos + 64, np.float32)
    lw = layer_struct(w)
    lib().ref_forward_attention_raw(_fp(out), _fp(np.ascontiguousarray(x, np.float32)), ctypes.byref(lw), pos,
                                    hidden, nh, nkv, hd, _fp(cos_t), _fp(sin_t), _fp(k_cache), _fp(v_cache),
                                    _fp(scratch))
    return out


def forward_mlp_raw(x, w: dict, hidden, inter) -> np.ndarray:
    out = np.zeros(hidden, np.float32)
    scratch = np.zeros(inter * 4 + 64, np.float32)
    lw = layer_struct(w)
    lib().ref_forward_mlp_raw(_fp(out), _fp(np.ascontiguousarray(x, np.float32)), ctypes.byref(lw), hidden, inter,
                              _fp(scratch))
    return out


def forward_layer_raw(x, w: dict, pos, hidden, nh, nkv, hd, inter, cos_t, sin_t, k_cache, v_cache) -> np.ndarray:
    out = np.zeros(hidden, np.float32)
    scratch = np.zeros(hidden * 64 + 4 * nh * hd + 4 * nkv * hd + 3 * inter + pos + 64, np.float32)
    lw = layer_struct(w)
    lib().ref_forward_layer_raw(_fp(out), _fp(np.ascontiguousarray(x, np.float32)), ctypes.byref(lw), pos, hidden,
                                nh, nkv, hd, inter, _fp(cos_t), _fp(sin_t), _fp(k_cache), _fp(v_cache), _fp(scratch))
    return out


# ---------------------------------------------------------------- model level
class RefModel:
    """CPU reference engine over a ``{hf_name: float32 ndarray}`` weight dict.

    Mirrors ``init_model_mojo`` (core.mojo:274-364) dimension inference and the
    fixed ``max_seq_len = 8192`` (core.mojo:328) unless ``max_seq_len`` is given.
    ``mode``: 0 = reference semantics, 1 = gemma3 extension (window, dual theta).
    """

    def __init__(self, weights: dict[str, np.ndarray], *, max_seq_len: int = 8192, mode: int = 0,
                 sliding_window: int = 512, global_every: int = 6, theta_local: float = 10000.0,
                 theta_global: float = 1000000.0) -> None:
        self._keep: list[np.ndarray] = []

        def get(name: str) -> np.ndarray | None:
            a = weights.get(name)
            if a is None:
                return None
            a = np.ascontiguousarray(a, dtype=np.float32)
            self._keep.append(a)
            return a

        embed = get("model.embed_tokens.weight")
        norm = get("model.norm.weight")
        lm_head = get("lm_head.weight")
        assert embed is not None and norm is not None and lm_head is not None
        layers = []
        i = 0
        while f"model.layers.{i}.input_layernorm.weight" in weights:
            layers.append({f: get(f"model.layers.{i}.{k}") for f, k in LAYER_KEYS})
            i += 1
        assert layers, "no layers found"
        l0 = layers[0]
        hd = int(l0["q_norm"].shape[0]) if l0["q_norm"] is not None else 256
        self.head_dim = hd
        self.num_kv_heads = int(l0["k_proj"].shape[0]) // hd
        self.num_heads = int(l0["q_proj"].shape[0]) // hd
        self.hidden_size = int(embed.shape[1])
        self.intermediate_size = int(l0["gate_proj"].shape[0])
        self.vocab_size = int(lm_head.shape[0])
        self.num_layers = len(layers)
        self.max_seq_len = max_seq_len
        arr = (_LayerW * len(layers))()
        for j, lw in enumerate(layers):
            arr[j] = layer_struct(lw)
        self._layers_arr = arr
        self._h = lib().ref_model_create(
            _fp(embed), _fp(norm), _fp(lm_head), arr, len(layers), self.hidden_size, self.num_heads,
            self.num_kv_heads, hd, self.intermediate_size, self.vocab_size, max_seq_len, mode, sliding_window,
            global_every, theta_local, theta_global)

    def close(self) -> None:
        if self._h:
            lib().ref_model_destroy(self._h)
            self._h = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    @property
    def pos(self) -> int:
        return int(lib().ref_model_pos(self._h))

    @pos.setter
    def pos(self, p: int) -> None:
        lib().ref_model_set_pos(self._h, int(p))

    def step(self, token_id: int) -> np.ndarray:
        out = np.zeros(self.vocab_size, np.float32)
        if lib().ref_step(self._h, int(token_id), _fp(out)) != 0:
            raise RuntimeError("Sequence length exceeded")
        return out

    def step_no_logits(self, token_id: int) -> None:
        if lib().ref_step_no_logits(self._h, int(token_id)) != 0:
            raise RuntimeError("Sequence length exceeded")

    def embed(self, ids, ref_compat: bool = False) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(self.hidden_size, np.float32)
        lib().ref_embed_sequence(self._h, ids.ctypes.data_as(_I32), ids.size, _fp(out), int(ref_compat))
        return out

    def encode(self, ids, dense0=None, dense1=None) -> np.ndarray:
        """Bidirectional encoder embedding (ref_encode_sequence): mean of final-normed
        states, optional dense head ``dense0`` [d, hidden] / ``dense1`` [hidden, d], L2 norm."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.zeros(self.hidden_size, np.float32)
        d0 = np.ascontiguousarray(dense0, dtype=np.float32) if dense0 is not None else None
        d1 = np.ascontiguousarray(dense1, dtype=np.float32) if dense1 is not None else None
        rc = lib().ref_encode_sequence(self._h, ids.ctypes.data_as(_I32), ids.size,
                                       _fp(d0) if d0 is not None else None, d0.shape[0] if d0 is not None else 0,
                                       _fp(d1) if d1 is not None else None, _fp(out))
        if rc != 0:
            raise ValueError("sequence length outside [1, max_seq_len]")
        return out

    def kv_row(self, layer: int, pos: int) -> tuple[np.ndarray, np.ndarray]:
        """K and V at (layer, pos) as ``[num_kv_heads, head_dim]``."""
        n = self.num_kv_heads * self.head_dim
        off = (layer * self.max_seq_len + pos) * n
        k = np.ctypeslib.as_array(lib().ref_model_k_cache(self._h), shape=(off + n,))[off:].copy()
        v = np.ctypeslib.as_array(lib().ref_model_v_cache(self._h), shape=(off + n,))[off:].copy()
        return k.reshape(self.num_kv_heads, self.head_dim), v.reshape(self.num_kv_heads, self.head_dim)


# ---------------------------------------------------------------- sampling
def sample_next_token(logits, *, temperature: float, top_k: int, top_p: float, u: float | None = None) -> int:
    """Restatement of ``_sample_next_token`` (model.py:103-150).

    ``u`` is the uniform variate that ``default_rng().choice`` would draw
    (model.py:150); ``None`` draws it from an unseeded generator like the reference.
    """
    logits_array = np.asarray(logits, dtype=np.float64).reshape(-1)
    if logits_array.size == 0:
        raise ValueError("backend returned empty logits")
    if temperature <= 0:
        return int(np.argmax(logits_array))
    filtered = logits_array / temperature
    if 0 < top_k < filtered.size:
        top_indices = np.argpartition(filtered, -top_k)[-top_k:]
        mask = np.zeros(filtered.size, dtype=bool)
        mask[top_indices] = True
        filtered = np.where(mask, filtered, -np.inf)
    if 0.0 < top_p < 1.0:
        sorted_indices = np.argsort(filtered)[::-1]
        sorted_logits = filtered[sorted_indices]
        finite = np.isfinite(sorted_logits)
        if finite.any():
            fl = sorted_logits[finite]
            fl = fl - np.max(fl)
            fp = np.exp(fl)
            fp = fp / fp.sum()
            cum = np.cumsum(fp)
            overflow = cum > top_p
            if overflow.any():
                first = int(np.argmax(overflow))
                filtered[sorted_indices[finite][first + 1:]] = -np.inf
    if not np.isfinite(filtered).any():
        return int(np.argmax(logits_array))
    stable = filtered - np.max(filtered)
    probs = np.exp(stable)
    s = probs.sum()
    if s <= 0 or not np.isfinite(s):
        return int(np.argmax(logits_array))
    probs = probs / s
    if u is None:
        return int(np.random.default_rng().choice(probs.size, p=probs))
    cdf = probs.cumsum()
    cdf /= cdf[-1]
    return int(cdf.searchsorted(u, side="right"))


def sampling_probs(logits, *, temperature: float, top_k: int, top_p: float) -> np.ndarray:
    """The probability vector ``_sample_next_token`` draws from (T > 0)."""
    logits_array = np.asarray(logits, dtype=np.float64).reshape(-1)
    filtered = logits_array / temperature
    if 0 < top_k < filtered.size:
        top_indices = np.argpartition(filtered, -top_k)[-top_k:]
        mask = np.zeros(filtered.size, dtype=bool)
        mask[top_indices] = True
        filtered = np.where(mask, filtered, -np.inf)
    if 0.0 < top_p < 1.0:
        sorted_indices = np.argsort(filtered)[::-1]
        sorted_logits = filtered[sorted_indices]
        finite = np.isfinite(sorted_logits)
        fl = sorted_logits[finite] - np.max(sorted_logits[finite])
        fp = np.exp(fl)
        fp = fp / fp.sum()
        overflow = np.cumsum(fp) > top_p
        if overflow.any():
            first = int(np.argmax(overflow))
            filtered[sorted_indices[finite][first + 1:]] = -np.inf
    stable = filtered - np.max(filtered)
    probs = np.exp(stable)
    return probs / probs.sum()


def top_k_set(logits, k: int) -> set[int]:
    """Index set the reference keeps for top-k (model.py:115-119)."""
    a = np.asarray(logits, dtype=np.float64).reshape(-1)
    return {int(i) for i in np.argpartition(a, -k)[-k:]}


def default_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
