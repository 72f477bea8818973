"""``_core``: the operator boundary, a thin ctypes shim over ``libmogemma_cuda.so``.

Drop-in for the reference's CPython extension ``mogemma._core``
(``src/mo/mogemma/core.mojo:602-611``), which exports ``init_model``, ``step``
and ``generate_embeddings``.  The same three functions keep their signatures,
return types and error strings; the work runs in the sm_100a CUDA library
declared in ``include/mogemma_b200.h``.  Extra entry points (``prefill``,
``step_sample``, ``generate``, ``sample``) expose the on-device prefill,
sampling and decode loop that ``model.py`` uses when present.

There is no CPU fallback: importing this module raises ``ImportError`` when
the library is missing, and every call raises when the CUDA library fails.
"""

from __future__ import annotations

import ctypes
import os
from collections.abc import Sequence
from pathlib import Path
from typing import Any

import numpy as np
import numpy.typing as npt

_LIB_NAME = "libmogemma_cuda.so"
_LIB_PATH = Path(__file__).resolve().parent / _LIB_NAME

if not _LIB_PATH.exists():
    msg = f"{_LIB_NAME} is not built; run `make -C {_LIB_PATH.parent / 'csrc'}` (or __graft_entry__.build())"
    raise ImportError(msg)

_lib = ctypes.CDLL(str(_LIB_PATH))

ENGINE_NAME = "MoGemma B200 CUDA Engine"

# mg_status
MG_OK = 0
MG_ERR_INVALID = 1
MG_ERR_CUDA = 2
MG_ERR_OOM = 3
MG_ERR_SEQ_EXCEEDED = 4
MG_ERR_TIMEOUT = 5
MG_ERR_UNSUPPORTED = 6
MG_ERR_NCCL = 7

# mg_dtype
MG_F32, MG_BF16, MG_F16, MG_I32, MG_U8, MG_OTHER = 0, 1, 2, 3, 4, 99
_DTYPES = {"F32": MG_F32, "BF16": MG_BF16, "F16": MG_F16, "I32": MG_I32, "U8": MG_U8}


class TensorDesc(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char_p),
        ("data", ctypes.c_void_p),
        ("shape", ctypes.c_int64 * 4),
        ("ndim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class Options(ctypes.Structure):
    _fields_ = [
        ("struct_size", ctypes.c_int32),
        ("device", ctypes.c_int32),
        ("mode", ctypes.c_int32),
        ("weight_dtype", ctypes.c_int32),
        ("max_batch", ctypes.c_int32),
        ("capacity", ctypes.c_int32),
        ("sliding_window", ctypes.c_int32),
        ("global_every", ctypes.c_int32),
        ("rope_theta_local", ctypes.c_float),
        ("rope_theta_global", ctypes.c_float),
        ("seed", ctypes.c_uint64),
        ("stream", ctypes.c_void_p),
        ("decode_path", ctypes.c_int32),
        ("tp_rank", ctypes.c_int32),
        ("tp_size", ctypes.c_int32),
        ("prefill_path", ctypes.c_int32),
        ("reserved1", ctypes.c_void_p),
        ("synthetic_std", ctypes.c_float),
        ("reserved2", ctypes.c_int32),
        ("synthetic_seed", ctypes.c_uint64),
    ]


class ModelInfo(ctypes.Structure):
    _fields_ = [
        (n, ctypes.c_int32)
        for n in ("num_layers", "num_heads", "num_kv_heads", "head_dim", "hidden_size", "intermediate_size",
                  "vocab_size", "max_seq_len", "max_batch", "mode", "weight_dtype", "tp_size")
    ] + [
        ("weight_bytes_per_step", ctypes.c_int64),
        ("kv_bytes_per_pos", ctypes.c_int64),
        ("num_sms", ctypes.c_int32),
        ("persistent_ctas", ctypes.c_int32),
    ]


class Sampling(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_double),
        ("top_k", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("top_p", ctypes.c_double),
        ("uniforms_host", ctypes.POINTER(ctypes.c_double)),
    ]


class NanoInfo(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "num_layers", "num_heads", "num_kv_heads", "head_dim", "hidden_size", "intermediate_size", "vocab_size",
        "per_layer_dim", "modalities", "laurel_rank", "kv_share_start", "max_seq_len")]


_P = ctypes.c_void_p
_I32P = ctypes.POINTER(ctypes.c_int32)
_F32P = ctypes.POINTER(ctypes.c_float)

_lib.mg_last_error.restype = ctypes.c_char_p
_lib.mg_abi_version.restype = ctypes.c_int32
_lib.mg_model_create.argtypes = [ctypes.POINTER(TensorDesc), ctypes.c_int32, ctypes.POINTER(Options),
                                 ctypes.POINTER(_P)]
_lib.mg_model_info_get.argtypes = [_P, ctypes.POINTER(ModelInfo)]
_lib.mg_model_destroy.argtypes = [_P]
_lib.mg_model_stream.argtypes = [_P]
_lib.mg_model_stream.restype = _P
_lib.mg_rows_per_launch.argtypes = [_P]
_lib.mg_rows_per_launch.restype = ctypes.c_int32
_lib.mg_nano_create.argtypes = [ctypes.POINTER(TensorDesc), ctypes.c_int32, ctypes.c_int32, ctypes.c_int32,
                                ctypes.POINTER(_P)]
_lib.mg_nano_info_get.argtypes = [_P, ctypes.POINTER(NanoInfo)]
_lib.mg_nano_destroy.argtypes = [_P]
_lib.mg_nano_set_pos.argtypes = [_P, ctypes.c_int32]
_lib.mg_nano_get_pos.argtypes = [_P, _I32P]
_lib.mg_nano_step.argtypes = [_P, ctypes.c_int32, _F32P]
_lib.mg_nano_prefill.argtypes = [_P, _I32P, ctypes.c_int32]
_lib.mg_nano_embed.argtypes = [_P, _I32P, ctypes.c_int32, _F32P]
_lib.mg_set_pos.argtypes = [_P, ctypes.c_int32, ctypes.c_int32]
_lib.mg_get_pos.argtypes = [_P, _I32P, ctypes.c_int32]
_lib.mg_step.argtypes = [_P, _I32P, ctypes.c_int32, _F32P, _I32P, ctypes.POINTER(Sampling)]
_lib.mg_prefill.argtypes = [_P, _I32P, _I32P, ctypes.c_int32, ctypes.c_int32]
_lib.mg_generate.argtypes = [_P, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(Sampling), _I32P]
_lib.mg_set_tokens.argtypes = [_P, _I32P, ctypes.c_int32]
_lib.mg_sample.argtypes = [_F32P, ctypes.c_int32, ctypes.c_int32, ctypes.POINTER(Sampling), ctypes.c_uint64,
                           ctypes.c_uint64, _I32P]
_lib.mg_embed.argtypes = [_P, _I32P, _I32P, ctypes.c_int32, ctypes.c_int32, _F32P]
_lib.mg_encode.argtypes = [_P, _I32P, _I32P, ctypes.c_int32, ctypes.c_int32, _F32P]
_lib.mg_read_kv.argtypes = [_P, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _F32P, _F32P]
_lib.mg_tp_ipc_handle.argtypes = [_P, _P]
_lib.mg_tp_connect.argtypes = [_P, _P, ctypes.c_int32]
_lib.mg_tp_disconnect.argtypes = [_P]
TP_HANDLE_BYTES = 64  # MG_TP_HANDLE_BYTES
_lib.mg_trace_enable.argtypes = [_P, ctypes.c_int32]
_lib.mg_trace_read.argtypes = [_P, ctypes.POINTER(ctypes.c_uint64), ctypes.c_int64, ctypes.POINTER(ctypes.c_int64)]
_lib.mg_set_debug.argtypes = [_P, ctypes.c_uint64, ctypes.c_int32]
for _f in ("mg_model_create", "mg_model_info_get", "mg_model_destroy", "mg_set_pos", "mg_get_pos", "mg_step",
           "mg_prefill", "mg_generate", "mg_set_tokens", "mg_sample", "mg_embed", "mg_read_kv",
           "mg_tp_ipc_handle", "mg_tp_connect", "mg_tp_disconnect", "mg_encode", "mg_trace_enable", "mg_trace_read",
           "mg_set_debug"):
    getattr(_lib, _f).restype = ctypes.c_int


def lib() -> ctypes.CDLL:
    """The loaded ``libmogemma_cuda.so``."""
    return _lib


def _check(status: int) -> None:
    if status == MG_OK:
        return
    msg = (_lib.mg_last_error() or b"").decode("utf-8", "replace")
    if status == MG_ERR_SEQ_EXCEEDED:
        raise RuntimeError("Sequence length exceeded")
    if status == MG_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


def _i32(a: Any) -> npt.NDArray[np.int32]:
    return np.ascontiguousarray(a, dtype=np.int32)


def _env_int(name: str, default: int) -> int:
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


class ModelHandle:
    """Owns one ``mg_model``; destroyed with the ``llm`` dict that holds it."""

    def __init__(self, ptr: int, info: ModelInfo) -> None:
        self.ptr = ptr
        self.info = info
        self.pos = 0

    def close(self) -> None:
        if self.ptr:
            _lib.mg_model_destroy(self.ptr)
            self.ptr = 0

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    @property
    def stream(self) -> int:
        return int(_lib.mg_model_stream(self.ptr) or 0)

    @property
    def rows_per_launch(self) -> int:
        """Rows one persistent decode launch holds (more rows run one launch per group)."""
        return int(_lib.mg_rows_per_launch(self.ptr))

    def set_pos(self, pos: int, row: int = -1) -> None:
        _check(_lib.mg_set_pos(self.ptr, row, int(pos)))
        if row in (-1, 0):
            self.pos = int(pos)

    def set_debug(self, wait_budget_ns: int = 0, stall_phase: int = -1) -> None:
        """Failure-detection test hook: wait budget of the decode kernel and a phase whose outputs are withheld."""
        _check(_lib.mg_set_debug(self.ptr, int(wait_budget_ns), int(stall_phase)))

    def trace(self, on: bool = True) -> None:
        """Record a per-CTA, per-phase timeline of every decode launch."""
        _check(_lib.mg_trace_enable(self.ptr, int(on)))

    def read_trace(self) -> tuple[npt.NDArray[np.uint64], npt.NDArray[np.uint64]]:
        """Timeline of the last launch: ([ctas, phases, slots] stamps, [ctas, 2] kernel begin/end) in ns.

        Slots: start, ready, first tile, end, producer start, producer end,
        then for attention phases: q/k/v loaded, normed+roped, tiles done, partial written.
        """
        n = ctypes.c_int64(0)
        _check(_lib.mg_trace_read(self.ptr, (ctypes.c_uint64 * 1)(), 0, ctypes.byref(n)))
        buf = np.zeros(int(n.value), np.uint64)
        _check(_lib.mg_trace_read(self.ptr, buf.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), buf.size,
                                  ctypes.byref(n)))
        g = int(self.info.persistent_ctas)
        nph = 5 * int(self.info.num_layers) + 2
        slots = (buf.size - 2 * g) // (g * nph)
        return buf[: g * nph * slots].reshape(g, nph, slots), buf[g * nph * slots:].reshape(g, 2)

    def tp_handle(self) -> bytes:
        """IPC handle of this rank's exchange buffer (tensor-parallel models)."""
        buf = ctypes.create_string_buffer(TP_HANDLE_BYTES)
        _check(_lib.mg_tp_ipc_handle(self.ptr, ctypes.cast(buf, _P)))
        return buf.raw

    def tp_connect(self, handles: Sequence[bytes]) -> None:
        """Map the other ranks' exchange buffers (handles in rank order)."""
        blob = b"".join(handles)
        if len(blob) != TP_HANDLE_BYTES * len(handles):
            msg = "every handle must be TP_HANDLE_BYTES long"
            raise ValueError(msg)
        buf = ctypes.create_string_buffer(blob, len(blob))
        _check(_lib.mg_tp_connect(self.ptr, ctypes.cast(buf, _P), len(handles)))

    def get_pos(self) -> list[int]:
        n = max(8, int(self.info.max_batch))
        out = np.zeros(n, np.int32)
        _check(_lib.mg_get_pos(self.ptr, out.ctypes.data_as(_I32P), n))
        return [int(x) for x in out]


def _sampling(temperature: float, top_k: int, top_p: float, uniforms: Any = None) -> tuple[Sampling, Any]:
    s = Sampling()
    s.temperature = float(temperature)
    s.top_k = int(top_k)
    s.top_p = float(top_p)
    keep = None
    if uniforms is not None:
        keep = np.ascontiguousarray(uniforms, dtype=np.float64)
        s.uniforms_host = keep.ctypes.data_as(ctypes.POINTER(ctypes.c_double))
    return s, keep


def create_model(metadata: dict[str, Any], **options: Any) -> ModelHandle:
    """``mg_model_create`` over ``{name: (ptr, shape[, dtype])}`` loader metadata."""
    names = list(metadata.keys())
    descs = (TensorDesc * len(names))()
    keep: list[bytes] = []
    for i, name in enumerate(names):
        meta = metadata[name]
        ptr, shape = int(meta[0]), tuple(int(s) for s in meta[1])
        dtype = str(meta[2]) if len(meta) > 2 else "F32"
        nb = name.encode()
        keep.append(nb)
        descs[i].name = nb
        descs[i].data = ptr
        descs[i].ndim = min(len(shape), 4)
        for k in range(descs[i].ndim):
            descs[i].shape[k] = shape[k]
        descs[i].dtype = _DTYPES.get(dtype.upper(), MG_OTHER)
    o = Options()
    o.struct_size = ctypes.sizeof(Options)
    o.device = int(options.get("device", _env_int("MOGEMMA_B200_DEVICE", 0)))
    mode = options.get("mode", os.environ.get("MOGEMMA_B200_MODE", "ref"))
    o.mode = {"ref": 0, "gemma3": 1, 0: 0, 1: 1}[mode]
    wd = options.get("weight_dtype", os.environ.get("MOGEMMA_B200_WEIGHT_DTYPE", "f32"))
    o.weight_dtype = {"f32": MG_F32, "bf16": MG_BF16, MG_F32: MG_F32, MG_BF16: MG_BF16}[wd]
    o.max_batch = int(options.get("max_batch", _env_int("MOGEMMA_B200_MAX_BATCH", 1)))
    o.capacity = int(options.get("capacity", _env_int("MOGEMMA_B200_CAPACITY", 8192)))
    o.sliding_window = int(options.get("sliding_window", 512))
    o.global_every = int(options.get("global_every", 6))
    o.rope_theta_local = float(options.get("rope_theta_local", 10000.0))
    o.rope_theta_global = float(options.get("rope_theta_global", 1000000.0))
    o.seed = int(options.get("seed", _env_int("MOGEMMA_B200_SEED", 0))) & 0xFFFFFFFFFFFFFFFF
    o.stream = options.get("stream")
    o.decode_path = int(options.get("decode_path", _env_int("MOGEMMA_B200_DECODE_PATH", 0)))
    o.prefill_path = int(options.get("prefill_path", _env_int("MOGEMMA_B200_PREFILL", 0)))
    o.synthetic_std = float(options.get("synthetic_std", 0.0))
    o.synthetic_seed = int(options.get("synthetic_seed", 0)) & 0xFFFFFFFFFFFFFFFF
    o.tp_rank = int(options.get("tp_rank", 0))
    o.tp_size = int(options.get("tp_size", 1))
    out = _P()
    _check(_lib.mg_model_create(descs, len(names), ctypes.byref(o), ctypes.byref(out)))
    info = ModelInfo()
    _check(_lib.mg_model_info_get(out, ctypes.byref(info)))
    return ModelHandle(int(out.value), info)


class NanoHandle:
    """Owns one ``mg_nano`` (Gemma 3n decode engine)."""

    def __init__(self, ptr: int, info: NanoInfo) -> None:
        self.ptr = ptr
        self.info = info
        self.pos = 0

    def close(self) -> None:
        if self.ptr:
            _lib.mg_nano_destroy(self.ptr)
            self.ptr = 0

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:  # noqa: BLE001
            pass

    def set_pos(self, pos: int) -> None:
        _check(_lib.mg_nano_set_pos(self.ptr, int(pos)))
        self.pos = int(pos)


def _tensor_descs(metadata: dict[str, Any]) -> tuple[Any, list[bytes]]:
    names = list(metadata.keys())
    descs = (TensorDesc * len(names))()
    keep: list[bytes] = []
    for i, name in enumerate(names):
        meta = metadata[name]
        ptr, shape = int(meta[0]), tuple(int(s) for s in meta[1])
        dtype = str(meta[2]) if len(meta) > 2 else "F32"
        nb = name.encode()
        keep.append(nb)
        descs[i].name = nb
        descs[i].data = ptr
        descs[i].ndim = min(len(shape), 4)
        for k in range(descs[i].ndim):
            descs[i].shape[k] = shape[k]
        descs[i].dtype = _DTYPES.get(dtype.upper(), MG_OTHER)
    return descs, keep


def create_nano(metadata: dict[str, Any], **options: Any) -> NanoHandle:
    """``mg_nano_create`` over loader metadata of a Gemma 3n checkpoint."""
    descs, _keep = _tensor_descs(metadata)
    device = int(options.get("device", _env_int("MOGEMMA_B200_DEVICE", 0)))
    capacity = int(options.get("capacity", _env_int("MOGEMMA_B200_CAPACITY", 8192)))
    out = _P()
    _check(_lib.mg_nano_create(descs, len(descs), device, capacity, ctypes.byref(out)))
    info = NanoInfo()
    _check(_lib.mg_nano_info_get(out, ctypes.byref(info)))
    return NanoHandle(int(out.value), info)


def _init_nano(metadata: dict[str, Any], **options: Any) -> dict[str, Any]:
    """init_model_mojo's nano branch (core.mojo:296-312, 350-364)."""
    handle = create_nano(metadata, **options)
    info = handle.info
    runtime = {k: metadata.get(v) for k, v in (
        ("embed_tokens", "model.embed_tokens.weight"), ("norm", "model.norm.weight"), ("lm_head", "lm_head.weight"),
        ("per_layer_embed", "model.per_layer_embed.weight"))}
    return {
        "engine": ENGINE_NAME,
        "arch": "nano",
        "max_seq_len": int(info.max_seq_len),
        "num_layers": int(info.num_layers),
        "num_kv_heads": int(info.num_kv_heads),
        "head_dim": int(info.head_dim),
        "hidden_size": int(info.hidden_size),
        "intermediate_size": int(info.intermediate_size),
        "vocab_size": int(info.vocab_size),
        "per_layer_dim": int(info.per_layer_dim),
        "kv_share_start": int(info.kv_share_start),
        "runtime": runtime,
        "pos": 0,
        "_handle": handle,
    }


def _nano(llm: dict[str, Any]) -> NanoHandle | None:
    """The Gemma 3n handle of ``llm`` (position synced from ``llm["pos"]``), or None."""
    h = llm.get("_handle")
    if not isinstance(h, NanoHandle):
        return None
    if not h.ptr:
        msg = "llm was closed"
        raise RuntimeError(msg)
    pos = int(llm.get("pos", 0))
    if pos != h.pos:
        h.set_pos(pos)
    return h


# ------------------------------------------------------------- reference API
def init_model(metadata: dict[str, Any], **options: Any) -> dict[str, Any]:
    """Reference ``init_model`` (core.mojo:274-364): returns the ``llm`` dict.

    Keys follow core.mojo:350-364; the device model lives under ``_handle``.
    Extra keyword options (mode, weight_dtype, max_batch, capacity, device,
    seed, decode_path, ...) are private to this engine.
    """
    if "model.layers.0.altup.router.weight" in metadata:  # core.mojo:26-31: arch "nano"
        return _init_nano(metadata, **options)
    handle = create_model(metadata, **options)
    info = handle.info
    runtime = {
        "embed_tokens": metadata.get("model.embed_tokens.weight"),
        "norm": metadata.get("model.norm.weight"),
        "lm_head": metadata.get("lm_head.weight"),
    }
    return {
        "engine": ENGINE_NAME,
        "arch": "standard",
        "max_seq_len": int(info.max_seq_len),
        "num_layers": int(info.num_layers),
        "num_kv_heads": int(info.num_kv_heads),
        "head_dim": int(info.head_dim),
        "hidden_size": int(info.hidden_size),
        "intermediate_size": int(info.intermediate_size),
        "vocab_size": int(info.vocab_size),
        "per_layer_dim": 0,
        "kv_share_start": int(info.num_layers),
        "runtime": runtime,
        "pos": 0,
        "_handle": handle,
    }


def gather_handles(handle: bytes, group: Any = None) -> list[bytes]:
    """All ranks' exchange-buffer handles in rank order, over torch.distributed."""
    import torch.distributed as dist  # noqa: PLC0415

    out: list[Any] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return [bytes(h) for h in out]


def init_model_tp(metadata: dict[str, Any], group: Any = None, **options: Any) -> dict[str, Any]:
    """``init_model`` for one rank of a tensor-parallel group (one process per
    GPU, torch.distributed initialised).  Every rank loads the same checkpoint
    and keeps its shard; the exchange buffers are connected before returning."""
    import torch.distributed as dist  # noqa: PLC0415

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    llm = init_model(metadata, tp_rank=rank, tp_size=world, **options)
    if world > 1:
        h = llm["_handle"]
        h.tp_connect(gather_handles(h.tp_handle(), group))
        dist.barrier(group)
    return llm


def close_tp(llm: dict[str, Any], group: Any = None) -> None:
    """Destroy one rank's tensor-parallel model: every rank unmaps its peers'
    buffers before any rank frees its own."""
    import torch.distributed as dist  # noqa: PLC0415

    h = llm["_handle"]
    if int(h.info.tp_size) > 1:
        dist.barrier(group)
        _check(_lib.mg_tp_disconnect(h.ptr))
        dist.barrier(group)
    h.close()


def _handle(llm: dict[str, Any]) -> ModelHandle:
    h = llm.get("_handle")
    if isinstance(h, NanoHandle):
        msg = "this call is not available for Gemma 3n (nano) models: use init_model / step / prefill / " \
              "step_sample / generate_embeddings"
        raise RuntimeError(msg)
    if not isinstance(h, ModelHandle) or not h.ptr:
        msg = "llm was not created by mogemma_b200._core.init_model"
        raise RuntimeError(msg)
    pos = int(llm.get("pos", 0))
    if pos != h.pos:
        h.set_pos(pos, row=0)
    return h


def step(llm: dict[str, Any], token_id: int, temperature: float, top_k: int, top_p: float) -> npt.NDArray[np.float32]:
    """Reference ``step`` (core.mojo:366-461): one token at ``llm["pos"]``, returns
    fp32 logits of shape (vocab,) and advances ``llm["pos"]``.  The sampling
    arguments are accepted and unused, as in the reference."""
    del temperature, top_k, top_p
    nh = _nano(llm)
    if nh is not None:
        if nh.pos >= int(llm["max_seq_len"]):
            raise RuntimeError("Sequence length exceeded")
        logits = np.empty(int(llm["vocab_size"]), dtype=np.float32)
        _check(_lib.mg_nano_step(nh.ptr, int(token_id), logits.ctypes.data_as(_F32P)))
        nh.pos += 1
        llm["pos"] = nh.pos
        return logits
    h = _handle(llm)
    if h.pos >= int(llm["max_seq_len"]):
        raise RuntimeError("Sequence length exceeded")
    ids = _i32([int(token_id)])
    logits = np.empty(int(llm["vocab_size"]), dtype=np.float32)
    _check(_lib.mg_step(h.ptr, ids.ctypes.data_as(_I32P), 1, logits.ctypes.data_as(_F32P), None, None))
    h.pos += 1
    llm["pos"] = h.pos
    return logits


def step_sample(llm: dict[str, Any], token_id: int, temperature: float, top_k: int, top_p: float,
                uniform: float | None = None) -> int:
    """One decode step with the draw of ``_sample_next_token`` done on device;
    returns the sampled token id (4 bytes cross the bus instead of the logits).
    Gemma 3n models return their logits to the host and draw with ``sample``
    (Philox stream keyed by the model's seed option and the position)."""
    nh = _nano(llm)
    if nh is not None:
        pos = nh.pos
        logits = step(llm, token_id, temperature, top_k, top_p)
        return int(sample(logits, temperature, top_k, top_p, seed=int(llm.get("seed", 0)), offset=pos,
                          uniforms=None if uniform is None else [uniform])[0])
    h = _handle(llm)
    if h.pos >= int(llm["max_seq_len"]):
        raise RuntimeError("Sequence length exceeded")
    ids = _i32([int(token_id)])
    out = np.zeros(1, np.int32)
    s, keep = _sampling(temperature, top_k, top_p, None if uniform is None else [uniform])
    _check(_lib.mg_step(h.ptr, ids.ctypes.data_as(_I32P), 1, None, out.ctypes.data_as(_I32P), ctypes.byref(s)))
    del keep
    h.pos += 1
    llm["pos"] = h.pos
    return int(out[0])


def step_rows(llm: dict[str, Any], token_ids: Sequence[int], *, logits: bool = True,
              sampling: tuple[float, int, float] | None = None,
              uniforms: Sequence[float] | None = None) -> tuple[npt.NDArray[np.float32] | None, npt.NDArray[np.int32] | None]:
    """One decode step for rows 0..len(token_ids)-1 (each at its own position).

    Returns ([rows, vocab] logits or None, [rows] drawn tokens or None).
    Positions are per row on the device; ``llm["pos"]`` mirrors row 0.
    """
    h = _handle(llm)
    ids = _i32(list(token_ids))
    n = int(ids.size)
    lg = np.empty((n, int(llm["vocab_size"])), np.float32) if logits else None
    out = np.zeros(n, np.int32) if sampling is not None else None
    s = keep = None
    if sampling is not None:
        s, keep = _sampling(sampling[0], sampling[1], sampling[2], uniforms)
    _check(_lib.mg_step(h.ptr, ids.ctypes.data_as(_I32P), n, lg.ctypes.data_as(_F32P) if lg is not None else None,
                        out.ctypes.data_as(_I32P) if out is not None else None,
                        ctypes.byref(s) if s is not None else None))
    del keep
    h.pos += 1
    llm["pos"] = h.pos
    return lg, out


def set_row_pos(llm: dict[str, Any], row: int, pos: int) -> None:
    """Set one row's next position (a stream reusing a row restarts it at 0)."""
    h = _handle(llm)
    h.set_pos(int(pos), row=int(row))
    llm["pos"] = h.pos  # llm["pos"] mirrors row 0


def row_positions(llm: dict[str, Any]) -> list[int]:
    """Next position of every row."""
    return _handle(llm).get_pos()


def prefill_rows(llm: dict[str, Any], rows: Sequence[Sequence[int]]) -> None:
    """Prefill several rows (ragged) at their current positions."""
    h = _handle(llm)
    max_len = max((len(r) for r in rows), default=0)
    if max_len == 0:
        return
    ids = np.zeros((len(rows), max_len), np.int32)
    lens = np.zeros(len(rows), np.int32)
    for i, r in enumerate(rows):
        ids[i, : len(r)] = r
        lens[i] = len(r)
    _check(_lib.mg_prefill(h.ptr, ids.ctypes.data_as(_I32P), lens.ctypes.data_as(_I32P), len(rows), max_len))
    h.pos += int(lens[0])
    llm["pos"] = h.pos


def prefill(llm: dict[str, Any], tokens: Sequence[int]) -> None:
    """Feed ``tokens`` at ``llm["pos"]`` without computing logits (the
    reference's prefill loop discards them, model.py:344-345)."""
    toks = _i32(list(tokens))
    if toks.size == 0:
        return
    nh = _nano(llm)
    if nh is not None:
        if nh.pos + toks.size > int(llm["max_seq_len"]):
            raise RuntimeError("Sequence length exceeded")
        _check(_lib.mg_nano_prefill(nh.ptr, toks.ctypes.data_as(_I32P), int(toks.size)))
        nh.pos += int(toks.size)
        llm["pos"] = nh.pos
        return
    h = _handle(llm)
    if h.pos + toks.size > int(llm["max_seq_len"]):
        raise RuntimeError("Sequence length exceeded")
    lens = _i32([toks.size])
    _check(_lib.mg_prefill(h.ptr, toks.ctypes.data_as(_I32P), lens.ctypes.data_as(_I32P), 1, int(toks.size)))
    h.pos += int(toks.size)
    llm["pos"] = h.pos


def generate(llm: dict[str, Any], token_id: int, n_steps: int, temperature: float, top_k: int,
             top_p: float) -> list[int]:
    """Device-resident decode loop: feeds ``token_id`` then each sampled token."""
    h = _handle(llm)
    ids = _i32([int(token_id)])
    _check(_lib.mg_set_tokens(h.ptr, ids.ctypes.data_as(_I32P), 1))
    out = np.zeros(int(n_steps), np.int32)
    s, _keep = _sampling(temperature, top_k, top_p)
    _check(_lib.mg_generate(h.ptr, int(n_steps), 1, ctypes.byref(s), out.ctypes.data_as(_I32P)))
    h.pos += int(n_steps)
    llm["pos"] = h.pos
    return [int(x) for x in out]


def sample(logits: Any, temperature: float, top_k: int, top_p: float, *, seed: int = 0, offset: int = 0,
           uniforms: Any = None) -> npt.NDArray[np.int32]:
    """``_sample_next_token`` rules on device for a [batch, vocab] (or [vocab]) array."""
    arr = np.ascontiguousarray(logits, dtype=np.float32)
    if arr.ndim == 1:
        arr = arr[None, :]
    if arr.size == 0:
        raise ValueError("backend returned empty logits")
    out = np.zeros(arr.shape[0], np.int32)
    s, _keep = _sampling(temperature, top_k, top_p, uniforms)
    _check(_lib.mg_sample(arr.ctypes.data_as(_F32P), arr.shape[0], arr.shape[1], ctypes.byref(s), int(seed),
                          int(offset), out.ctypes.data_as(_I32P)))
    return out


def _ensure_embedding_matrix(emb: npt.NDArray[np.float32], rows: int, cols: int) -> npt.NDArray[np.float32]:
    # core.mojo:43-52
    if emb.ndim != 2:
        raise RuntimeError("generate_embeddings output must be a 2D float32 matrix")
    if emb.shape[0] != rows:
        raise RuntimeError("generate_embeddings output row count does not match inputs")
    if emb.shape[1] != cols:
        raise RuntimeError("generate_embeddings output columns do not match hidden_size")
    return emb


def generate_embeddings(llm: dict[str, Any], input_array: Any) -> npt.NDArray[np.float32]:
    """Reference ``generate_embeddings`` (core.mojo:463-600): mean of final-normed
    states per sequence, shape (batch, hidden_size), fp32.  Ragged lists are
    accepted; the model's KV rows serve as scratch."""
    rows = [list(map(int, r)) for r in (input_array.tolist() if isinstance(input_array, np.ndarray) else input_array)]
    if len(rows) == 0:
        raise RuntimeError("inputs must contain at least one row")
    max_len = max(len(r) for r in rows)
    if max_len == 0:
        raise RuntimeError("inputs must contain at least one token")
    nh = _nano(llm)
    if nh is not None:  # forward_nano_sequence per row (layers.mojo:1007-1063)
        out = np.zeros((len(rows), int(llm["hidden_size"])), np.float32)
        for i, r in enumerate(rows):
            if not r:
                raise RuntimeError("inputs must contain at least one token")
            ids = _i32(r)
            _check(_lib.mg_nano_embed(nh.ptr, ids.ctypes.data_as(_I32P), len(r), out[i].ctypes.data_as(_F32P)))
        return _ensure_embedding_matrix(out, len(rows), int(llm["hidden_size"]))
    h = _handle(llm)
    ids = np.zeros((len(rows), max_len), np.int32)
    lens = np.zeros(len(rows), np.int32)
    for i, r in enumerate(rows):
        ids[i, : len(r)] = r
        lens[i] = len(r)
    hidden = int(llm["hidden_size"])
    out = np.zeros((len(rows), hidden), np.float32)
    _check(_lib.mg_embed(h.ptr, ids.ctypes.data_as(_I32P), lens.ctypes.data_as(_I32P), len(rows), max_len,
                         out.ctypes.data_as(_F32P)))
    return _ensure_embedding_matrix(out, len(rows), hidden)


def encode_embeddings(llm: dict[str, Any], input_array: Any) -> npt.NDArray[np.float32]:
    """Bidirectional encoder embeddings ([batch, hidden], unit L2 norm) of ragged
    token lists or a 2-D id array; the model must use ``prefill_path=1``."""
    rows = [list(r) for r in input_array]
    if not rows or any(len(r) == 0 for r in rows):
        raise RuntimeError("inputs must contain at least one token per row")
    max_len = max(len(r) for r in rows)
    ids = np.zeros((len(rows), max_len), np.int32)
    lens = np.zeros(len(rows), np.int32)
    for i, r in enumerate(rows):
        ids[i, : len(r)] = r
        lens[i] = len(r)
    out = np.zeros((len(rows), int(llm["hidden_size"])), np.float32)
    h = _handle(llm)
    _check(_lib.mg_encode(h.ptr, ids.ctypes.data_as(_I32P), lens.ctypes.data_as(_I32P), len(rows), max_len,
                          out.ctypes.data_as(_F32P)))
    return out


def read_kv(llm: dict[str, Any], layer: int, pos: int, row: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """K and V rows cached at (layer, row, pos) as [num_kv_heads, head_dim]."""
    h = _handle(llm)
    nkv, hd = int(llm["num_kv_heads"]), int(llm["head_dim"])
    k = np.zeros(nkv * hd, np.float32)
    v = np.zeros(nkv * hd, np.float32)
    _check(_lib.mg_read_kv(h.ptr, layer, row, pos, k.ctypes.data_as(_F32P), v.ctypes.data_as(_F32P)))
    return k.reshape(nkv, hd), v.reshape(nkv, hd)
