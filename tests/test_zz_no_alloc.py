"""mg_sample_static (device logits, no allocation) against mg_sample.

mg_sample_static serves callers that keep all device memory in their own pool
and cannot have the library call cudaMalloc; its only scratch is a static
device array shared by every call.  Each case calls it twice in a row on the
same stream and checks both results against mg_sample's tokens for the same
logits, sampling arguments and variates (tokens must be identical).  One case
passes rows with a padded stride (ld > vocab), and one checks that repeated
calls leave the device's free memory unchanged.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from mogemma_b200 import _core

pytestmark = pytest.mark.gpu

MAX_ROWS = 8  # MG_SAMPLE_STATIC_MAX_ROWS

_lib = _core.lib()
_lib.mg_sample_static.argtypes = [
    ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32, ctypes.c_double, ctypes.c_int32,
    ctypes.c_double, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p,
]
_lib.mg_sample_static.restype = ctypes.c_int


def _logits(batch: int, vocab: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, vocab)).astype(np.float32) * 3.0
    # ties at the maximum: the first index must win (numpy argmax rule)
    for b in range(batch):
        j = int(np.argmax(x[b]))
        k = (j * 7919 + 13) % vocab
        x[b, max(j, k)] = x[b, j]
    return x


def _static(torch, dev_logits, out, temperature, top_k, top_p, uniforms, seed, offset) -> int:
    batch, vocab = dev_logits.shape
    stream = torch.cuda.current_stream().cuda_stream
    return _lib.mg_sample_static(
        ctypes.c_void_p(dev_logits.data_ptr()), dev_logits.stride(0), batch, vocab, temperature, top_k, top_p,
        ctypes.c_void_p(uniforms.data_ptr()) if uniforms is not None else None, seed, offset,
        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream))


CASES = [
    # batch, vocab, temperature, top_k, top_p, with_uniforms
    (4, 262144, 0.0, 0, 1.0, False),
    (4, 262144, 0.8, 40, 1.0, True),
    (3, 262144, 1.0, 64, 0.9, False),
    (MAX_ROWS, 1000, 0.7, 5, 1.0, True),
    (2, 50, 1.3, 0, 0.5, True),
    (1, 262144, 0.6, 1, 1.0, False),
]


@pytest.mark.parametrize(("batch", "vocab", "temperature", "top_k", "top_p", "with_u"), CASES)
def test_static_sampler_matches_mg_sample(batch, vocab, temperature, top_k, top_p, with_u) -> None:
    torch = pytest.importorskip("torch")
    x = _logits(batch, vocab, seed=vocab + batch)
    u = np.random.default_rng(batch).random(batch) if with_u else None
    seed, offset = 1234, 17
    want = _core.sample(x, temperature, top_k, top_p, seed=seed, offset=offset, uniforms=u)

    dev = torch.from_numpy(x).cuda()
    du = torch.from_numpy(u).cuda() if u is not None else None
    for _ in range(2):  # two calls in a row share the static scratch
        out = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
        rc = _static(torch, dev, out, temperature, top_k, top_p, du, seed, offset)
        assert rc == _core.MG_OK, _lib.mg_last_error().decode()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_static_sampler_padded_rows() -> None:
    """Rows of a wider buffer (ld = vocab + 37): the padding holds values that
    would win the draw if it were read."""
    torch = pytest.importorskip("torch")
    batch, vocab, pad = 5, 262144, 37
    x = _logits(batch, vocab, seed=99)
    wide = np.full((batch, vocab + pad), 1e4, np.float32)
    wide[:, :vocab] = x
    u = np.random.default_rng(5).random(batch)
    dev = torch.from_numpy(wide).cuda()[:, :vocab]
    assert dev.stride(0) == vocab + pad
    du = torch.from_numpy(u).cuda()
    for temperature, top_k in ((0.0, 0), (0.9, 32)):
        want = _core.sample(x, temperature, top_k, 1.0, seed=7, offset=3, uniforms=u)
        for _ in range(2):
            out = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
            rc = _static(torch, dev, out, temperature, top_k, 1.0, du, 7, 3)
            assert rc == _core.MG_OK, _lib.mg_last_error().decode()
            torch.cuda.synchronize()
            np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_static_sampler_leaves_free_memory_unchanged() -> None:
    torch = pytest.importorskip("torch")
    batch, vocab = 4, 262144
    dev = torch.from_numpy(_logits(batch, vocab, seed=3)).cuda()
    outs = [torch.full((batch,), -1, dtype=torch.int32, device="cuda") for _ in range(8)]
    assert _static(torch, dev, outs[0], 0.8, 16, 1.0, None, 1, 0) == _core.MG_OK  # first call loads the kernels
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for k, out in enumerate(outs):
        assert _static(torch, dev, out, 0.8, 16, 1.0, None, 1, k) == _core.MG_OK, _lib.mg_last_error().decode()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_static_sampler_rejects_out_of_range() -> None:
    torch = pytest.importorskip("torch")
    dev = torch.zeros((MAX_ROWS + 1, 128), dtype=torch.float32, device="cuda")
    out = torch.zeros(MAX_ROWS + 1, dtype=torch.int32, device="cuda")
    rc = _static(torch, dev, out, 0.0, 0, 1.0, None, 0, 0)
    assert rc == _core.MG_ERR_INVALID
    assert f"batch {MAX_ROWS + 1}" in _lib.mg_last_error().decode()
    big = torch.zeros((1, 262144), dtype=torch.float32, device="cuda")
    rc = _static(torch, big, out, 1.0, 0, 1.0, None, 0, 0)  # no top-k filter: every token is a candidate
    assert rc == 6  # MG_ERR_UNSUPPORTED
    assert "top_k" in _lib.mg_last_error().decode()
