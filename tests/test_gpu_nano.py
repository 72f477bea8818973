"""Gemma 3n ("nano") decode on the device against the nano oracle (oracle/ref_nano.c).

A 12-layer synthetic model covers every part of forward_nano_step
(src/mo/mogemma/layers.mojo:959-1004): AltUp predict/correct with non-trivial
coefficients, Laurel, per-layer inputs and mapping, activation sparsity in
layers 0-9 and dense MLPs after, and KV sharing from layer 8 (full-attention
layer 9 reads layer 4's cache, the others layer 7's).  Tolerance as for the
standard path: max |dev - ref| <= 1e-5 + 2e-4 max |ref| (fp32, other
summation order).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle_nano
from mogemma_b200 import _core, synth

pytestmark = pytest.mark.gpu

D = synth.nano_tiny()
SCALES = {"altup.prediction_coefs": 10.0, "altup.correction_coefs": 10.0, "altup.router.weight": 50.0}


def close(dev: np.ndarray, ref: np.ndarray) -> None:
    err = float(np.max(np.abs(dev - ref)))
    assert err <= 1e-5 + 2e-4 * float(np.max(np.abs(ref))), err


@pytest.fixture(scope="module")
def weights() -> dict[str, np.ndarray]:
    return synth.make_nano_weights(D, seed=5, scales=SCALES)


def test_init_keys(weights) -> None:
    llm = _core.init_model(synth.metadata_of(weights), capacity=64)
    assert llm["arch"] == "nano"
    assert llm["num_layers"] == D.layers
    assert llm["per_layer_dim"] == D.per_layer_dim
    assert llm["kv_share_start"] == D.kv_share_start
    assert llm["head_dim"] == D.head_dim
    llm["_handle"].close()


def test_step_logits_match_oracle(weights) -> None:
    llm = _core.init_model(synth.metadata_of(weights), capacity=64)
    ref = oracle_nano.NanoRefModel(weights, max_seq_len=64)
    for t in synth.prompt_ids(10, D.vocab, seed=9):
        close(_core.step(llm, int(t), 0.0, 0, 1.0), ref.step(int(t)))
    assert llm["pos"] == 10
    llm["_handle"].close()


def test_prefill_then_greedy_stream_equals_oracle(weights) -> None:
    llm = _core.init_model(synth.metadata_of(weights), capacity=64)
    ref = oracle_nano.NanoRefModel(weights, max_seq_len=64)
    prompt = [int(t) for t in synth.prompt_ids(12, D.vocab, seed=3)]
    _core.prefill(llm, prompt[:-1])
    for t in prompt[:-1]:
        ref.step_no_logits(t)
    cur_d = cur_r = prompt[-1]
    for _ in range(16):
        lg = ref.step(cur_r)
        top2 = np.sort(lg)[-2:]
        cur_r = int(np.argmax(lg))
        cur_d = _core.step_sample(llm, cur_d, 0.0, 0, 1.0)
        assert cur_d == cur_r, f"margin {top2[1] - top2[0]:.3e}"
    llm["_handle"].close()


def test_embeddings_match_oracle(weights) -> None:
    llm = _core.init_model(synth.metadata_of(weights), capacity=64)
    rows = [[int(t) for t in synth.prompt_ids(n, D.vocab, seed=20 + n)] for n in (3, 7)]
    got = _core.generate_embeddings(llm, rows)
    for i, r in enumerate(rows):
        want = oracle_nano.NanoRefModel(weights, max_seq_len=64).embed(r)
        close(got[i], want)
    llm["_handle"].close()


def test_sequence_length_exceeded(weights) -> None:
    llm = _core.init_model(synth.metadata_of(weights), capacity=3)
    for t in (1, 2, 3):
        _core.step(llm, t, 0.0, 0, 1.0)
    with pytest.raises(RuntimeError, match="Sequence length exceeded"):
        _core.step(llm, 4, 0.0, 0, 1.0)
    llm["_handle"].close()
