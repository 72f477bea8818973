"""The oracle's bidirectional encoder (ref_encode_sequence) on its own: identities
that tie it to the causal embedding path the reference tests pin."""

from __future__ import annotations

import numpy as np

import oracle
from mogemma_b200 import synth


def _model(mode: int = 0):
    d = synth.tiny(window=4)
    w = synth.make_weights(d, seed=5)
    return d, w, oracle.RefModel(w, max_seq_len=32, mode=mode, sliding_window=d.window)


def test_one_token_encode_is_normalised_causal_embedding() -> None:
    d, _, ref = _model()
    for t in (0, 7, d.vocab - 1):
        e = ref.embed([t])
        np.testing.assert_allclose(ref.encode([t]), e / np.linalg.norm(e), rtol=0, atol=1e-6)


def test_encode_unit_norm_and_identity_head() -> None:
    d, _, ref = _model(mode=1)
    ids = [int(t) for t in synth.prompt_ids(11, d.vocab, seed=2)]
    plain = ref.encode(ids)
    assert abs(float(np.linalg.norm(plain)) - 1.0) < 1e-5
    eye = np.eye(d.hidden, dtype=np.float32)
    np.testing.assert_allclose(ref.encode(ids, eye, eye), plain, rtol=0, atol=1e-6)


def test_encode_sees_later_tokens() -> None:
    """Changing the last token moves every state, so the pooled vector differs
    from the causal one (where the earlier states are fixed)."""
    d, _, ref = _model()
    ids = [int(t) for t in synth.prompt_ids(9, d.vocab, seed=3)]
    alt = ids[:-1] + [(ids[-1] + 1) % d.vocab]
    causal = ref.embed(ids)
    bidir = ref.encode(ids)
    assert float(np.max(np.abs(bidir - causal / np.linalg.norm(causal)))) > 1e-3
    assert float(np.max(np.abs(ref.encode(alt) - bidir))) > 1e-4
