"""Bidirectional encoder embeddings (mg_encode) against the oracle's ref_encode_sequence.

The device path rounds the projection inputs and weights to bf16 (prefill_path 1),
so the bound is the bf16 one of the batched prefill:
  max |dev - ref| <= ENC_TOL * max |ref|  per row (rows are unit vectors).
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from mogemma_b200 import _core, synth

pytestmark = pytest.mark.gpu

ENC_TOL = 2e-2


@pytest.mark.parametrize(("mode", "head", "lens", "hd"), [(0, False, (1, 17, 40, 5, 33), 64),
                                                         (1, True, (1, 17, 40, 5, 33), 64),
                                                         (1, False, (300, 129, 7), 64), (0, True, (257, 64), 64),
                                                         (1, True, (200, 3, 61), 128), (1, False, (150, 20), 256),
                                                         (0, False, (140,), 256), (1, True, (600, 100), 4096)])
def test_encode_matches_oracle(mode: int, head: bool, lens: tuple[int, ...], hd: int) -> None:
    """Short rows (one key block), and rows over several 128-query tiles and
    128-key blocks, with the 16-token window on local layers in mode 1; head
    dims 64, 128 and 256 (each a tensor-core attention instantiation).  hd 4096
    marks the wide-MLP case (head dim 128, intermediate 4096): 700 tokens give
    the persistent GEMM with the fused GeGLU epilogue."""
    d = synth.tiny(window=16, head_dim=128, intermediate=4096) if hd == 4096 else synth.tiny(window=16, head_dim=hd)
    w = synth.make_weights(d, seed=21)
    d0 = d1 = None
    if head:
        rng = np.random.default_rng(4)
        d0 = (rng.standard_normal((384, d.hidden)) * 0.05).astype(np.float32)
        d1 = (rng.standard_normal((d.hidden, 384)) * 0.05).astype(np.float32)
        w["embed_head.dense0.weight"] = d0
        w["embed_head.dense1.weight"] = d1
    rows = [[int(t) for t in synth.prompt_ids(n, d.vocab, seed=60 + i)] for i, n in enumerate(lens)]
    llm = _core.init_model(synth.metadata_of(w), prefill_path=1, max_batch=2, capacity=max(lens) + 8,
                           mode="gemma3" if mode else "ref", sliding_window=d.window)
    out = _core.encode_embeddings(llm, rows)
    assert out.shape == (len(rows), d.hidden)
    ref = oracle.RefModel(w, max_seq_len=max(lens) + 8, mode=mode, sliding_window=d.window)
    for b, r in enumerate(rows):
        e = ref.encode(r, d0, d1)
        assert float(np.max(np.abs(out[b] - e))) <= ENC_TOL * float(np.max(np.abs(e))), (b, len(r))
        assert abs(float(np.linalg.norm(out[b])) - 1.0) < 1e-4


def test_encode_rejects_token_path_model() -> None:
    d = synth.tiny()
    w = synth.make_weights(d, seed=1)
    llm = _core.init_model(synth.metadata_of(w), capacity=16)
    with pytest.raises(RuntimeError, match="prefill_path 1"):
        _core.encode_embeddings(llm, [[1, 2, 3]])
