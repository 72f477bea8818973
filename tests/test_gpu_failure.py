"""Failure detection of the decode kernel's bounded waits, without a GPU fault.

A test hook (mg_set_debug) gives every wait of the decode kernel a short
budget and makes one CTA withhold its outputs of one phase -- a flag that
nothing sets.  The CTAs waiting on them must give up within the budget, record the
site, fast-forward to the kernel's end and return: the call reports
MG_ERR_TIMEOUT ("gave up waiting"), the row's position is restored, and after
the hook is cleared the next step at the same position matches the oracle.
Every kind of hand-off is covered: tagged words (q/k/v, o_proj output,
down_proj output), counters (attention partials, gate/up output) and the
lm_head -> draw counter.
"""

from __future__ import annotations

import time

import numpy as np
import pytest

import oracle
from mogemma_b200 import _core, synth

pytestmark = pytest.mark.gpu

D = synth.tiny(layers=2)
BUDGET_NS = 50_000_000  # 50 ms


@pytest.fixture(scope="module")
def model():
    w = synth.make_weights(D, seed=3)
    llm = _core.init_model(synth.metadata_of(w), capacity=64)
    yield w, llm
    llm["_handle"].close()


# phase = 5 * layer + {0 QKV, 1 attention, 2 o_proj, 3 gate/up, 4 down}; 5 * layers: lm_head
@pytest.mark.parametrize("phase", [0, 1, 2, 3, 4, 5 + 2, 5 * D.layers])
def test_withheld_phase_times_out_and_model_recovers(model, phase: int) -> None:
    w, llm = model
    h = llm["_handle"]
    toks = [int(t) for t in synth.prompt_ids(6, D.vocab, seed=phase)]
    h.set_pos(0)
    llm["pos"] = 0
    _core.prefill(llm, toks[:4])
    h.set_debug(BUDGET_NS, phase)
    t0 = time.perf_counter()
    with pytest.raises(RuntimeError, match="gave up waiting"):
        _core.step(llm, toks[4], 0.0, 0, 1.0) if phase != 5 * D.layers else \
            _core.step_rows(llm, [toks[4]], sampling=(0.7, 16, 1.0))
    elapsed = time.perf_counter() - t0
    assert elapsed < 5.0, elapsed  # the 50 ms budget, not the 2 s default, ended the waits
    assert h.get_pos()[0] == 4  # the failed step did not advance the row
    h.set_debug(0, -1)
    llm["pos"] = 4
    ref = oracle.RefModel(w, max_seq_len=64)
    for t in toks[:4]:
        ref.step_no_logits(t)
    for t in toks[4:]:
        dev, want = _core.step(llm, t, 0.0, 0, 1.0), ref.step(t)
        err = float(np.max(np.abs(dev - want)))
        assert err <= 1e-5 + 2e-4 * float(np.max(np.abs(want))), err


def test_debug_hook_rejects_unknown_phase(model) -> None:
    _w, llm = model
    with pytest.raises(ValueError, match="stall_phase"):
        llm["_handle"].set_debug(0, 5 * D.layers + 2)
