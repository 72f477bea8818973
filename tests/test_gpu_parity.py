"""Parity of the CUDA engine (through the C ABI / _core shim) with the oracle.

Tolerances (fp32 arithmetic, different summation order than the reference):
  logits: max |dev - ref| <= LOGIT_ATOL + LOGIT_RTOL * max|ref|
  greedy: identical token streams (the top-1/top-2 margin is reported on failure)
  sampling: identical token for identical logits and uniform variate; top-k
  index sets identical.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

import oracle
from mogemma_b200 import _core, synth

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 2e-4
LOGIT_ATOL = 1e-5
GOLD = Path(__file__).resolve().parent / "golden"


def close_logits(dev: np.ndarray, ref: np.ndarray) -> None:
    err = float(np.max(np.abs(dev - ref)))
    scale = float(np.max(np.abs(ref)))
    assert err <= LOGIT_ATOL + LOGIT_RTOL * scale, f"max err {err:.3e} vs scale {scale:.3e}"


def margin(logits: np.ndarray) -> float:
    top2 = np.sort(logits)[-2:]
    return float(top2[1] - top2[0])


def build(d: synth.Gemma3Dims, *, seed: int = 0, bf16: bool = False, **opts):
    w = synth.make_weights(d, seed=seed, bf16=bf16)
    llm = _core.init_model(synth.metadata_of(w), **opts)
    return w, llm


TINY = synth.tiny()


@pytest.mark.parametrize("decode_path", [0, 1])
def test_decode_logits_match_oracle(decode_path: int) -> None:
    w, llm = build(TINY, decode_path=decode_path)
    ref = oracle.RefModel(w)
    toks = synth.prompt_ids(24, TINY.vocab, seed=3)
    for t in toks:
        dev = _core.step(llm, int(t), 0.0, 0, 1.0)
        close_logits(dev, ref.step(int(t)))
    assert llm["pos"] == len(toks)


def test_persistent_and_phase_paths_bit_identical() -> None:
    w = synth.make_weights(TINY, seed=5)
    a = _core.init_model(synth.metadata_of(w), decode_path=0)
    b = _core.init_model(synth.metadata_of(w), decode_path=1)
    for t in synth.prompt_ids(10, TINY.vocab, seed=9):
        np.testing.assert_array_equal(_core.step(a, int(t), 0, 0, 1), _core.step(b, int(t), 0, 0, 1))


def test_bf16_weights_match_oracle_on_upcast() -> None:
    w, llm = build(TINY, bf16=True, weight_dtype="bf16")
    ref = oracle.RefModel(w)
    for t in synth.prompt_ids(12, TINY.vocab, seed=4):
        close_logits(_core.step(llm, int(t), 0.0, 0, 1.0), ref.step(int(t)))


@pytest.mark.parametrize(("heads", "kv_heads", "head_dim", "qk_norm"), [(6, 2, 48, True), (2, 1, 256, False)])
def test_odd_shapes_and_missing_qk_norm(heads: int, kv_heads: int, head_dim: int, qk_norm: bool) -> None:
    # without q_norm the reference infers head_dim = 256 (core.mojo:319-321)
    d = synth.tiny(hidden=200, layers=3, heads=heads, kv_heads=kv_heads, head_dim=head_dim, intermediate=300,
                   vocab=1000, qk_norm=qk_norm)
    w, llm = build(d)
    ref = oracle.RefModel(w)
    for t in synth.prompt_ids(20, d.vocab, seed=11):
        close_logits(_core.step(llm, int(t), 0.0, 0, 1.0), ref.step(int(t)))


def test_gemma3_window_and_dual_theta() -> None:
    d = synth.tiny(layers=6, window=8)
    w, llm = build(d, mode="gemma3", sliding_window=8, global_every=3)
    ref = oracle.RefModel(w, mode=1, sliding_window=8, global_every=3)
    for t in synth.prompt_ids(40, d.vocab, seed=12):
        close_logits(_core.step(llm, int(t), 0.0, 0, 1.0), ref.step(int(t)))


def test_prefill_matches_stepwise_and_kv_cache() -> None:
    w, llm = build(TINY)
    ref = oracle.RefModel(w)
    toks = [int(t) for t in synth.prompt_ids(37, TINY.vocab, seed=6)]
    _core.prefill(llm, toks[:-1])
    for t in toks[:-1]:
        ref.step_no_logits(t)
    assert llm["pos"] == len(toks) - 1
    for layer in (0, TINY.layers - 1):
        for p in (0, 17, len(toks) - 2):
            kd, vd = _core.read_kv(llm, layer, p)
            kr, vr = ref.kv_row(layer, p)
            np.testing.assert_allclose(kd, kr, rtol=1e-4, atol=1e-5)
            np.testing.assert_allclose(vd, vr, rtol=1e-4, atol=1e-5)
    close_logits(_core.step(llm, toks[-1], 0, 0, 1), ref.step(toks[-1]))


def test_greedy_stream_identical() -> None:
    w, llm = build(TINY)
    ref = oracle.RefModel(w)
    toks = [int(t) for t in synth.prompt_ids(16, TINY.vocab, seed=7)]
    _core.prefill(llm, toks[:-1])
    dev_stream = _core.generate(llm, toks[-1], 24, 0.0, 50, 1.0)
    for t in toks[:-1]:
        ref.step_no_logits(t)
    cur, ref_stream, margins = toks[-1], [], []
    for _ in range(24):
        lg = ref.step(cur)
        cur = int(np.argmax(lg))
        ref_stream.append(cur)
        margins.append(margin(lg))
    assert dev_stream == ref_stream, f"margins {margins}"


def test_batched_rows_match_independent_runs() -> None:
    w, llm = build(TINY, max_batch=4)
    rows = [[int(t) for t in synth.prompt_ids(n, TINY.vocab, seed=20 + n)] for n in (5, 9, 1, 14)]
    _core.prefill_rows(llm, [r[:-1] for r in rows])
    lg, _ = _core.step_rows(llm, [r[-1] for r in rows])
    for i, r in enumerate(rows):
        ref = oracle.RefModel(w)
        for t in r[:-1]:
            ref.step_no_logits(t)
        close_logits(lg[i], ref.step(r[-1]))


def test_rows_beyond_the_kernel_rows_in_fp32() -> None:
    """12 rows on a model created with prefill_path 0: the decode kernel runs one launch per row group
    (two launches of 6 rows when a launch holds 8), each row in the reference's fp32 arithmetic at its own
    position."""
    w, llm = build(TINY, max_batch=12, capacity=64)
    assert 1 <= llm["_handle"].rows_per_launch <= 8
    rows = [[int(t) for t in synth.prompt_ids(3 + 2 * i, TINY.vocab, seed=50 + i)] for i in range(12)]
    _core.prefill_rows(llm, [r[:-1] for r in rows])
    assert llm["_handle"].get_pos()[:12] == [len(r) - 1 for r in rows]
    lg, drawn = _core.step_rows(llm, [r[-1] for r in rows], sampling=(0.0, 0, 1.0))
    for i, r in enumerate(rows):
        ref = oracle.RefModel(w, max_seq_len=64)
        for t in r[:-1]:
            ref.step_no_logits(t)
        close_logits(lg[i], ref.step(r[-1]))
        assert int(drawn[i]) == int(np.argmax(lg[i]))
    # sampled draws of the second group use their own Philox rows: a fixed seed repeats them
    us = np.linspace(0.05, 0.95, 12)
    _, tok = _core.step_rows(llm, [int(t) for t in drawn], sampling=(0.8, 20, 1.0), uniforms=us)
    assert ((tok >= 0) & (tok < TINY.vocab)).all()


def test_models_with_different_stages_interleave() -> None:
    """Two models of one process whose kernels need different shared-memory stages (1 and 8 rows) step in
    turn: the kernel's allowance is raised for the larger one and never lowered for the smaller one."""
    w = synth.make_weights(TINY, seed=6)
    small = _core.init_model(synth.metadata_of(w), capacity=64)
    big = _core.init_model(synth.metadata_of(w), max_batch=8, capacity=64)
    small2 = _core.init_model(synth.metadata_of(w), capacity=64)
    ref = oracle.RefModel(w, max_seq_len=64)
    for t in synth.prompt_ids(4, TINY.vocab, seed=2):
        want = ref.step(int(t))
        close_logits(_core.step(small, int(t), 0.0, 0, 1.0), want)
        lg, _tok = _core.step_rows(big, [int(t)] * 8, sampling=(0.0, 0, 1.0))
        close_logits(lg[7], want)
        close_logits(_core.step(small2, int(t), 0.0, 0, 1.0), want)
    for m in (small, big, small2):
        m["_handle"].close()


def _split_phases(d: synth.Gemma3Dims, esz: int, ctas: int) -> set[str]:
    """Phases whose row groups the kernel splits between two CTAs: the tile shape and the rule of gemv_geom."""
    out = set()
    if esz == 4:
        return out  # only the bf16 kernels split
    hp, ip, ap = (-(-k // 128) * 128 for k in (d.hidden, d.intermediate, d.heads * d.head_dim))
    for name, n, kp, pair in (("QKV", (d.heads + 2 * d.kv_heads) * d.head_dim, hp, False), ("O", d.hidden, ap, False),
                              ("GU", d.intermediate, hp, True), ("D", d.hidden, ip, False)):
        rps = 8 * (2 if esz == 2 else 1)
        nseg = max(1, -(-kp * rps * (2 if pair else 1) * esz // 36864))
        while kp % nseg or (kp // nseg) % 8:
            nseg += 1
        groups = -(-n // rps)
        units = groups * nseg
        if nseg > 1 and units // ctas >= nseg and -(-groups // ctas) * nseg - -(-units // ctas) >= 2:
            out.add(name)
    return out


@pytest.mark.parametrize(("hidden", "inter", "bf16", "want"),
                         [(1536, 2560, True, {"GU"}), (2560, 4096, True, {"D"}), (1280, 4096, False, set())])
def test_split_row_groups_match_oracle(monkeypatch, hidden: int, inter: int, bf16: bool, want: set) -> None:
    """bf16 shapes whose whole row groups leave some CTAs two or more tiles above the even share (as
    Gemma3-4B's down_proj: 160 groups on 148 CTAs) split the (group, segment) tiles evenly; the two CTAs of
    a split group add their partial sums.  Logits at 1 and 3 rows match the oracle, with and without the
    split; the fp32 kernels never split."""
    import torch  # noqa: PLC0415

    d = synth.tiny(hidden=hidden, layers=2, heads=4, kv_heads=1, head_dim=256, intermediate=inter, vocab=2048)
    assert _split_phases(d, 2 if bf16 else 4, torch.cuda.get_device_properties(0).multi_processor_count) == want
    w = synth.make_weights(d, seed=8, bf16=bf16)
    wd = "bf16" if bf16 else "f32"
    rows = [[int(t) for t in synth.prompt_ids(n, d.vocab, seed=60 + n)] for n in (5, 9, 3)]
    for split in ("1", "0"):
        monkeypatch.setenv("MOGEMMA_B200_SPLIT", split)
        one = _core.init_model(synth.metadata_of(w), capacity=64, weight_dtype=wd)
        three = _core.init_model(synth.metadata_of(w), max_batch=3, capacity=64, weight_dtype=wd)
        ref = oracle.RefModel(w, max_seq_len=64)
        for t in rows[1]:
            close_logits(_core.step(one, t, 0.0, 0, 1.0), ref.step(t))
        _core.prefill_rows(three, [r[:-1] for r in rows])
        lg, _tok = _core.step_rows(three, [r[-1] for r in rows], sampling=(0.0, 0, 1.0))
        for i, r in enumerate(rows):
            ref = oracle.RefModel(w, max_seq_len=64)
            for t in r[:-1]:
                ref.step_no_logits(t)
            close_logits(lg[i], ref.step(r[-1]))
        one["_handle"].close()
        three["_handle"].close()


@pytest.mark.parametrize("params", [(0.0, 50, 1.0), (0.7, 64, 1.0), (0.7, 10, 0.9), (1.0, 3, 1.0)])
def test_fused_draw_matches_rules_on_device_logits(params: tuple[float, int, float]) -> None:
    w, llm = build(TINY)
    rng = np.random.default_rng(0)
    for t in synth.prompt_ids(12, TINY.vocab, seed=8):
        u = float(rng.random())
        lg, tok = _core.step_rows(llm, [int(t)], sampling=params, uniforms=[u])
        want = oracle.sample_next_token(lg[0], temperature=params[0], top_k=params[1], top_p=params[2], u=u)
        assert int(tok[0]) == want


def test_general_sampler_matches_reference_golden() -> None:
    import make_golden  # noqa: PLC0415

    for case in json.loads((GOLD / "sampling.json").read_text()):
        logits = make_golden.logits_for(case)
        got = _core.sample(logits, case["temperature"], case["top_k"], case["top_p"], uniforms=[case["u"]])
        assert int(got[0]) == case["expected"], case


def test_topk_set_identical_on_identical_logits() -> None:
    rng = np.random.default_rng(1)
    logits = rng.standard_normal(262144).astype(np.float32)
    us = np.linspace(0.001, 0.999, 100)
    rows = np.repeat(logits[None, :], len(us), 0)
    for k in (1, 7, 64):
        # a huge temperature makes the kept tokens near-equiprobable, so 100
        # evenly spaced variates hit every kept index exactly once or more
        toks = _core.sample(rows, 1e6, k, 1.0, uniforms=us)
        assert {int(x) for x in toks} == oracle.top_k_set(logits, k)


def test_embeddings_mean_pool_match_oracle() -> None:
    w, llm = build(TINY, max_batch=2)
    seqs = [[int(t) for t in synth.prompt_ids(n, TINY.vocab, seed=30 + n)] for n in (3, 11, 6)]
    emb = _core.generate_embeddings(llm, seqs)
    assert emb.shape == (3, TINY.hidden)
    for i, s in enumerate(seqs):
        ref = oracle.RefModel(w)
        np.testing.assert_allclose(emb[i], ref.embed(s, ref_compat=False), rtol=2e-4, atol=2e-5)


def test_sequence_length_exceeded_and_bad_token() -> None:
    w, llm = build(TINY, capacity=4)
    for t in range(4):
        _core.step(llm, t, 0, 0, 1)
    with pytest.raises(RuntimeError, match="Sequence length exceeded"):
        _core.step(llm, 1, 0, 0, 1)
    llm["pos"] = 0
    with pytest.raises(ValueError, match="out of range"):
        _core.step(llm, TINY.vocab + 5, 0, 0, 1)
    _core.step(llm, 3, 0, 0, 1)  # model still usable


def test_gemma3_1b_full_size_decode_matches_oracle() -> None:
    d = synth.CONFIGS["gemma3-1b"]
    w = synth.make_weights(d, seed=0)
    llm = _core.init_model(synth.metadata_of(w), capacity=1024)
    oracle.set_threads(oracle.default_threads())
    ref = oracle.RefModel(w, max_seq_len=1024)
    toks = [int(t) for t in synth.prompt_ids(6, d.vocab, seed=1)]
    _core.prefill(llm, toks[:-1])
    for t in toks[:-1]:
        ref.step_no_logits(t)
    cur = toks[-1]
    for _ in range(3):
        dev = _core.step(llm, cur, 0, 0, 1)
        lg = ref.step(cur)
        close_logits(dev, lg)
        assert int(np.argmax(dev)) == int(np.argmax(lg)), f"margin {margin(lg)}"
        cur = int(np.argmax(lg))
    oracle.set_threads(1)
