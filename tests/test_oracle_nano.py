"""The Gemma 3n ("nano") oracle (oracle/ref_nano.c) against the reference's own
nano tests and an independent float64 NumPy restatement.

* Known answers of src/mo/tests/test_nano_layers.mojo (Laurel 2.0, per-layer
  mapping ~1.0, AltUp predict/correct identity, a layer with non-zero output)
  and src/mo/tests/test_altup_contract.mojo (predictions and corrections 1.0).
* init keys of src/py/tests/test_mojo_core.py:86-204 (arch, num_layers,
  head_dim, per_layer_dim; 3-D per-layer tables) and the zero-weight step
  (logits shape, pos advances).
* A 12-layer random model (sparse and dense MLPs, full and sliding KV sharing
  from layer 8): logits, KV-share detection and the mean-pooled embedding match
  a float64 NumPy restatement of layers.mojo:121-171, 373-1063 written
  independently of the C code.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
from scipy.special import erf

import oracle  # noqa: F401  (builds libmg_oracle.so on first use)
from mogemma_b200 import synth
import oracle_nano as nano

H4, NM4 = 4, 4


def test_laurel_known_answer() -> None:
    # test_nano_layers.mojo:17-46: all-ones weights, x = 1 -> 1 + norm(up(down(x))) = 2
    out = nano.laurel(np.ones(H4), np.ones((2, H4)), np.ones((H4, 2)), np.ones(H4))
    np.testing.assert_allclose(out, 2.0, atol=1e-5)


def test_per_layer_mapping_known_answer() -> None:
    # test_nano_layers.mojo:49-85: all-ones weights and inputs settle near 1.0
    out = nano.per_layer_mapping(np.ones(H4), np.ones(2), np.ones((2, H4)), np.ones((H4, 2)), np.ones(H4))
    np.testing.assert_allclose(out, 1.0, atol=1e-3)


def _identity_altup() -> dict[str, np.ndarray]:
    return {"router": np.zeros((NM4, H4)), "router_norm": np.ones(H4),
            "prediction_coefs": np.zeros((NM4, NM4, NM4)), "correction_coefs": np.zeros((NM4, NM4)),
            "output_scale": np.ones(H4)}


def test_altup_identity_contract() -> None:
    # test_altup_contract.mojo:21-72 and test_nano_layers.mojo:88-137
    altup = _identity_altup()
    pred = nano.altup_predict(np.ones((NM4, H4)), altup)
    corrected = nano.altup_correct(pred, np.ones(H4), altup)
    np.testing.assert_allclose(pred, 1.0, atol=1e-5)
    np.testing.assert_allclose(corrected, 1.0, atol=1e-5)


def test_nano_layer_output_non_zero() -> None:
    # test_nano_layers.mojo:140-252 (h 4, I 4, 2 q heads / 1 kv head of dim 2, pld 2, all-ones weights);
    # q/k norm weights are ones here (that test leaves them unset)
    h, inter, nq, nkv, hd, pld = 4, 4, 2, 1, 2, 2
    ones = np.ones
    arrays = {n: ones(h) for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                                   "post_feedforward_layernorm", "router_norm", "output_scale", "laurel_norm",
                                   "plm_norm")}
    arrays.update(q_proj=ones((nq * hd, h)), k_proj=ones((nkv * hd, h)), v_proj=ones((nkv * hd, h)),
                  o_proj=ones((h, nq * hd)), gate_proj=ones((inter, h)), up_proj=ones((inter, h)),
                  down_proj=ones((h, inter)), q_norm=ones(hd), k_norm=ones(hd), router=ones((NM4, h)),
                  prediction_coefs=ones((NM4, NM4, NM4)), correction_coefs=ones((NM4, NM4)),
                  laurel_down=ones((pld, h)), laurel_up=ones((h, pld)), plm_gate=ones((pld, h)),
                  plm_projection=ones((h, pld)))
    w, _keep = nano.layer_struct(arrays)
    out = np.zeros((NM4, h), np.float32)
    fc = np.zeros(hd, np.float32)
    fc[0] = 1.0
    fs = np.zeros(hd, np.float32)
    kc = np.zeros(10 * nkv * hd, np.float32)
    vc = np.zeros(10 * nkv * hd, np.float32)
    pli = np.ones(pld, np.float32)
    streams = np.ones((NM4, h), np.float32)
    fp = nano._fp  # noqa: SLF001
    import ctypes  # noqa: PLC0415

    nano.lib().ref_nano_layer(fp(out), fp(streams), ctypes.byref(w), 0, fp(pli), 0, h, nq, nkv, hd, inter, pld,
                              fp(fc), fp(fs), fp(kc), fp(vc), NM4, 1)
    assert np.isfinite(out).all()
    assert np.any(out != 0), "forward_nano_layer output should be non-zero"


def _zero_nano(pld: int, table_layers: int = 30, altup_mats: bool = True) -> dict[str, np.ndarray]:
    # src/py/tests/test_mojo_core.py:86-142: vocab 10, hidden 4, head dim 2, one layer, all zeros
    z = np.zeros
    t = {"model.embed_tokens.weight": z((10, 4)), "model.norm.weight": z(4), "lm_head.weight": z((10, 4)),
         "model.per_layer_embed.weight": z((10, table_layers, pld)),
         "model.per_layer_embed.projection.weight": z((4, table_layers, pld)),
         "model.per_layer_embed.norm.weight": z(pld)}
    p = "model.layers.0."
    t.update({p + "altup.router.weight": z((4, 4)), p + "altup.router_norm.weight": z(4),
              p + "altup.prediction_coefs": z((4, 4, 4)), p + "altup.correction_coefs": z((4, 4)),
              p + "altup.output_scale": z(4), p + "laurel.down_proj.weight": z((2, 4)),
              p + "laurel.up_proj.weight": z((4, 2)), p + "laurel.norm.weight": z(4),
              p + "per_layer_map.gate.weight": z((pld, 4)), p + "per_layer_map.projection.weight": z((4, pld)),
              p + "per_layer_map.norm.weight": z(4), p + "input_layernorm.weight": z(4),
              p + "post_attention_layernorm.weight": z(4), p + "self_attn.q_proj.weight": z((8, 4)),
              p + "self_attn.k_proj.weight": z((4, 4)), p + "self_attn.v_proj.weight": z((4, 4)),
              p + "self_attn.o_proj.weight": z((4, 8)), p + "mlp.gate_proj.weight": z((16, 4)),
              p + "mlp.up_proj.weight": z((16, 4)), p + "mlp.down_proj.weight": z((4, 16)),
              p + "self_attn.q_norm.weight": z(2), p + "self_attn.k_norm.weight": z(2),
              p + "pre_feedforward_layernorm.weight": z(4), p + "post_feedforward_layernorm.weight": z(4)})
    if altup_mats:
        for i in range(3):
            t[f"model.altup.projection.{i}.weight"] = z((4, 4))
            t[f"model.altup.unembed.{i}.weight"] = z((4, 4))
    return {k: np.asarray(v, np.float32) for k, v in t.items()}


@pytest.mark.parametrize("pld", [2, 256])
def test_init_keys_like_reference(pld: int) -> None:
    m = nano.NanoRefModel(_zero_nano(pld), max_seq_len=8)
    assert m.info["arch"] == "nano"
    assert m.info["num_layers"] == 1
    assert m.info["head_dim"] == 2
    assert m.info["per_layer_dim"] == pld
    assert m.info["kv_share_start"] == 1  # a single all-zero k/v layer: no earlier layer had k/v


def test_zero_weight_step_advances() -> None:
    # test_mojo_core.py:204-234: logits of vocab size, pos 1 after one step
    m = nano.NanoRefModel(_zero_nano(2), max_seq_len=8)
    logits = m.step(1)
    assert logits.shape == (10,)
    assert np.isfinite(logits).all()
    assert m.pos == 1


def test_sequence_length_exceeded() -> None:
    m = nano.NanoRefModel(_zero_nano(2), max_seq_len=2)
    m.step(1)
    m.step(2)
    with pytest.raises(RuntimeError, match="Sequence length exceeded"):
        m.step(3)


# ------------------------------------------------------------- float64 restatement
class _NpNano:
    """layers.mojo:373-1063 in float64 NumPy, written from the reference source independently of the C code."""

    def __init__(self, w: dict[str, np.ndarray], max_seq: int) -> None:
        self.w = {k: np.asarray(v, np.float64) for k, v in w.items()}
        g = self.w
        self.L = 0
        while f"model.layers.{self.L}.input_layernorm.weight" in g:
            self.L += 1
        p0 = "model.layers.0."
        self.hd = g[p0 + "self_attn.q_norm.weight"].shape[0]
        self.H = g["model.embed_tokens.weight"].shape[1]
        self.nq = g[p0 + "self_attn.q_proj.weight"].shape[0] // self.hd
        self.nkv = g[p0 + "self_attn.k_proj.weight"].shape[0] // self.hd
        self.nm = g[p0 + "altup.router.weight"].shape[0]
        self.P = g[p0 + "per_layer_map.gate.weight"].shape[0]
        self.kss = self.L
        seen = False
        for i in range(self.L):
            zero = not np.any(g[f"model.layers.{i}.self_attn.k_proj.weight"]) and \
                not np.any(g[f"model.layers.{i}.self_attn.v_proj.weight"])
            if not zero:
                seen = True
            elif seen:
                self.kss = i
                break
        self.kc = np.zeros((self.L, max_seq, self.nkv, self.hd))
        self.vc = np.zeros_like(self.kc)
        inv = 1.0 / 10000.0 ** (np.arange(0, self.hd, 2) / self.hd)
        ang = np.arange(max_seq)[:, None] * inv[None, :]
        self.cos, self.sin = np.cos(ang), np.sin(ang)
        self.pos = 0

    @staticmethod
    def rms_w(x: np.ndarray, wt: np.ndarray) -> np.ndarray:
        return x / np.sqrt(np.mean(x * x) + 1e-6) * wt

    @staticmethod
    def rms_u(x: np.ndarray) -> np.ndarray:
        return x / np.sqrt(np.mean(x * x) + 1e-6)

    @staticmethod
    def mag(v: np.ndarray) -> float:
        return float(np.sqrt(np.mean(v * v) + 1e-6))

    @staticmethod
    def gelu(x: np.ndarray) -> np.ndarray:
        return 0.5 * x * (1.0 + erf(x / math.sqrt(2.0)))

    def rope(self, v: np.ndarray, pos: int) -> np.ndarray:
        half = self.hd // 2
        c, s = self.cos[pos], self.sin[pos]
        x1, x2 = v[:half], v[half:]
        return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s])

    def modalities(self, x: np.ndarray, p: str) -> np.ndarray:
        g = self.w
        r = self.rms_w(x, g[p + "altup.router_norm.weight"]) / self.H
        return np.tanh(g[p + "altup.router.weight"] @ r)

    def layer(self, streams: np.ndarray, l: int, pli: np.ndarray) -> np.ndarray:
        g, p, pos = self.w, f"model.layers.{l}.", self.pos
        nm = self.nm
        mod = self.modalities(streams[0], p)
        pc = g[p + "altup.prediction_coefs"]  # [router][out][in]
        coef = np.einsum("roi,r->io", pc, mod)
        pred = streams + np.einsum("id,io->od", streams, coef)
        active = pred[0]
        an = self.rms_w(active, g[p + "input_layernorm.weight"])
        laurel = an + self.rms_w(g[p + "laurel.up_proj.weight"] @ (g[p + "laurel.down_proj.weight"] @ an),
                                 g[p + "laurel.norm.weight"])
        # attention (scaling 1.0); layers from kss on read the last earlier cache of their kind
        write, kv_l = True, l
        if self.kss < self.L and l >= self.kss:
            write = False
            full = [i for i in range(self.kss) if (i + 1) % 5 == 0]
            sliding = [i for i in range(self.kss) if (i + 1) % 5 != 0]
            kv_l = full[-1] if (l + 1) % 5 == 0 and full else (sliding[-1] if sliding else self.kss - 1)
        q = (g[p + "self_attn.q_proj.weight"] @ an).reshape(self.nq, self.hd)
        q = np.stack([self.rope(self.rms_w(qh, g[p + "self_attn.q_norm.weight"]), pos) for qh in q])
        if write:
            k = (g[p + "self_attn.k_proj.weight"] @ an).reshape(self.nkv, self.hd)
            v = (g[p + "self_attn.v_proj.weight"] @ an).reshape(self.nkv, self.hd)
            self.kc[l, pos] = np.stack([self.rope(self.rms_w(kh, g[p + "self_attn.k_norm.weight"]), pos) for kh in k])
            self.vc[l, pos] = np.stack([self.rms_u(vh) for vh in v])
        att = np.zeros((self.nq, self.hd))
        per = self.nq // self.nkv
        for h in range(self.nq):
            ks, vs = self.kc[kv_l, : pos + 1, h // per], self.vc[kv_l, : pos + 1, h // per]
            sc = ks @ q[h]
            e = np.exp(sc - sc.max())
            att[h] = (e / e.sum()) @ vs
        attn = g[p + "self_attn.o_proj.weight"] @ att.reshape(-1)
        al = (active + self.rms_w(attn, g[p + "post_attention_layernorm.weight"]) + laurel) * 0.7071067811865475
        ffin = self.rms_w(al, g[p + "pre_feedforward_layernorm.weight"])
        gate = g[p + "mlp.gate_proj.weight"] @ ffin
        if l < 10:
            cutoff = gate.mean() + gate.std() * 1.6448536269514722
            gate = np.maximum(gate - cutoff, 0.0)
        ff = g[p + "mlp.down_proj.weight"] @ (self.gelu(gate) * (g[p + "mlp.up_proj.weight"] @ ffin))
        activated = al + self.rms_w(ff, g[p + "post_feedforward_layernorm.weight"])
        mod2 = self.modalities(activated, p)
        corr = 1.0 + g[p + "altup.correction_coefs"].T @ mod2  # [router][out]
        corrected = pred + (activated - pred[0])[None, :] * corr[:, None]
        first = corrected[0] * g[p + "altup.output_scale"]
        delta = self.rms_w(g[p + "per_layer_map.projection.weight"]
                           @ (self.gelu(g[p + "per_layer_map.gate.weight"] @ first) * pli),
                           g[p + "per_layer_map.norm.weight"])
        out = corrected.copy()
        out[1:] += delta[None, :]
        assert out.shape == (nm, self.H)
        return out

    def hidden(self, tok: int) -> np.ndarray:
        g, H, P = self.w, self.H, self.P
        x = g["model.embed_tokens.weight"][tok] * math.sqrt(H)
        streams = [x]
        for i in range(self.nm - 1):
            pr = g[f"model.altup.projection.{i}.weight"] @ x
            streams.append(pr * (self.mag(x) / max(self.mag(pr), 1e-6)))
        streams = np.stack(streams)
        proj = g["model.per_layer_embed.projection.weight"]  # [H][T][P]
        table = g["model.per_layer_embed.weight"]  # [V][T][P]
        pli = np.stack([(self.rms_w(x @ proj[:, l, :] / math.sqrt(H), g["model.per_layer_embed.norm.weight"])
                         + table[tok, l] * math.sqrt(P)) * 0.7071067811865475 for l in range(self.L)])
        for l in range(self.L):
            streams = self.layer(streams, l, pli[l])
        target = self.mag(streams[0])
        acc = streams[0].copy()
        for m in range(1, self.nm):
            t = g[f"model.altup.unembed.{m - 1}.weight"] @ streams[m]
            acc += t * (target / max(self.mag(t), 1e-6))
        return self.rms_w(acc / self.nm, g["model.norm.weight"])

    def step(self, tok: int) -> np.ndarray:
        h = self.hidden(tok)
        self.pos += 1
        return self.w["lm_head.weight"] @ h


@pytest.fixture(scope="module")
def tiny() -> tuple[synth.NanoDims, dict[str, np.ndarray]]:
    d = synth.nano_tiny()
    w = synth.make_nano_weights(d, seed=5, scales={"altup.prediction_coefs": 10.0, "altup.correction_coefs": 10.0,
                                                   "altup.router.weight": 50.0})
    return d, w


def test_kv_share_start_detected(tiny) -> None:
    d, w = tiny
    m = nano.NanoRefModel(w, max_seq_len=16)
    assert m.info["kv_share_start"] == d.kv_share_start
    w2 = synth.make_nano_weights(synth.nano_tiny(kv_share_start=None), seed=5)
    assert nano.NanoRefModel(w2, max_seq_len=16).info["kv_share_start"] == 12


def test_step_logits_match_float64_restatement(tiny) -> None:
    d, w = tiny
    m = nano.NanoRefModel(w, max_seq_len=16)
    ref = _NpNano(w, 16)
    toks = [int(t) for t in synth.prompt_ids(7, d.vocab, seed=9)]
    for t in toks:
        got, want = m.step(t), ref.step(t)
        err = float(np.max(np.abs(got - want)))
        assert err <= 1e-5 + 1e-3 * float(np.max(np.abs(want))), err
    assert m.pos == len(toks)


def test_embedding_is_mean_of_final_hidden_states(tiny) -> None:
    d, w = tiny
    ids = [int(t) for t in synth.prompt_ids(5, d.vocab, seed=4)]
    got = nano.NanoRefModel(w, max_seq_len=16).embed(ids)
    ref = _NpNano(w, 16)
    want = np.zeros(d.hidden)
    for t in ids:
        want += ref.hidden(t)
        ref.pos += 1
    want /= len(ids)
    np.testing.assert_allclose(got, want, rtol=0, atol=1e-5 + 1e-3 * float(np.max(np.abs(want))))


def test_activation_sparsity_keeps_the_top_tail() -> None:
    g = np.random.default_rng(0).standard_normal(4096).astype(np.float32)
    out = nano.activation_sparsity(g)
    cutoff = g.mean() + g.std() * 1.6448536269514722
    np.testing.assert_allclose(out, np.maximum(g - cutoff, 0.0), atol=1e-5)
    assert 0.03 < np.mean(out > 0) < 0.07  # about the top 5 % of a normal sample stays
