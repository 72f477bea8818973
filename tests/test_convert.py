"""Orbax -> HuggingFace conversion (src/py/mogemma/convert.py:124-149; its tests
src/py/tests/test_convert.py:126-169) on synthetic Orbax dictionaries: names,
shapes, exact values (each HuggingFace tensor against the Orbax tensor it is
cut from), family detection, and a safetensors round trip through the loader
into the engine's weight names.  CPU only; reading a real Orbax directory needs
tensorstore, which this image lacks."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from mogemma_b200 import convert, synth
from mogemma_b200.loader import SafetensorsLoader


def _orbax(layers: int = 2, heads: int = 4, kv: int = 2, hidden: int = 32, hd: int = 8, inter: int = 48,
           vocab: int = 20, seed: int = 0) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)

    def r(*shape):
        return rng.standard_normal(shape).astype(np.float32)

    o = {"transformer/embedder.input_embedding": r(vocab, hidden), "transformer/final_norm.scale": r(hidden)}
    for n in range(layers):
        p = f"transformer/layer_{n}/"
        for k in ("pre_attention_norm", "post_attention_norm", "pre_ffw_norm", "post_ffw_norm"):
            o[p + k + ".scale"] = r(hidden)
        o[p + "attn/_query_norm.scale"] = r(hd)
        o[p + "attn/_key_norm.scale"] = r(hd)
        o[p + "attn/q_einsum.w"] = r(heads, hidden, hd)
        o[p + "attn/kv_einsum.w"] = r(2, kv, hidden, hd)
        o[p + "attn/attn_vec_einsum.w"] = r(heads, hd, hidden)
        o[p + "mlp/gating_einsum.w"] = r(2, inter, hidden)
        o[p + "mlp/linear.w"] = r(inter, hidden)
    return o


def test_reference_shapes() -> None:
    """The shapes the reference test asserts (8 heads, 2 kv heads, hd 256, hidden 2048, inter 8192)."""
    orbax = {
        "transformer/embedder.input_embedding": np.zeros((20, 2048), np.float32),
        "transformer/final_norm.scale": np.zeros((2048,), np.float32),
        "transformer/layer_0/pre_attention_norm.scale": np.zeros((2048,), np.float32),
        "transformer/layer_0/post_attention_norm.scale": np.zeros((2048,), np.float32),
        "transformer/layer_0/pre_ffw_norm.scale": np.zeros((2048,), np.float32),
        "transformer/layer_0/post_ffw_norm.scale": np.zeros((2048,), np.float32),
        "transformer/layer_0/attn/_query_norm.scale": np.zeros((256,), np.float32),
        "transformer/layer_0/attn/_key_norm.scale": np.zeros((256,), np.float32),
        "transformer/layer_0/attn/q_einsum.w": np.zeros((8, 2048, 256), np.float32),
        "transformer/layer_0/attn/kv_einsum.w": np.zeros((2, 2, 2048, 256), np.float32),
        "transformer/layer_0/attn/attn_vec_einsum.w": np.zeros((8, 256, 2048), np.float32),
        "transformer/layer_0/mlp/gating_einsum.w": np.zeros((2, 8192, 2048), np.float32),
        "transformer/layer_0/mlp/linear.w": np.zeros((8192, 2048), np.float32),
    }
    hf = convert.convert_tensors(orbax)
    l0 = "model.layers.0"
    assert hf[f"{l0}.self_attn.q_proj.weight"].shape == (8 * 256, 2048)
    assert hf[f"{l0}.self_attn.k_proj.weight"].shape == (2 * 256, 2048)
    assert hf[f"{l0}.self_attn.v_proj.weight"].shape == (2 * 256, 2048)
    assert hf[f"{l0}.self_attn.o_proj.weight"].shape == (2048, 8 * 256)
    assert hf[f"{l0}.mlp.gate_proj.weight"].shape == (8192, 2048)
    assert hf[f"{l0}.mlp.up_proj.weight"].shape == (8192, 2048)
    assert hf[f"{l0}.mlp.down_proj.weight"].shape == (2048, 8192)
    assert hf["lm_head.weight"] is hf["model.embed_tokens.weight"]


def test_values_follow_the_einsum_layouts() -> None:
    o = _orbax()
    hf = convert.convert_tensors(o)
    heads, hidden, hd = o["transformer/layer_1/attn/q_einsum.w"].shape
    q = hf["model.layers.1.self_attn.q_proj.weight"]
    for h in range(heads):  # row h*hd + j of q_proj is q_einsum[h, :, j]
        np.testing.assert_array_equal(q[h * hd:(h + 1) * hd], o["transformer/layer_1/attn/q_einsum.w"][h].T)
    kv = o["transformer/layer_1/attn/kv_einsum.w"]
    k, v = hf["model.layers.1.self_attn.k_proj.weight"], hf["model.layers.1.self_attn.v_proj.weight"]
    np.testing.assert_array_equal(k[hd:2 * hd], kv[0, 1].T)
    np.testing.assert_array_equal(v[:hd], kv[1, 0].T)
    ov = o["transformer/layer_1/attn/attn_vec_einsum.w"]
    o_proj = hf["model.layers.1.self_attn.o_proj.weight"]
    np.testing.assert_array_equal(o_proj[:, 2 * hd:3 * hd], ov[2].T)  # column h*hd + j is attn_vec[h, j, :]
    g = o["transformer/layer_1/mlp/gating_einsum.w"]
    np.testing.assert_array_equal(hf["model.layers.1.mlp.gate_proj.weight"], g[0])
    np.testing.assert_array_equal(hf["model.layers.1.mlp.up_proj.weight"], g[1])
    np.testing.assert_array_equal(hf["model.layers.1.mlp.down_proj.weight"], o["transformer/layer_1/mlp/linear.w"].T)
    np.testing.assert_array_equal(hf["model.layers.0.input_layernorm.weight"],
                                  o["transformer/layer_0/pre_attention_norm.scale"])
    assert all(a.dtype == np.float32 for a in hf.values())


def test_projection_math_is_preserved() -> None:
    """x @ W^T of a converted projection equals the Orbax einsum it came from."""
    o = _orbax(seed=3)
    hf = convert.convert_tensors(o)
    x = np.random.default_rng(1).standard_normal(32).astype(np.float64)
    qe = o["transformer/layer_0/attn/q_einsum.w"].astype(np.float64)
    want = np.einsum("d,hdk->hk", x, qe).reshape(-1)
    np.testing.assert_allclose(hf["model.layers.0.self_attn.q_proj.weight"].astype(np.float64) @ x, want, rtol=1e-6)
    a = np.random.default_rng(2).standard_normal((4, 8))
    ve = o["transformer/layer_0/attn/attn_vec_einsum.w"].astype(np.float64)
    want_o = np.einsum("hk,hkd->d", a, ve)
    np.testing.assert_allclose(hf["model.layers.0.self_attn.o_proj.weight"].astype(np.float64) @ a.reshape(-1),
                               want_o, rtol=1e-6)


def test_family_detection_and_errors() -> None:
    assert convert.detect_family(["transformer/embedder.input_embedding", "transformer/layer_0/attn/q_einsum.w"]) == \
        "gemma3"
    assert convert.detect_family(["transformer/layer_0/altup.modality_router.w"]) == "gemma3_nano"
    assert convert.detect_family(["transformer/layer_0/per_layer_mapping.per_layer_input_gate.w"]) == "gemma3_nano"
    o = _orbax()
    o["transformer/layer_0/altup.modality_router.w"] = np.zeros((2, 2), np.float32)
    with pytest.raises(ValueError, match="nano"):
        convert.convert_tensors(o)
    o = _orbax()
    del o["transformer/layer_1/mlp/linear.w"]
    with pytest.raises(KeyError, match="layer_1/mlp/linear.w"):
        convert.convert_tensors(o)


def test_bf16_sources_widen_to_f32() -> None:
    o = _orbax()
    bits = (o["transformer/layer_0/mlp/linear.w"].view(np.uint32) & 0xFFFF0000).view(np.float32)
    o["transformer/layer_0/mlp/linear.w"] = bits.astype(np.float64)  # any float source dtype
    hf = convert.convert_tensors(o)
    assert hf["model.layers.0.mlp.down_proj.weight"].dtype == np.float32
    np.testing.assert_array_equal(hf["model.layers.0.mlp.down_proj.weight"], bits.T)


def test_safetensors_round_trip_into_engine_names(tmp_path: Path) -> None:
    o = _orbax(layers=3, seed=5)
    path = convert.write_safetensors(o, tmp_path / "ckpt")
    want = convert.convert_tensors(o)
    with SafetensorsLoader(path.parent) as ld:
        assert set(ld.tensors) == set(want)
        for name, arr in want.items():
            np.testing.assert_array_equal(ld.array(name), arr)
        # every name the engine reads for these dimensions is present
        d = synth.tiny(hidden=32, layers=3, heads=4, kv_heads=2, head_dim=8, intermediate=48, vocab=20)
        assert set(synth.tensor_shapes(d)) | {"lm_head.weight"} == set(ld.tensors)
        for name, shape in synth.tensor_shapes(d).items():
            assert ld.tensors[name].shape == shape


def test_reading_orbax_without_tensorstore_says_so(tmp_path: Path) -> None:
    pytest.importorskip("numpy")
    try:
        import tensorstore  # noqa: F401, PLC0415
    except ModuleNotFoundError:
        with pytest.raises(ModuleNotFoundError, match="tensorstore"):
            convert.read_orbax(tmp_path)
    else:
        pytest.skip("tensorstore is installed")
