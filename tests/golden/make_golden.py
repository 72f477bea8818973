"""Generate tests/golden/*.json from the reference's own Python code.

Run where a checkout of the reference is readable:
  python tests/golden/make_golden.py REFERENCE_DIR
(REFERENCE_DIR: the reference project's root, holding src/py and src/mo).

* sampling.json: outputs of the reference ``_sample_next_token``
  (src/py/mogemma/model.py:103-150) on seeded logits.  The reference draws with
  an unseeded ``np.random.default_rng()``; here that constructor is replaced by
  a seeded one for each case, and the seed is recorded so the tests can
  replay the same uniform variate.
* known_answers.json: the numeric assertions of the reference's Mojo op and
  layer tests (src/mo/tests/test_ops.mojo, src/mo/tests/test_layers.mojo),
  read from those files as text and recorded with their inputs.

The tests only read the JSON; nothing at test time reads the reference tree.
"""

from __future__ import annotations

import json
import re
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _reference_dir() -> Path:
    if len(sys.argv) != 2:  # noqa: PLR2004
        sys.exit("usage: python tests/golden/make_golden.py REFERENCE_DIR")
    return Path(sys.argv[1])


REF = _reference_dir() if __name__ == "__main__" else Path()


def _import_reference_model():
    sys.path.insert(0, str(REF / "src/py"))
    if "obstore" not in sys.modules:  # hub.py imports it at module level; unused here
        stub = types.ModuleType("obstore")
        stub.store = types.SimpleNamespace(GCSStore=object)
        sys.modules["obstore"] = stub
    import mogemma.model as ref_model  # noqa: PLC0415

    return ref_model


def logits_for(case: dict) -> np.ndarray:
    """Regenerate a case's logits (also used by the tests)."""
    rng = np.random.default_rng(case["logit_seed"])
    v = rng.standard_normal(case["vocab"]).astype(np.float32) * np.float32(case["scale"])
    for idx, val in case.get("set", []):
        v[idx] = np.float32(val)
    return v


def sampling_cases() -> list[dict]:
    cases = []
    specs = [
        # vocab, scale, temperature, top_k, top_p
        (3, 1.0, 0.0, 50, 1.0),
        (10, 1.0, 0.7, 0, 1.0),
        (10, 1.0, 1.0, 3, 1.0),
        (64, 2.0, 0.7, 10, 0.9),
        (1000, 3.0, 0.7, 64, 1.0),
        (1000, 3.0, 1.3, 64, 0.8),
        (4096, 4.0, 0.5, 0, 0.95),
        (4096, 4.0, 1.0, 200, 1.0),
        (4096, 4.0, 0.9, 2000, 0.7),
        (262144, 1.0, 0.7, 64, 1.0),
        (262144, 1.0, 0.7, 50, 0.9),
        (262144, 6.0, 1.0, 0, 1.0),
        (262144, 6.0, 0.8, 0, 0.5),
        (262144, 1.0, 0.0, 64, 1.0),
    ]
    for i, (vocab, scale, t, k, p) in enumerate(specs):
        for draw in range(3):
            cases.append({"vocab": vocab, "scale": scale, "temperature": t, "top_k": k, "top_p": p,
                          "logit_seed": 1000 + i, "draw_seed": 5000 + 17 * i + draw})
    # ties: argmax must return the first maximum
    cases.append({"vocab": 16, "scale": 0.0, "temperature": 0.0, "top_k": 0, "top_p": 1.0, "logit_seed": 7,
                  "draw_seed": 1, "set": [[3, 2.5], [9, 2.5]]})
    return cases


def make_sampling(ref_model) -> list[dict]:
    out = []
    orig = np.random.default_rng
    for case in sampling_cases():
        logits = logits_for(case)
        seed = case["draw_seed"]
        np.random.default_rng = lambda *_a, _s=seed, **_k: orig(_s)  # noqa: E731
        try:
            tok = ref_model._sample_next_token(logits, temperature=case["temperature"], top_k=case["top_k"],
                                               top_p=case["top_p"])
        finally:
            np.random.default_rng = orig
        case = dict(case)
        case["expected"] = int(tok)
        case["u"] = float(orig(seed).random())
        out.append(case)
    return out


def make_known_answers() -> dict:
    ops = (REF / "src/mo/tests/test_ops.mojo").read_text()
    layers = (REF / "src/mo/tests/test_layers.mojo").read_text()

    def nums(pattern: str, text: str) -> list[float]:
        return [float(x) for x in re.findall(pattern, text)]

    softmax = nums(r"assert_almost_equal\(x\[\d\], ([0-9.]+)", ops)
    return {
        "source": ["src/mo/tests/test_ops.mojo", "src/mo/tests/test_layers.mojo"],
        "rms_norm_ones_w2": {"x": [1.0] * 4, "w": [2.0] * 4, "nelts": 2,
                             "expected": nums(r"assert_almost_equal\(out\[0\], ([0-9.]+), atol=1e-5\)", ops)[0],
                             "cite": "test_ops.mojo:6-25"},
        "geglu_g1_u2": {"gate": [1.0] * 4, "up": [2.0] * 4, "nelts": 2,
                        "expected": nums(r"assert_almost_equal\(out\[0\], ([0-9.]+), atol=1e-4\)", ops)[0],
                        "cite": "test_ops.mojo:27-42"},
        "rope_rotate": {"vec": [1.0, 0.0, 0.0, 1.0], "cos": [0.0, 1.0], "sin": [1.0, 0.0], "nelts": 1,
                        "expected": [0.0, 0.0, 1.0, 1.0], "cite": "test_ops.mojo:44-70"},
        "vec_mat_mul_2x4": {"x": [1.0] * 4, "w": [2.0] * 8, "in_dim": 4, "out_dim": 2, "nelts": 2,
                            "expected": [8.0, 8.0], "cite": "test_ops.mojo:72-86"},
        "softmax_123": {"x": [1.0, 2.0, 3.0], "nelts": 1, "expected": softmax[-3:], "cite": "test_ops.mojo:96-107"},
        "forward_mlp_ones": {"hidden": 4, "intermediate": 2, "expected": 32.0, "atol": 2e-3,
                             "cite": "test_layers.mojo:18-52"},
        "forward_attention_ones": {"hidden": 4, "heads": 2, "kv_heads": 1, "head_dim": 2, "pos": 0,
                                   "cos": [1.0, 0.0], "sin": [0.0, 0.0], "expected": 16.0, "atol": 2e-3,
                                   "cite": "test_layers.mojo:62-134"},
        "forward_attention_qk_norm_ones": {"hidden": 4, "heads": 2, "kv_heads": 1, "head_dim": 2, "pos": 0,
                                           "cos": [1.0, 0.0], "sin": [0.0, 0.0], "expected": 16.0,
                                           "atol": 2e-3, "cite": "test_layers.mojo:136-200"},
        "stale_forward_layer_value_not_used": nums(r"expected: Float32 = ([0-9.]+)", layers)[-1],
    }


def main() -> None:
    ref_model = _import_reference_model()
    (HERE / "sampling.json").write_text(json.dumps(make_sampling(ref_model), indent=1) + "\n")
    (HERE / "known_answers.json").write_text(json.dumps(make_known_answers(), indent=1) + "\n")
    print("wrote", HERE / "sampling.json", HERE / "known_answers.json")


if __name__ == "__main__":
    main()
