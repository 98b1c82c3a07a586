"""Pins the oracle's forward pass to the reference's Python oracle pattern.

The goldens are transformers ``Qwen3ForCausalLM`` in float32 with eager
attention on the same seeded weights (python/check_mxfp4.py:38-62 does the
same for the reference engine).  Tolerances follow the reference tests:
hidden-state relative L2 < 1e-5 (engine/tests/mxfp4.rs:84) and equal greedy
tokens (engine/tests/generation.rs:45-46).
"""
import json

import numpy as np
import pytest

import oracle as O


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def load(golden_dir, name):
    data = np.load(golden_dir / f"forward_{name}.npz")
    meta = json.loads(str(data["meta"]))
    return data, meta


@pytest.mark.parametrize("name", ["tiny", "tiny_untied", "tiny_mxfp4"])
def test_tiny_forward_matches_transformers(golden_dir, name):
    data, meta = load(golden_dir, name)
    model = O.Model.synthetic(meta["preset"], meta["seed"], mxfp4=meta["mxfp4"])
    prompt = [int(t) for t in data["prompt"]]
    assert prompt == O.prompt_ids(len(prompt), model.cfg.vocab, 2)
    hidden = model.hidden(prompt, 1)
    assert rel_l2(hidden, data["hidden_1"]) < 1e-5
    ids, logits = model.predict(prompt, model.cache(), all=True, logits=True)
    assert rel_l2(logits, data["logits"]) < 1e-5
    assert np.abs(logits - data["logits"]).max() < 1e-4
    tokens = model.generate(prompt, len(data["tokens"]) - len(prompt))
    assert tokens == [int(t) for t in data["tokens"]]


@pytest.mark.slow
@pytest.mark.parametrize("name", ["qwen3_0_6b", "qwen3_0_6b_mxfp4"])
def test_qwen3_0_6b_forward_matches_transformers(golden_dir, name):
    data, meta = load(golden_dir, name)
    model = O.Model.synthetic(meta["preset"], meta["seed"], mxfp4=meta["mxfp4"])
    prompt = [int(t) for t in data["prompt"]]
    hidden = model.hidden(prompt, 1)
    assert rel_l2(hidden, data["hidden_1"]) < 1e-5
    ids, logits = model.predict(prompt, model.cache(), all=True, logits=True)
    top = data["top_ids"]
    ours = np.take_along_axis(logits, top, axis=1)
    assert np.abs(ours - data["top_logits"]).max() < 1e-3
    assert ids == [int(t) for t in top[:, 0]]
    tokens = model.generate(prompt, len(data["tokens"]) - len(prompt))
    assert tokens == [int(t) for t in data["tokens"]]


def test_synthetic_stream_is_pinned(golden_dir):
    data = np.load(golden_dir / "synth.npz")
    for seed in (0, 1):
        for idx in (0, 1, 5, 12):
            np.testing.assert_array_equal(O.synth_bf16(seed, idx, 64), data[f"s{seed}_t{idx}_head"])
            np.testing.assert_array_equal(O.synth_bf16(seed, idx, 37, first=1_000_003),
                                          data[f"s{seed}_t{idx}_mid"])
    blob = O.synth_bf16(0, 3, 1 << 20)
    assert O.bf16_to_f32(blob).astype(np.float64).sum() == float(data["s0_t3_sum_f64"])
    assert O.prompt_ids(32, 151936, 2) == [int(t) for t in data["prompt_32_seed2"]]


def test_synthetic_weights_look_like_n_0_002():
    w = O.bf16_to_f32(O.synth_bf16(0, 7, 1 << 18))
    assert abs(w.mean()) < 2e-4
    assert abs(w.std() - 0.02) < 2e-4


def test_rope_and_norm_building_blocks():
    # rope at position 0 is the identity; norms of a constant row equal the gain
    x = np.random.default_rng(0).standard_normal((1, 256)).astype(np.float32)
    y = x.copy()
    O.lib().jlo_rope(O.ptr(y, O.ctypes.c_float), 1, 2, 0)
    np.testing.assert_array_equal(x, y)
    ones = np.full(4, 0x3F80, np.uint16)
    row = np.full((1, 4), 3.0, np.float32)
    out = np.empty_like(row)
    O.lib().jlo_rms_norm(O.ptr(row, O.ctypes.c_float), 1, 4, O.ptr(ones, O.ctypes.c_uint16),
                         O.ptr(out, O.ctypes.c_float))
    np.testing.assert_allclose(out, 1.0, rtol=1e-6)


def test_argmax_first_maximum_wins():
    v = np.array([1.0, 3.0, 3.0, -np.inf, np.nan], np.float32)
    assert O.lib().jlo_argmax(O.ptr(v, O.ctypes.c_float), 5) == 1
