"""The projection kernels, one at a time, against the oracle's matmul
(engine/src/lib.rs:240-266) on the same weights.

MXFP4 projections run on the tensor cores (tcgen05 block-scaled MMA over the
checkpoint's E2M1/E8M0 bytes, activations as eight E2M1 pieces); the bound
below is the f32-accumulation noise floor, far inside the north-star 2e-2.
"""
import numpy as np
import pytest

import jalapeno as J
import oracle as O
from gpu_util import rel_l2

pytestmark = pytest.mark.gpu

REL = 2e-6


def reference(ref: O.Model, layer: int, which: int, x: np.ndarray) -> np.ndarray:
    if which == J.PROJ_QKV:
        return np.concatenate([ref.matmul(p, layer, x) for p in ("q", "k", "v")], axis=1)
    if which == J.PROJ_O:
        return ref.matmul("o", layer, x)
    if which == J.PROJ_GATE_UP:
        g = ref.matmul("gate", layer, x).astype(np.float64)
        u = ref.matmul("up", layer, x).astype(np.float64)
        return (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
    if which == J.PROJ_DOWN:
        return ref.matmul("down", layer, x)
    return ref.matmul("lm_head" if not ref.cfg.tied else "embed", -1, x)


def inputs(rows: int, width: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    # RMS-normalised activations with heavy-ish tails and exact zeros
    x = rng.standard_normal((rows, width)) * np.exp(rng.standard_normal((rows, width)) * 0.5)
    x[:, ::37] = 0.0
    return x.astype(np.float32)


@pytest.fixture(scope="module")
def models():
    out = {}
    for name, seed in (("tiny", 0), ("tiny-draft", 1), ("tiny-untied", 0)):
        cfg = O.PRESETS[name]
        out[name] = (O.Model.synthetic(cfg, seed, mxfp4=True),
                     J.Model.from_config(cfg, seed, mxfp4=True))
    return out


WIDTH_IN = {J.PROJ_QKV: "hidden", J.PROJ_O: "q", J.PROJ_GATE_UP: "hidden", J.PROJ_DOWN: "inter",
            J.PROJ_HEAD: "hidden"}


def width(cfg, which):
    return {"hidden": cfg.hidden, "q": cfg.q_width, "inter": cfg.inter}[WIDTH_IN[which]]


@pytest.mark.parametrize("name", ["tiny", "tiny-draft"])
@pytest.mark.parametrize("which", [J.PROJ_QKV, J.PROJ_O, J.PROJ_GATE_UP, J.PROJ_DOWN])
@pytest.mark.parametrize("rows", [1, 2, 5, 16])
def test_mxfp4_projection_matches_oracle(models, name, which, rows):
    ref, gpu = models[name]
    x = inputs(rows, width(ref.cfg, which), rows * 10 + which)
    got = gpu.project(0, which, x)
    want = reference(ref, 0, which, x)
    assert got.shape == want.shape
    assert rel_l2(got, want) < REL, (name, which, rows)


def test_projection_rows_are_independent(models):
    # a row's result does not depend on how many rows share the launch
    ref, gpu = models["tiny"]
    x = inputs(5, ref.cfg.hidden, 99)
    five = gpu.project(1, J.PROJ_GATE_UP, x)
    for i in range(5):
        np.testing.assert_array_equal(gpu.project(1, J.PROJ_GATE_UP, x[i:i + 1])[0], five[i])


def test_bf16_head_matches_oracle(models):
    ref, gpu = models["tiny-untied"]
    x = inputs(3, ref.cfg.hidden, 5)
    assert rel_l2(gpu.project(0, J.PROJ_HEAD, x), reference(ref, 0, J.PROJ_HEAD, x)) < REL


def test_extreme_scales():
    # E8M0 scale bytes at the ends of the range (the reference's subnormal
    # 2^-127 known answer, engine/src/mxfp4.rs:56-65) through the MMA path
    cfg = O.PRESETS["tiny-draft"]
    ref = O.Model.synthetic(cfg, 1, mxfp4=True)
    x = inputs(2, cfg.hidden, 7) * np.float32(2.0 ** 40)
    gpu = J.Model.from_config(cfg, 1, mxfp4=True)
    got = gpu.project(0, J.PROJ_QKV, x)
    want = reference(ref, 0, J.PROJ_QKV, x)
    assert rel_l2(got, want) < REL
