"""jl_project_noalloc: the projection entry point that allocates nothing.

Its scratch is one fixed device array per device, so it is checked against
jl_project (which uses the model's own scratch) on the same weights and
inputs, twice in a row, for every projection kind: the second call reuses the
array the first left behind.  This file sorts last so that it also runs after
every other GPU test has used the library in the same process.
"""
import numpy as np
import pytest

import jalapeno as J
import oracle as O
from gpu_util import rel_l2

pytestmark = pytest.mark.gpu

REL = 2e-6  # same kernels as jl_project: agreement to f32 noise (in practice exact)


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch


@pytest.fixture(scope="module")
def model():
    cfg = O.PRESETS["tiny-untied"]
    return J.Model.synthesize(cfg.layers, cfg.hidden, cfg.q_heads, cfg.kv_heads, cfg.inter, cfg.vocab,
                              cfg.tied, seed=3, mxfp4=True, mxfp4_embed=True,
                              max_positions=cfg.max_positions, eos=cfg.eos)


def widths(info, which):
    q, kv = info.q_heads * 128, info.kv_heads * 128
    return {J.PROJ_QKV: (info.hidden, q + 2 * kv), J.PROJ_O: (q, info.hidden),
            J.PROJ_GATE_UP: (info.hidden, info.inter), J.PROJ_DOWN: (info.inter, info.hidden),
            J.PROJ_HEAD: (info.hidden, info.vocab)}[which]


@pytest.mark.parametrize("which", [J.PROJ_QKV, J.PROJ_O, J.PROJ_GATE_UP, J.PROJ_DOWN, J.PROJ_HEAD])
@pytest.mark.parametrize("rows", [1, 3, 8])
def test_matches_project(torch_cuda, model, which, rows):
    torch = torch_cuda
    win, wout = widths(model.info, which)
    rng = np.random.default_rng(100 * which + rows)
    layer = model.info.layers - 1
    for call in range(2):
        x = rng.standard_normal((rows, win)).astype(np.float32)
        want = model.project(layer, which, x)
        xd = torch.from_numpy(x).to("cuda:0")
        yd = torch.full((rows, wout), float("nan"), dtype=torch.float32, device="cuda:0")
        torch.cuda.synchronize()
        model.project_noalloc(layer, which, xd.data_ptr(), rows, yd.data_ptr())
        got = yd.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: output not fully written"
        assert rel_l2(got, want) <= REL, f"call {call}: rel_l2 {rel_l2(got, want):.3g}"


def test_two_calls_on_one_stream(torch_cuda, model):
    torch = torch_cuda
    win, wout = widths(model.info, J.PROJ_GATE_UP)
    x = torch.randn(4, win, device="cuda:0")
    y1 = torch.empty(4, wout, device="cuda:0")
    y2 = torch.empty(4, wout, device="cuda:0")
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    model.project_noalloc(0, J.PROJ_GATE_UP, x.data_ptr(), 4, y1.data_ptr(), stream.cuda_stream)
    model.project_noalloc(0, J.PROJ_GATE_UP, x.data_ptr(), 4, y2.data_ptr(), stream.cuda_stream)
    assert torch.equal(y1, y2)
    want = model.project(0, J.PROJ_GATE_UP, x.cpu().numpy())
    assert rel_l2(y1.cpu().numpy(), want) <= REL


def test_rejects_too_many_rows(torch_cuda, model):
    torch = torch_cuda
    x = torch.zeros(9, model.info.hidden, device="cuda:0")
    y = torch.zeros(9, model.info.hidden, device="cuda:0")
    with pytest.raises(J.JlError, match="rows must be 1..8"):
        model.project_noalloc(0, J.PROJ_O, x.data_ptr(), 9, y.data_ptr())


def test_rejects_bf16_projection(torch_cuda):
    torch = torch_cuda
    cfg = O.PRESETS["tiny"]
    m = J.Model.from_config(cfg, 0, mxfp4=False)
    x = torch.zeros(1, cfg.hidden, device="cuda:0")
    y = torch.zeros(1, cfg.hidden, device="cuda:0")
    with pytest.raises(J.JlError, match="not MXFP4"):
        m.project_noalloc(0, J.PROJ_O, x.data_ptr(), 1, y.data_ptr())


FIRST_CALL = r"""
import sys
sys.path[:0] = {paths!r}
import numpy as np
import torch
import jalapeno as J
import oracle as O
cfg = O.PRESETS["tiny-untied"]
m = J.Model.synthesize(cfg.layers, cfg.hidden, cfg.q_heads, cfg.kv_heads, cfg.inter, cfg.vocab,
                       cfg.tied, seed=3, mxfp4=True, mxfp4_embed=True,
                       max_positions=cfg.max_positions, eos=cfg.eos)
x = torch.randn(2, cfg.hidden, device="cuda:0")
y = torch.empty(2, cfg.inter, device="cuda:0")
torch.cuda.synchronize()
before = torch.cuda.mem_get_info(0)[0]
m.project_noalloc(0, J.PROJ_GATE_UP, x.data_ptr(), 2, y.data_ptr())
after = torch.cuda.mem_get_info(0)[0]
print("free bytes", before, after)
assert after == before, f"the first call changed free device memory by {{before - after}} bytes"
"""


def test_first_call_allocates_no_device_memory(torch_cuda):
    """The library sets the fixed array up when a model is created, not on
    the first call: in a fresh process, the device's free memory is the same
    before and after the first call."""
    import subprocess
    import sys
    from pathlib import Path

    repo = Path(__file__).resolve().parents[1]
    paths = [str(repo / "jalapenos-at-home_b200"), str(repo / "oracle")]
    r = subprocess.run([sys.executable, "-c", FIRST_CALL.format(paths=paths)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
