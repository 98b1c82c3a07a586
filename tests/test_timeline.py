"""The kernel-timeline reader (jalapenos-at-home_b200/timeline.py) on
synthetic stamp tables: launch labels, phase intervals, and the per-layer
total it prints.  No GPU: the timeline build itself runs on the B200."""
import importlib.util

import numpy as np

from conftest import REPO


def load_timeline():
    spec = importlib.util.spec_from_file_location("timeline_tool", REPO / "jalapenos-at-home_b200" / "timeline.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def fake_table(names, ctas=3, step=1000):
    st = np.zeros((len(names), 512, 8), dtype=np.uint64)
    t = 10_000
    for i, name in enumerate(names):
        points = 8 if name.startswith("k_mx_gemv") else 4 if name.startswith("k_dec_proj") else 6
        for c in range(ctas):
            for k in range(points):
                st[i, c, k] = t + 100 * k + 10 * c
        t += step
    return st


def test_labels_number_repeated_kernels_within_a_layer():
    T = load_timeline()
    names = ["k_mx_gemv<qkv>", "k_attn_decode", "k_mx_gemv<add>", "k_mx_gemv<swiglu>", "k_mx_gemv<add>"] * 2
    assert T.label_launches(names)[:5] == ["k_mx_gemv<qkv>", "k_attn_decode", "k_mx_gemv<add>",
                                           "k_mx_gemv<swiglu>", "k_mx_gemv<add> #2"]
    assert T.label_launches(names)[5:] == T.label_launches(names)[:5]


def test_phase_intervals_and_ends():
    T = load_timeline()
    names = ["k_mx_gemv<qkv>", "k_attn_decode", "k_mx_gemv<add>", "k_mx_gemv<swiglu>", "k_mx_gemv<add>",
             "k_mx_gemv<head>"]
    rows = T.summarize(names, fake_table(names))
    assert [r["kernel"] for r in rows] == T.label_launches(names)
    # stamps 100 ns apart per point: every interval between consecutive points is 0.1 us
    q = rows[0]
    assert abs(q["activations in"] - 0.1) < 1e-9 and abs(q["K slice MMAs"] - 0.1) < 1e-9
    assert abs(q["epilogue"] - 0.1) < 1e-9 and abs(q["exit"] - 0.1) < 1e-9
    # launches start 1 us apart and stamp 8 (projections) or 6 (attention)
    # points 0.1 us apart: each end is relative to the previous launch's end
    pts = [8 if n.startswith("k_mx_gemv") else 6 for n in names]
    for i in range(1, len(rows)):
        assert abs(rows[i]["end"] - (1.0 + 0.1 * (pts[i] - pts[i - 1]))) < 1e-9
    # CTAs that never stamped (rows past the grid) are left out
    assert all(r["ctas"] == 3 for r in rows)


def test_draft_labels_and_missing_points():
    T = load_timeline()
    names = ["k_dec_proj<qkv>", "k_attn_decode<raw>", "k_dec_proj<add>", "k_dec_proj<swiglu>", "k_dec_proj<add>"]
    st = fake_table(names)
    st[1, :, 5] = 0  # the draft attention writes no pieces
    rows = T.summarize(names, st)
    assert rows[4]["kernel"] == "k_dec_proj<add> #2"
    assert "pieces" not in rows[1] and abs(rows[1]["scores"] - 0.1) < 1e-9
