"""Kernel phase timeline of one decode pass (the timeline build of the
library: `make -C jalapenos-at-home_b200 timeline`).

    python jalapenos-at-home_b200/timeline.py verify [--rows 5] [--prompt 32]   # Qwen3-8B MXFP4 verify pass
    python jalapenos-at-home_b200/timeline.py draft [--prompt 32]               # Qwen3-0.6B MXFP4 draft step

Builds the benchmark's model (seeded synthetic weights), runs Model.time_pass
(or time_pass_draft) after a prompt of --prompt tokens, and reads the stamps the
kernels wrote during the last replay of the pass.  For every kernel kind it
prints, averaged over the layers, times in microseconds relative to the end
of the previous launch (its last CTA's last stamp): when its CTAs started,
when their grid-dependency wait returned, the median time between its
phase points, and its own end.  Point meanings are listed in
csrc/timeline.cuh.
"""
from __future__ import annotations

import argparse
import os
import pathlib
import sys

HERE = pathlib.Path(__file__).resolve().parent
os.environ.setdefault("JALAPENO_LIB", str(HERE / "lib" / "libjalapeno_timeline.so"))
sys.path.insert(0, str(HERE))

import numpy as np  # noqa: E402

import jalapeno as J  # noqa: E402

QWEN3_8B = dict(layers=36, hidden=4096, q_heads=32, kv_heads=8, inter=12288, vocab=151936, tied=False)
QWEN3_06B = dict(layers=28, hidden=1024, q_heads=16, kv_heads=8, inter=3072, vocab=151936, tied=True)

# intervals between the phase points each kernel stamps: (label, from, to);
# a tuple of points means the first of them that was stamped
PHASES = {
    "k_mx_gemv": [("activations in", 1, 2), ("K slice MMAs", 2, 3), ("split-K partials", 3, 4),
                  ("epilogue", (4, 3), (5, 6)), ("pieces", 5, 6), ("exit", 6, 7)],
    "k_dec_proj": [("inputs in", 1, 2), ("dots + write", 2, 3)],
    "k_attn_decode": [("q, K/V in", 1, 2), ("scores", 2, 3), ("merge + write", 3, 4), ("pieces", 4, 5)],
}


def pick(s, pts):
    """Per CTA, the stamp of the first point of `pts` that CTA wrote (0 if none)."""
    pts = pts if isinstance(pts, tuple) else (pts,)
    out = np.zeros(len(s), dtype=np.int64)
    for q in reversed(pts):
        out = np.where(s[:, q] > 0, s[:, q], out)
    return out


def label_launches(names):
    """Kernel names, with the second and later launches of one kernel inside
    a layer numbered (the o and down projections share k_mx_gemv<add>); a
    layer starts at its q|k|v projection."""
    out, seen = [], {}
    for name in names:
        if name in ("k_mx_gemv<qkv>", "k_dec_proj<qkv>"):
            seen = {}
        seen[name] = seen.get(name, 0) + 1
        out.append(name if seen[name] == 1 else f"{name} #{seen[name]}")
    return out


def summarize(names, st):
    rows = []
    prev_end = None
    for i, name in enumerate(label_launches(names)):
        s = st[i].astype(np.int64)
        live = s[:, 0] > 0
        if not live.any():
            continue
        s = s[live]
        end = s.max()
        base = prev_end if prev_end is not None else s[:, 0].min()
        rec = {"kernel": name, "ctas": int(live.sum()), "start_first": (s[:, 0].min() - base) / 1e3,
               "start_last": (s[:, 0].max() - base) / 1e3, "end": (end - base) / 1e3}
        dep = s[:, 1][s[:, 1] > 0]
        rec["dep_first"] = (dep.min() - base) / 1e3 if len(dep) else float("nan")
        rec["dep_last"] = (dep.max() - base) / 1e3 if len(dep) else float("nan")
        for label, a, b in PHASES.get(name.split("<")[0], []):
            ta, tb = pick(s, a), pick(s, b)
            ok = (ta > 0) & (tb > 0)
            if ok.any():
                rec[label] = float(np.median(tb[ok] - ta[ok])) / 1e3
        rows.append(rec)
        prev_end = end
    return rows


def report(rows, layers):
    kinds = []
    for r in rows:
        if r["kernel"] not in kinds:
            kinds.append(r["kernel"])
    print(f"{'kernel':22s} {'launches':>8s} {'CTAs':>5s} {'start':>15s} {'dependency':>15s} {'end':>7s}  phases (median)")
    total = 0.0
    for k in kinds:
        rs = [r for r in rows if r["kernel"] == k]
        f = lambda key: np.mean([r[key] for r in rs if key in r])
        phases = [(label, np.mean([r[label] for r in rs if label in r]))
                  for label, _, _ in PHASES.get(k.split("<")[0], []) if any(label in r for r in rs)]
        end = f("end")
        total += end * len(rs)
        print(f"{k:22s} {len(rs):8d} {rs[0]['ctas']:5d} {f('start_first'):6.2f}..{f('start_last'):6.2f} "
              f"{f('dep_first'):6.2f}..{f('dep_last'):6.2f} {end:7.2f}  " +
              ", ".join(f"{label} {v:.2f}" for label, v in phases))
    head = sum(r["end"] for r in rows if "head" in r["kernel"])
    print(f"sum of ends {total:.1f} us: output table {head:.1f} us, the {layers} layers "
          f"{(total - head) / layers:.2f} us each")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("pass_kind", choices=["verify", "draft"])
    ap.add_argument("--rows", type=int, default=5, help="verify: rows of the pass (k + 1)")
    ap.add_argument("--prompt", type=int, default=32, help="context (prompt tokens) before the timed pass")
    args = ap.parse_args()
    cfg, seed = (QWEN3_8B, 0) if args.pass_kind == "verify" else (QWEN3_06B, 1)
    m = J.Model.synthesize(**cfg, seed=seed, mxfp4=True, kv_pool_tokens=max(4096, args.prompt + 256))
    prompt = J.prompt_ids(args.prompt, cfg["vocab"], 2)
    if args.pass_kind == "verify":
        _, ms = m.time_pass(prompt, args.rows, reps=5)
        print(f"Qwen3-8B MXFP4 pass of {args.rows} rows after a {args.prompt}-token prompt: {ms:.4f} ms "
              "(CUDA events, median)")
    else:
        _, ms = m.time_pass_draft(prompt, reps=5)
        print(f"Qwen3-0.6B MXFP4 draft step after a {args.prompt}-token prompt: {ms:.4f} ms (CUDA events, median)")
    names, st = J.timeline()
    report(summarize(names, st), cfg["layers"])


if __name__ == "__main__":
    main()
