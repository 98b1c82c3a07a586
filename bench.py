#!/usr/bin/env python
"""Qwen3-8B MXFP4 speculative-decode benchmark (BASELINE.json metric).

Workload (k = 4, batch 1, short context): target
Qwen3-8B with MXFP4 projections (seed 0), draft Qwen3-0.6B MXFP4 (seed 1),
32-token prompt (uniform ids, seed 2 + rank), 64 new tokens per step, greedy
speculative decoding with draft length 4.  Weights are seeded synthetic
tensors generated on the GPU, so a random draft would never agree with the
target; the headline therefore uses the oracle-draft mode of the config
(the draft still runs every pass, its proposals replaced by the target's
greedy tokens, each swapped with probability p = 0.25 for a uniform id),
which gives an acceptance rate near the reference's published runs.  The
same line carries the real-draft and p = 0 / 0.5 numbers.

A step is one call of jl_generate_speculative: prefill (not counted in
`value`, as in the reference's t(65) - t(1) method) plus the 64-token decode
loop, which runs on the GPU as one CUDA graph.  `value` is device time of the
decode loops (CUDA events on the stream it runs on); `e2e` is wall time of
the whole public call with host buffers (prompt in, tokens out), prefill
included.  Multi-GPU runs are independent replicas (one process per GPU, no
collective on the data path); the barrier and max-over-ranks timing use
torch.distributed only for control.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path[:0] = [str(REPO / "jalapenos-at-home_b200"), str(REPO / "oracle")]

PRESETS = {
    "qwen3-0.6b": dict(layers=28, hidden=1024, q_heads=16, kv_heads=8, inter=3072, vocab=151936, tied=True),
    "qwen3-1.7b": dict(layers=28, hidden=2048, q_heads=16, kv_heads=8, inter=6144, vocab=151936, tied=True),
    "qwen3-8b": dict(layers=36, hidden=4096, q_heads=32, kv_heads=8, inter=12288, vocab=151936, tied=False),
}
METRIC = "Qwen3-8B MXFP4 spec-decode tok/s (k=4) at 1-8 B200; % of HBM roofline"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--gamma", type=int, default=4)
    ap.add_argument("--new", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=32)
    ap.add_argument("--p", type=float, default=0.25, help="oracle-draft replacement probability")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-pytorch", action="store_true",
                    help="--impl reference: skip the transformers float32 baseline")
    ap.add_argument("--profile", action="store_true",
                    help="small run for ncu: one k+1-row target pass and one draft pass "
                         "(Model::time_pass), no timing loop")
    ap.add_argument("--config5", action="store_true",
                    help="BASELINE.json configs[4]: per-GPU batches of independent sequences with 4096-token "
                         "contexts and 256 new tokens (one JSON line per batch size)")
    ap.add_argument("--batches", default="1,8,32", help="--config5 batch sizes")
    ap.add_argument("--prefill", default="",
                    help="comma-separated prompt lengths: time Model::predict of one prompt of each length on "
                         "the Qwen3-8B MXFP4 target (one JSON line per length), nothing else")
    ap.add_argument("--prompt-attention", choices=["tensor", "cuda"], default="tensor",
                    help="with --prefill: prompt attention on tcgen05 MMAs (default) or on the CUDA-core kernel")
    ap.add_argument("--small", action="store_true",
                    help="with --profile or --prefill: two layers of each model at full width and an 8192-entry "
                         "vocabulary (under 0.5 GB on the device), for multi-pass ncu captures")
    return ap.parse_args()


def run_profile(args, dist):
    """The kernels of one speculative round, for a profiler's launch list: a
    k+1-row verify pass of the target and a one-row draft pass, each through
    the captured pass graph the decode loop replays."""
    import jalapeno as J

    if args.small:
        opts = dict(kv_pool_tokens=1024, max_pass_rows=64, device=dist.local)
        small = dict(layers=2, vocab=8192)
        target = J.Model.synthesize(**{**PRESETS["qwen3-8b"], **small}, seed=0, mxfp4=True,
                                    name="Qwen3-8B-MXFP4 (2 layers)", **opts)
        draft = J.Model.synthesize(**{**PRESETS["qwen3-0.6b"], **small}, seed=1, mxfp4=True,
                                   name="Qwen3-0.6B-MXFP4 (2 layers)", **opts)
        vocab = 8192
    else:
        target, draft = make_models(J, dist.local)
        vocab = 151936
    prompt = J.prompt_ids(args.prompt, vocab, 2)
    tw, tg = target.time_pass(prompt, args.gamma + 1, reps=1)
    dw, dg = draft.time_pass_draft(prompt, reps=1)
    print(json.dumps({"profile": True, "target_pass_ms": tg, "draft_pass_ms": dg,
                      "target_rows": args.gamma + 1}), flush=True)


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Dist:
    """Rank bookkeeping; torch.distributed only when launched by torchrun.
    The process group is NCCL over the GPUs, or gloo on host cores when
    JL_DIST_BACKEND=gloo (the multi-process tests, which have no GPU)."""

    def __init__(self, backend: str | None = None, timeout_s: int = 300):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend or os.environ.get("JL_DIST_BACKEND", "nccl")
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            timeout = datetime.timedelta(seconds=timeout_s)
            if self.backend == "nccl":
                torch.cuda.set_device(self.local)
                dist.init_process_group("nccl", timeout=timeout, device_id=torch.device("cuda", self.local))
            else:
                dist.init_process_group(self.backend, timeout=timeout)
            self.pg = dist

    def _sync(self):
        if self.backend == "nccl":
            import torch

            torch.cuda.synchronize(self.local)

    def barrier(self):
        self._sync()
        if self.pg:
            self.pg.barrier()
        self._sync()

    def max(self, v: float) -> float:
        return self._reduce(v, "max")

    def sum(self, v: float) -> float:
        return self._reduce(v, "sum")

    def _reduce(self, v, op):
        if not self.pg:
            return v
        import torch

        dev = f"cuda:{self.local}" if self.backend == "nccl" else "cpu"
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX if op == "max" else self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class Clocks:
    """Samples SM clocks and throttle reasons of one GPU while running."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_models(J, device: int):
    t = PRESETS["qwen3-8b"]
    d = PRESETS["qwen3-0.6b"]
    opts = dict(kv_pool_tokens=4096, max_pass_rows=256, device=device)
    target = J.Model.synthesize(**t, seed=0, mxfp4=True, name="Qwen3-8B-MXFP4", **opts)
    draft = J.Model.synthesize(**d, seed=1, mxfp4=True, name="Qwen3-0.6B-MXFP4", **opts)
    return target, draft


def oracle_from_device(O, gpu_model, preset, mxfp4):
    """An oracle model holding the GPU model's own weights (read back from the
    device; a few seconds instead of synthesizing on the host)."""
    import numpy as np

    cfg = O.Config(preset, **PRESETS[preset], max_positions=40960, eos=151645)
    tensors = {}

    def mat(name, rows, cols, q):
        if q:
            raw = gpu_model.read_tensor(name, rows * cols // 2 + rows * cols // 32)
            return O.Matrix(rows, cols, packed=raw[: rows * cols // 2].copy(),
                            scales=raw[rows * cols // 2:].copy())
        raw = gpu_model.read_tensor(name, rows * cols * 2)
        return O.Matrix(rows, cols, bf16=raw.view(np.uint16).copy())

    tensors["embed"] = mat("model.embed_tokens.weight", cfg.vocab, cfg.hidden, False)
    tensors["lm_head"] = None if cfg.tied else mat("lm_head.weight", cfg.vocab, cfg.hidden, False)
    tensors["norm"] = np.full(cfg.hidden, O.ONE_BF16, np.uint16)
    for layer in range(cfg.layers):
        for p in O.PROJECTIONS:
            shape = O.shape_of(cfg, p)
            tensors[f"{layer}.{p}"] = mat(f"model.layers.{layer}.{O.HF_NAMES[p]}", shape[0], shape[1],
                                          mxfp4)
        for n in O.NORM_CODE:
            tensors[f"{layer}.{n}"] = np.full(O.shape_of(cfg, n)[0], O.ONE_BF16, np.uint16)
    return O.Model(cfg, tensors)


class OracleSample:
    """The oracle's restatement of the reference's CPU path
    (engine/src/lib.rs, model.rs, speculative.rs) on the host cores, for the
    benchmark workload: both models prefilled once (untimed), then each
    sample decodes `rounds` speculative rounds from that state (the caches
    rolled back to the prompt), timed on the host clock.  The bf16-rounding
    KV cache matches the GPU's bf16 cache."""

    def __init__(self, O, t_ref, d_ref, prompt, stream, args, rounds=3):
        self.O, self.t_ref, self.d_ref, self.prompt, self.stream = O, t_ref, d_ref, prompt, stream
        self.args, self.rounds = args, rounds
        self.tc, self.dc = t_ref.cache(True), d_ref.cache(True)
        self.t_first = t_ref.predict(prompt, self.tc)[0]
        self.d_first = d_ref.predict(prompt, self.dc)[0]

    def run(self):
        self.tc.truncate(len(self.prompt))
        self.dc.truncate(len(self.prompt))
        res = self.O.generate_scheduled(
            self.t_ref, self.d_ref, self.prompt, self.args.new, self.O.DraftSchedule.fixed(self.args.gamma),
            round_bf16=True, oracle_stream=self.stream, oracle_p=self.args.p, oracle_seed=5,
            max_rounds=self.rounds, prefilled=(self.tc, self.dc, self.t_first, self.d_first))
        new = len(res.tokens) - len(self.prompt)
        return res, new / res.decode_s

    def describe(self, res, threads):
        new = len(res.tokens) - len(self.prompt)
        return (f"oracle spec decode of the same workload (8B MXFP4 + 0.6B MXFP4, k={self.args.gamma}, "
                f"p={self.args.p}, bf16-rounded KV) on {threads} threads: {res.rounds} rounds, {new} "
                f"tokens in {res.decode_s:.2f} s after an untimed prefill")


def cpu_baseline(O, target, draft, prompt, greedy, args):
    """cpu_baseline of the main line: the oracle port on this host's cores,
    on the GPU models' own weights, timed on three speculative rounds after
    an untimed prefill.  Its tokens are compared with the GPU stream."""
    O.set_threads(physical_cores())
    t_ref = oracle_from_device(O, target, "qwen3-8b", True)
    d_ref = oracle_from_device(O, draft, "qwen3-0.6b", True)
    sample = OracleSample(O, t_ref, d_ref, prompt, greedy, args)
    res, value = sample.run()
    match = res.tokens == greedy[: len(res.tokens)]
    return {"value": value, "unit": "tok/s", "cores": O.threads(), "kind": "port",
            "sample": sample.describe(res, O.threads()), "tokens_equal_gpu_stream": match}


def physical_cores() -> int:
    try:
        import psutil

        n = psutil.cpu_count(logical=False)
        if n:
            return int(n)
    except ImportError:
        pass
    return os.cpu_count() or 1


def pytorch_baseline(O, t_ref, d_ref, prompt, stream, args, threads):
    """The reference's Python path (transformers Qwen3ForCausalLM, float32,
    eager attention; python/speculative_decoding.py with both KV caches kept,
    python/check_mxfp4.py's dequantized MXFP4 weights) on the same workload
    and host cores: one generation after an untimed prefill, warm-up rounds,
    then timed rounds."""
    import torch
    import transformers

    import torch_baseline as TB

    torch.set_num_threads(threads)
    t0 = time.perf_counter()
    ht, hd = TB.hf_model(t_ref.cfg, t_ref), TB.hf_model(d_ref.cfg, d_ref)
    build_s = time.perf_counter() - t0
    warm = min(args.warmup, 3)
    toks, acc, drafted, rounds, marks = TB.speculative(
        ht, hd, prompt, args.new, args.gamma, t_ref.eos, t_ref.cfg.vocab, stream, args.p, 5,
        max_rounds=warm + args.steps)
    marks = [(0.0, len(prompt))] + marks
    warm = min(warm, max(0, len(marks) - 4))
    (ta, na), (tb, nb) = marks[warm], marks[-1]
    value = (nb - na) / (tb - ta)
    del ht, hd
    return {"value": value, "unit": "tok/s", "cores": threads, "kind": "pytorch",
            "sample": (f"transformers {transformers.__version__} Qwen3ForCausalLM float32 eager on torch "
                       f"{torch.__version__}, {threads} threads, 8B + 0.6B with MXFP4 projections dequantized, "
                       f"k={args.gamma}, oracle draft p={args.p}, KV caches kept between rounds: {warm} warm-up "
                       f"rounds, then {len(marks) - 1 - warm} timed rounds, {nb - na} tokens in {tb - ta:.2f} s "
                       f"(models built in {build_s:.0f} s); tokens equal to the oracle's (f32 cache): "
                       f"{toks == stream[: len(toks)]}")}


def run_reference(args, dist):
    """--impl reference: the reference's CPU implementation of this path on
    the host cores.  Its Rust engine does not build here (no cargo; its GPU
    path is Metal), so the oracle's restatement of it runs: weights
    synthesized on the host (the same seeded tensors the GPU synthesizes),
    the oracle-draft stream from the oracle's own greedy decode, every
    physical core.  Nothing of this repository's GPU engine is loaded.
    One speculative generation of the workload (64 new tokens) after an
    untimed prefill: its first min(W, 3) rounds are the warm-up, the next up
    to K rounds (at least 3) are timed.  Rank 0 measures; other ranks wait at
    a host barrier."""
    import oracle as O

    if dist.rank == 0:
        threads = physical_cores()
        O.set_threads(threads)
        t_ref = O.Model.synthetic("qwen3-8b", 0, mxfp4=True)
        d_ref = O.Model.synthetic("qwen3-0.6b", 1, mxfp4=True)
        prompt = O.prompt_ids(args.prompt, 151936, 2)
        stream = t_ref.generate(prompt, args.new, round_bf16=True)
        warm = min(args.warmup, 3)
        tc, dc = t_ref.cache(True), d_ref.cache(True)
        first = (t_ref.predict(prompt, tc)[0], d_ref.predict(prompt, dc)[0])
        res = O.generate_scheduled(t_ref, d_ref, prompt, args.new, O.DraftSchedule.fixed(args.gamma),
                                   round_bf16=True, oracle_stream=stream, oracle_p=args.p, oracle_seed=5,
                                   max_rounds=warm + args.steps, prefilled=(tc, dc, *first))
        marks = [(0.0, len(prompt))] + res.round_marks
        warm = min(warm, max(0, len(marks) - 4))  # at least 3 timed rounds
        (ta, na), (tb, nb) = marks[warm], marks[-1]
        timed_rounds = len(marks) - 1 - warm
        value = (nb - na) / (tb - ta)
        sample = (f"oracle spec decode of the workload (8B MXFP4 + 0.6B MXFP4, k={args.gamma}, p={args.p}, "
                  f"bf16-rounded KV) on {O.threads()} threads, one generation after an untimed prefill: "
                  f"{warm} warm-up rounds, then {timed_rounds} timed rounds, {nb - na} tokens in {tb - ta:.2f} s; "
                  f"oracle tokens equal to the oracle's own greedy stream: {res.tokens == stream[: len(res.tokens)]}")
        line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s",
                "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 activations, MXFP4 weights", "data": "synthetic (seeded, synthesized on the host)",
                "config": workload_config(args),
                "cpu_baseline": {"value": value, "unit": "tok/s", "cores": O.threads(), "kind": "port",
                                 "sample": sample},
                "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        if not args.no_pytorch:
            # transformers keeps K/V in f32: its oracle-draft stream is the
            # oracle's greedy stream with an f32 cache
            stream32 = t_ref.generate(prompt, args.new)
            line["pytorch_baseline"] = pytorch_baseline(O, t_ref, d_ref, prompt, stream32, args, threads)
        print(json.dumps(line), flush=True)
    dist.barrier()


def aggregate(dist, new_tokens: int, decode_ms: float, e2e_s: float):
    """Whole-job throughput of the replicas: every rank's generated tokens over
    the slowest rank's time (device decode time, and wall time of the public
    call for e2e).  Returns (value tok/s, e2e tok/s, total tokens, the slowest
    rank's decode ms)."""
    max_decode_ms = dist.max(decode_ms)
    max_e2e_s = dist.max(e2e_s)
    all_tokens = dist.sum(new_tokens)
    return all_tokens / (max_decode_ms / 1000.0), all_tokens / max_e2e_s, all_tokens, max_decode_ms


def run_config5(args, dist):
    """each GPU decodes a batch of B independent
    sequences (random 4096-token contexts, seeds 3 + index, 256 new tokens,
    k = 4, oracle draft p) in lockstep rounds through
    jl_generate_speculative_batch; replicas on N GPUs.  `value` = all ranks'
    new tokens over the slowest rank's decode time; HBM GB/s per GPU from the
    algorithmic bytes (weights per lockstep pass, each sequence's KV per pass
    it takes part in); the roofline is that of the path's formula: bytes per
    round W_t + k W_d + B KV_t(ctx) + B k KV_d(ctx) at the measured copy
    bandwidth."""
    for line in config5_lines(args, dist, [int(x) for x in args.batches.split(",")]):
        if dist.rank == 0:
            print(json.dumps(line), flush=True)


def config5_lines(args, dist, batches):
    """The configs[4] measurements for each per-GPU batch size (one dict each)."""
    import jalapeno as J

    peak, peak_kind = measured_peaks()
    ctx, new, k = 4096, 256, args.gamma
    lines = []
    t, d = PRESETS["qwen3-8b"], PRESETS["qwen3-0.6b"]
    opts = dict(kv_pool_tokens=max(batches) * (ctx + new + 128) + 1024, max_pass_rows=256, device=dist.local)
    target = J.Model.synthesize(**t, seed=0, mxfp4=True, name="Qwen3-8B-MXFP4", **opts)
    draft = J.Model.synthesize(**d, seed=1, mxfp4=True, name="Qwen3-0.6B-MXFP4", **opts)
    ti, di = target.info, draft.info
    w_t, w_d = ti.pass_bytes, di.pass_bytes
    kv_t, kv_d = ti.kv_bytes_per_token, di.kv_bytes_per_token
    for B in batches:
        prompts = [J.prompt_ids(ctx, ti.vocab, 3 + i + 1000 * dist.rank) for i in range(B)]
        g = J.generate_batch(target, prompts, new + 2 * k)
        streams = [s.tokens for s in g.results]
        t0 = time.perf_counter()
        r = J.generate_speculative_batch(target, draft, prompts, new, J.DraftSchedule.fixed(k),
                                         oracle_streams=streams, oracle_p=args.p,
                                         oracle_seeds=[5 + i for i in range(B)])
        wall = time.perf_counter() - t0
        assert all(s.tokens == st[: ctx + new] for s, st in zip(r.results, streams)), \
            "speculative output differs from greedy"
        tokens = sum(len(s.tokens) - ctx for s in r.results)
        value, e2e, all_tokens, max_ms = aggregate(dist, tokens, r.decode_ms, wall)
        greedy_value, _, _, _ = aggregate(dist, B * (new + 2 * k - 1), g.decode_ms, 1.0)
        # algorithmic bytes: weights once per lockstep pass, KV once per sequence per pass
        draft_sets = max(s.draft.passes for s in r.results)
        kv = sum(s.verify.passes * kv_t + s.draft.passes * kv_d for s in r.results) * (ctx + new / 2)
        moved = r.rounds * w_t + draft_sets * w_d + kv
        round_bytes = w_t + k * w_d + B * (ctx + new / 2) * (kv_t + k * kv_d)
        roof = peak * 1e9 * (tokens / max(r.rounds, 1)) / round_bytes
        line = {"metric": "configs[4] aggregate spec-decode tok/s (k=4, per-GPU batch, 4096-token contexts)",
                "value": value, "unit": "tok/s", "n_gpus": dist.world, "batch_per_gpu": B,
                "higher_is_better": True, "scaling": "weak", "dtype": "mxfp4 weights, f32 activations",
                "data": "synthetic: seeded N(0, 0.02) weights, uniform random contexts",
                "ms_decode": max_ms, "tokens": all_tokens, "rounds": r.rounds,
                "acceptance": sum(s.accepted for s in r.results) / max(1, sum(s.drafted for s in r.results)),
                "hbm_gbs_per_gpu": moved / (r.decode_ms / 1000.0) / 1e9,
                "roofline": {"tok_s": roof * dist.world, "frac": value / (roof * dist.world), "peak_gbs": peak,
                             "peak": peak_kind},
                "greedy_batch_tok_s": greedy_value, "prefill_s": r.prefill_ms / 1000.0,
                "e2e": {"value": e2e, "unit": "tok/s (wall, prefill included)"},
                "config": {"workload": "Qwen3-8B MXFP4 + Qwen3-0.6B MXFP4, batched speculative decode",
                           "batch_per_gpu": B, "context_tokens": ctx, "new_tokens": new, "k": k,
                           "draft_mode": f"oracle p={args.p}", "parallelism": f"replicas x{dist.world}"}}
        lines.append(line)
    del target, draft
    return lines


def other_configs(J, draft, args, peak, device):
    """BASELINE.json configs[0..2] and a compact configs[4], each with its
    path roofline at the measured copy bandwidth.  Decode time is device time
    of the generation loop (CUDA events), prefill excluded.
      Qwen3-1.7B bf16 greedy, 32-token prompt, 64 tokens.
      the same with MXFP4 projections.
      Qwen3-1.7B MXFP4 target + Qwen3-0.6B MXFP4 draft, k = 4,
                  oracle draft p in {0, 0.25, 0.5}, and the real draft.
      8B + 0.6B, k = 4, batch 8 of 4096-token contexts, 256 new
                  tokens per sequence (bench.py --config5 runs batches 1/8/32)."""
    out = {}
    c17 = dict(PRESETS["qwen3-1.7b"])
    prompt = J.prompt_ids(args.prompt, c17["vocab"], 2)
    for mx in (False, True):
        m = J.Model.synthesize(**c17, seed=0, mxfp4=mx, kv_pool_tokens=1024, max_pass_rows=256, device=device)
        J.generate_batch(m, [prompt], args.new)  # warm: graphs
        r = J.generate_batch(m, [prompt], args.new)
        new = len(r.results[0].tokens) - len(prompt)
        tps = new / (r.decode_ms / 1000.0)
        roof = peak * 1e9 / m.info.pass_bytes
        out[f"1.7B {'MXFP4' if mx else 'bf16'} greedy"] = {
            "tok_s": tps, "roofline_tok_s": roof, "frac": tps / roof, "pass_bytes": m.info.pass_bytes}
        if mx:
            greedy = m.generate(prompt, args.new)
            w_t, w_d = m.info.pass_bytes, draft.info.pass_bytes
            for p, stream in ((0.0, True), (0.25, True), (0.5, True), (0.0, False)):
                kw = dict(oracle_stream=greedy, oracle_p=p, oracle_seed=5) if stream else {}
                J.generate_speculative(m, draft, prompt, args.new, args.gamma, **kw)  # warm
                rs = J.generate_speculative(m, draft, prompt, args.new, args.gamma, **kw)
                assert rs.tokens == greedy, "speculative output differs from greedy"
                n = len(rs.tokens) - len(prompt)
                tps = n / (rs.decode_ms / 1000.0)
                roof = peak * 1e9 * (n / max(rs.rounds, 1)) / (w_t + args.gamma * w_d)
                out[f"1.7B MXFP4 + 0.6B, k={args.gamma}, " + (f"oracle p={p}" if stream else "real draft")] = {
                    "tok_s": tps, "accepted": rs.accepted, "drafted": rs.drafted, "roofline_tok_s": roof,
                    "frac": tps / roof}
        del m
    return out


def workload_config(args):
    return {"workload": "Qwen3-8B MXFP4 target + Qwen3-0.6B MXFP4 draft, greedy speculative decode",
            "k": args.gamma, "batch_per_gpu": 1, "prompt_tokens": args.prompt,
            "new_tokens": args.new, "draft_mode": f"oracle p={args.p}",
            "embed_lm_head": "bf16", "kv_cache": "bf16 paged", "seeds": "target 0, draft 1, prompt 2+rank",
            "l2": "weights 4.9 GB per target pass, larger than the 126 MB L2",
            "parallelism": f"replicas x{args.gpus}, no collective"}


def run_prefill(args, dist):
    """Prompt processing of the target (model.rs:209-240 with all = false):
    each length's prompt as the multi-chunk tensor-core passes predict runs,
    with the prompt attention of a bf16 pool on tensor cores.  One untimed
    call, then the fastest of three timed calls (wall clock around the
    synchronous public call: ids in, one id out).  Rank 0 prints."""
    import jalapeno as J

    lengths = [int(x) for x in args.prefill.split(",") if x]
    t = dict(PRESETS["qwen3-8b"])
    if args.small:  # for ncu captures: two layers at full width, an 8192-entry vocabulary
        t.update(layers=2, vocab=8192)
    target = J.Model.synthesize(**t, seed=0, mxfp4=True, name="Qwen3-8B-MXFP4",
                                kv_pool_tokens=max(lengths) + 64, device=dist.local)
    tc = target.prompt_attention(args.prompt_attention == "tensor")
    for n in lengths:
        prompt = J.prompt_ids(n, t["vocab"], 3)
        target.predict(prompt, target.cache())
        best = float("inf")
        for _ in range(3):
            cache = target.cache()
            t0 = time.perf_counter()
            target.predict(prompt, cache)
            best = min(best, time.perf_counter() - t0)
            del cache
        if dist.rank == 0:
            print(json.dumps({"metric": "Qwen3-8B MXFP4 prefill" + (" (2 layers, --small)" if args.small else ""),
                              "prompt_tokens": n, "ms": round(best * 1e3, 2),
                              "tok_s": round(n / best, 1), "kv": "bf16 paged", "data": "synthetic",
                              "prompt_attention": "tcgen05" if tc else "cuda cores"}), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        # host-only: a gloo barrier (other ranks wait while rank 0 measures)
        dist = Dist(backend="gloo", timeout_s=3600)
        run_reference(args, dist)
        dist.close()
        return
    dist = Dist()
    if args.profile:
        run_profile(args, dist)
        dist.close()
        return
    if args.config5:
        run_config5(args, dist)
        dist.close()
        return
    if args.prefill:
        run_prefill(args, dist)
        dist.close()
        return
    import jalapeno as J

    peak, peak_kind = measured_peaks()
    target, draft = make_models(J, dist.local)
    ti, di = target.info, draft.info
    prompt = J.prompt_ids(args.prompt, ti.vocab, 2 + dist.rank)
    greedy = target.generate(prompt, args.new)

    def step(p, stream=True):
        t0 = time.perf_counter()
        r = J.generate_speculative(target, draft, prompt, args.new, args.gamma,
                                   oracle_stream=greedy if stream else None, oracle_p=p,
                                   oracle_seed=5)
        wall = time.perf_counter() - t0
        assert r.tokens == greedy, "speculative output differs from greedy"
        return r, wall

    for _ in range(args.warmup):
        step(args.p)
    dist.barrier()
    results = []
    with Clocks(dist.local) as clocks:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            results.append(step(args.p))
        dist.barrier()
        wall_total = time.perf_counter() - t0
    new_tokens = sum(len(r.tokens) - len(prompt) for r, _ in results)
    decode_ms = sum(r.decode_ms for r, _ in results)
    e2e_s = sum(w for _, w in results)
    value, e2e, all_tokens, max_decode_ms = aggregate(dist, new_tokens, decode_ms, e2e_s)
    r0 = results[0][0]
    rounds = sum(r.rounds for r, _ in results)
    verify = sum(r.verify.passes for r, _ in results)
    drafts = sum(r.draft.passes for r, _ in results)

    # algorithmic bytes of the decode loops: every verify pass reads the
    # target's weights, every draft pass the draft's; KV reads are added per
    # pass from the context length (bf16 cache).
    ctx = len(prompt) + args.new / 2
    kv_t = ti.kv_bytes_per_token * ctx
    kv_d = di.kv_bytes_per_token * ctx
    bytes_total = verify * (ti.pass_bytes + kv_t) + drafts * (di.pass_bytes + kv_d)
    path_gbs = bytes_total / (decode_ms / 1000.0) / 1e9
    tokens_per_round = new_tokens / rounds
    bytes_per_round = ti.pass_bytes + args.gamma * di.pass_bytes
    roof_tps = peak * 1e9 * tokens_per_round / bytes_per_round

    # dominant kernel family: the target's MXFP4 projections (k_mx_gemv); the
    # largest, gate/up, timed as the fused kernel of a k+1-row verify pass
    # (launched back to back on the model's stream, CUDA events, inputs left
    # by the timed decode steps).  Algorithmic bytes per launch: the gate and
    # up weights (codes + scales).
    kern = {"gate_up": J.PROJ_GATE_UP, "down": J.PROJ_DOWN, "o": J.PROJ_O, "qkv": J.PROJ_QKV,
            "head": J.PROJ_HEAD}
    kt = {}
    for name, which in kern.items():
        ms, nb = target.time_projection(0, which, args.gamma + 1, iters=20)
        kt[name] = (ms, nb)
    ms, nb = kt["gate_up"]
    achieved = nb / (ms / 1000.0) / 1e9
    traffic = None
    tfile = REPO / "profiles" / "traffic.json"
    if tfile.exists():
        traffic = json.loads(tfile.read_text()).get("gate_up_verify_8b")

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": max_decode_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32 activations, MXFP4 weights",
        "data": "synthetic (seeded N(0,0.02) weights generated on the GPU, uniform prompt ids)",
        "config": workload_config(args),
        "acceptance": {"accepted": sum(r.accepted for r, _ in results),
                       "drafted": sum(r.drafted for r, _ in results), "rounds": rounds,
                       "tokens_per_round": tokens_per_round},
        "path_roofline": {"bytes_per_round_k": bytes_per_round, "roofline_tok_s": roof_tps,
                          "frac": value / dist.world / roof_tps, "achieved_gbs": path_gbs,
                          "peak_gbs": peak, "peak_kind": peak_kind},
        "roofline": {"bound": "hbm", "kernel": "k_mx_gemv<SWIGLU>: fused MXFP4 gate/up projection, k+1-row verify",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "bytes_per_launch": nb, "ms_per_launch": ms,
                     "peak_kind": peak_kind},
        "kernels_gbs": {k: v[1] / (v[0] / 1000.0) / 1e9 for k, v in kt.items()},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4 * (len(prompt) + len(greedy)),
                "d2h_bytes_per_step": 4 * len(greedy) + 16 * (rounds // args.steps)},
        "gpu_launches": None,
        "clocks": clocks.summary(),
        "wall_s": wall_total,
    }
    # kernels launched in the timed steps: per step the prefills (target and
    # draft, 16-row chunks), every verify pass (k+1 rows), every draft step
    # (one row; catch-ups take the same kernels) plus its bookkeeping kernel,
    # and three loop kernels per round (round begin, verify setup, accept)
    kt16, kd16 = target.pass_kernels(16), draft.pass_kernels(16)
    kt_v, kd_1 = target.pass_kernels(args.gamma + 1), draft.pass_kernels(1, draft_step=True)
    launches = 0
    for r, _ in results:
        launches += (r.prefill.passes // 2) * (kt16 + kd16) + r.verify.passes * kt_v
        launches += r.draft.passes * (kd_1 + 1) + 3 * r.rounds
    line["gpu_launches"] = launches
    if not args.no_sweep:
        sweep = {}
        for p, stream in ((0.0, True), (0.5, True), (0.0, False)):
            r, w = step(p, stream)
            n = len(r.tokens) - len(prompt)
            sweep["real draft" if not stream else f"oracle p={p}"] = {
                "tok_s": n / (r.decode_ms / 1000.0), "accepted": r.accepted, "drafted": r.drafted}
        # the configuration's other draft lengths (same prompt and oracle stream)
        for k in (2, 8):
            r = J.generate_speculative(target, draft, prompt, args.new, k, oracle_stream=greedy,
                                       oracle_p=args.p, oracle_seed=5)
            assert r.tokens == greedy, "speculative output differs from greedy"
            sweep[f"k={k} oracle p={args.p}"] = {
                "tok_s": (len(r.tokens) - len(prompt)) / (r.decode_ms / 1000.0), "accepted": r.accepted,
                "drafted": r.drafted}
        # greedy decode of the target alone, same device loop
        t0 = time.perf_counter()
        target.generate(prompt, args.new)
        sweep["greedy (no draft) e2e tok/s"] = args.new / (time.perf_counter() - t0)
        # the configuration's long-context setting: a prefilled 2048-token context
        if args.prompt < 2048:
            lp = J.prompt_ids(2048, ti.vocab, 3 + dist.rank)
            lg = target.generate(lp, args.new)
            J.generate_speculative(target, draft, lp, args.new, args.gamma, oracle_stream=lg,
                                   oracle_p=args.p, oracle_seed=5)  # warm: graphs for the longer context
            r = J.generate_speculative(target, draft, lp, args.new, args.gamma, oracle_stream=lg,
                                       oracle_p=args.p, oracle_seed=5)
            assert r.tokens == lg, "speculative output differs from greedy"
            sweep[f"context 2048, k={args.gamma} oracle p={args.p}"] = {
                "tok_s": (len(r.tokens) - len(lp)) / (r.decode_ms / 1000.0), "accepted": r.accepted,
                "drafted": r.drafted}
        line["sweep"] = sweep
        line["configs"] = other_configs(J, draft, args, peak, dist.local)
        c5 = config5_lines(args, dist, [8])[0]
        line["configs"]["configs[4] batch 8, 4096-token contexts, 256 new tokens"] = {
            key: c5[key] for key in ("value", "acceptance", "hbm_gbs_per_gpu", "roofline", "greedy_batch_tok_s",
                                     "ms_decode")}
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        import oracle as O  # the checker, timed as the CPU baseline only

        line["cpu_baseline"] = cpu_baseline(O, target, draft, prompt, greedy, args)
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
