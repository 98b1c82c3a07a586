"""Helpers for the GPU parity tests (comparisons against the CPU oracle)."""
from __future__ import annotations

import dataclasses
import warnings

import numpy as np

import oracle as O

# north_star: logits within 2e-2 abs/rel of the reference on the same weights
LOGIT_TOL = 2e-2
# engine/tests/mxfp4.rs:84: hidden-state relative L2 below 1e-5
HIDDEN_REL_L2 = 1e-5


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def logits_close(actual, expected, tol=LOGIT_TOL) -> bool:
    actual = np.asarray(actual, np.float64)
    expected = np.asarray(expected, np.float64)
    return bool(np.all(np.abs(actual - expected) <= tol * np.maximum(1.0, np.abs(expected))))


def top2_margin(logits_row) -> float:
    top = np.partition(np.asarray(logits_row, np.float64), -2)[-2:]
    return float(abs(top[1] - top[0]))


@dataclasses.dataclass
class StreamCheck:
    compared: int = 0      # generated positions compared with the oracle
    escapes: list = dataclasses.field(default_factory=list)  # (index, gpu, oracle, top-2 margin)


def compare_streams(gpu_tokens, oracle_model: O.Model, prompt, n_new, round_bf16=False,
                    tie_margin=1e-3) -> StreamCheck:
    """Token-for-token comparison of a GPU greedy stream with the oracle over
    every generated position.  The oracle decodes the GPU's own tokens
    (teacher forcing), so one near tie does not end the comparison.  A
    mismatch is tolerated only where the oracle's top-2 logit margin is below
    tie_margin (a near tie the two summation orders may resolve differently)
    and is recorded as an escape; any other mismatch fails."""
    cache = oracle_model.cache(round_bf16)
    ids, lg = oracle_model.predict(prompt, cache, logits=True)
    check = StreamCheck()
    for i in range(n_new):
        pos = len(prompt) + i
        if pos >= len(gpu_tokens):
            break
        expected, got = ids[0], gpu_tokens[pos]
        if got != expected:
            margin = top2_margin(lg[0])
            assert margin < tie_margin, (
                f"token {i}: gpu {got} != oracle {expected} (top-2 margin {margin})")
            check.escapes.append((i, got, expected, margin))
        check.compared += 1
        if got == oracle_model.eos or pos + 1 >= len(gpu_tokens):
            break
        ids, lg = oracle_model.predict([got], cache, logits=True)
    return check


def assert_stream_matches(gpu_tokens, oracle_model: O.Model, prompt, n_new, **kw) -> StreamCheck:
    """compare_streams over the whole generated stream: the prompt is kept,
    the stream has n_new tokens (or ends at eos or the context limit), every
    one is compared, and near-tie escapes are reported as warnings."""
    assert list(gpu_tokens[: len(prompt)]) == list(prompt)
    generated = len(gpu_tokens) - len(prompt)
    limit = min(n_new, oracle_model.context_limit() - len(prompt))
    assert generated == limit or (generated > 0 and gpu_tokens[-1] == oracle_model.eos), (
        f"{generated} tokens generated, expected {limit}")
    check = compare_streams(gpu_tokens, oracle_model, prompt, n_new, **kw)
    assert check.compared == generated, (check.compared, generated)
    if check.escapes:
        warnings.warn(f"near-tie escapes (index, gpu, oracle, margin): {check.escapes}")
    return check


def first_layers(cfg: O.Config, layers: int) -> O.Config:
    """Same seeded stream, truncated to the first `layers` layers (tensor
    indices of those layers do not depend on the layer count)."""
    return dataclasses.replace(cfg, layers=layers)
