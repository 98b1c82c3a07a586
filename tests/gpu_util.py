"""Helpers for the GPU parity tests (comparisons against the CPU oracle)."""
from __future__ import annotations

import dataclasses

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


def compare_streams(gpu_tokens, oracle_model: O.Model, prompt, n_new, round_bf16=False,
                    tie_margin=1e-3):
    """Token-for-token comparison of a GPU greedy stream with the oracle.
    Returns the number of generated positions compared.  A mismatch is only
    tolerated where the oracle's own top-2 logit margin is below tie_margin
    (a near tie the two summation orders may resolve differently); the
    comparison stops there because later tokens depend on it."""
    cache = oracle_model.cache(round_bf16)
    ids, lg = oracle_model.predict(prompt, cache, logits=True)
    tokens = list(prompt)
    for i in range(n_new):
        expected = ids[0]
        pos = len(prompt) + i
        if pos >= len(gpu_tokens):
            return i
        if gpu_tokens[pos] != expected:
            margin = top2_margin(lg[0])
            assert margin < tie_margin, (
                f"token {i}: gpu {gpu_tokens[pos]} != oracle {expected} (top-2 margin {margin})")
            return i
        tokens.append(expected)
        if expected == oracle_model.eos:
            return i + 1
        ids, lg = oracle_model.predict([expected], cache, logits=True)
    return n_new


def first_layers(cfg: O.Config, layers: int) -> O.Config:
    """Same seeded stream, truncated to the first `layers` layers (tensor
    indices of those layers do not depend on the layer count)."""
    return dataclasses.replace(cfg, layers=layers)
