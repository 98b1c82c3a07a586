"""Tensor-core prompt attention (k_attn_prefill_tc, csrc/attn_prefill_tc.cu).

Prompts of fused MXFP4 models with a bf16 KV pool run their attention on
tcgen05 MMAs: a CTA per (KV head, 128 / group positions), K/V pages by TMA,
Q and the softmax weights as bf16 hi + lo pieces.  Every prompt row's logits
are compared with the oracle running a bf16-rounded cache (lib.rs:401-441),
with the same greedy token required on every row (a near tie, oracle top-2
margin below 1e-3, may resolve either way and is reported).

The cases cover GQA groups 1, 2, 4 and 8 (MMA rows = 128, 64, 32 or 16
positions x the group's heads), a prompt inside one 16-row chunk, prompts
ending mid-page and mid-tile, and prompts of several 256-row passes, whose
later passes start at a position > 0 and read the pages earlier passes wrote.

Two bounds:
  * Against the oracle, a bf16 pool is noisy whichever kernel reads it: the
    GPU's f32 K/V differ from the oracle's in the last bits, and some of them
    round to the neighbouring bf16 value.  Over a few hundred positions that
    alone reaches 1e-4 (the CUDA-core kernel measures 1.0-1.2e-4 on the
    256-position cases here), so prompts are held to 2e-4 against the oracle.
  * The kernel's own error is measured against the CUDA-core kernel on one
    layer, where both read bit-identical K/V: there the logits agree to 1e-5.
"""
import dataclasses
import warnings

import numpy as np
import pytest

import jalapeno as J
import oracle as O
from gpu_util import rel_l2, top2_margin

pytestmark = pytest.mark.gpu

TINY = O.PRESETS["tiny"]
ORACLE_BF16 = 2e-4  # logits against the oracle with a bf16-rounded cache
KERNEL_AB = 1e-5    # logits, tensor-core against CUDA-core kernel on identical K/V


def grouped(q_heads, kv_heads, layers=TINY.layers):
    return dataclasses.replace(TINY, name=f"tiny-q{q_heads}-kv{kv_heads}", q_heads=q_heads,
                               kv_heads=kv_heads, max_positions=2048, layers=layers)


def check_rows(ids, lg, rids, rlg):
    escapes = []
    for i, (a, b) in enumerate(zip(ids, rids)):
        if a != b:
            margin = top2_margin(rlg[i])
            assert margin < 1e-3, f"row {i}: gpu {a} != oracle {b} (top-2 margin {margin})"
            escapes.append((i, a, b, margin))
    if escapes:
        warnings.warn(f"near-tie escapes (row, gpu, oracle, margin): {escapes}")


@pytest.mark.parametrize("n", [20, 130, 300, 1000])
@pytest.mark.parametrize("heads", [(2, 2), (4, 2), (8, 2), (16, 2)],
                         ids=["group1", "group2", "group4", "group8"])
def test_prompt_attention_matches_oracle(heads, n):
    cfg = grouped(*heads)
    ref = O.Model.synthetic(cfg, 3, mxfp4=True)
    m = J.Model.from_config(cfg, 3, mxfp4=True, kv_dtype=J.KV_BF16)
    prompt = O.prompt_ids(n, cfg.vocab, 5)
    assert m.prompt_attention(), "bf16 pools run prompts on tensor cores"
    ids, lg = m.predict(prompt, m.cache(), all=True, logits=True)
    rids, rlg = ref.predict(prompt, ref.cache(round_bf16=True), all=True, logits=True)
    assert rel_l2(lg, rlg) < ORACLE_BF16
    check_rows(ids, lg, rids, rlg)


def test_prompt_then_decode_matches_oracle():
    """Greedy decoding on top of a 600-token prompt: the decode kernels read
    the pages the prompt passes wrote, and the stream follows the oracle."""
    from gpu_util import assert_stream_matches
    cfg = grouped(8, 2)
    ref = O.Model.synthetic(cfg, 4, mxfp4=True)
    m = J.Model.from_config(cfg, 4, mxfp4=True, kv_dtype=J.KV_BF16)
    prompt = O.prompt_ids(600, cfg.vocab, 6)
    assert_stream_matches(m.generate(prompt, 16), ref, prompt, 16, round_bf16=True)


def test_prompt_of_an_exact_number_of_tiles():
    """A prompt of exactly 256 positions (one full pass, two full key tiles):
    no V row is cleared, every page is read whole."""
    cfg = grouped(8, 2)
    ref = O.Model.synthetic(cfg, 5, mxfp4=True)
    m = J.Model.from_config(cfg, 5, mxfp4=True, kv_dtype=J.KV_BF16)
    prompt = O.prompt_ids(256, cfg.vocab, 7)
    ids, lg = m.predict(prompt, m.cache(), all=True, logits=True)
    rids, rlg = ref.predict(prompt, ref.cache(round_bf16=True), all=True, logits=True)
    assert rel_l2(lg, rlg) < ORACLE_BF16
    check_rows(ids, lg, rids, rlg)


@pytest.mark.parametrize("n", [20, 300, 1000])
@pytest.mark.parametrize("heads", [(2, 2), (4, 2), (8, 2), (16, 2)],
                         ids=["group1", "group2", "group4", "group8"])
def test_tensor_core_against_cuda_core_kernel(heads, n):
    """One layer, two models of one seed: the q|k|v pass writes bit-identical
    bf16 K/V in both, so the logits differ only by the two attention kernels'
    arithmetic (summation order; Q and the weights as bf16 hi + lo pieces)."""
    cfg = grouped(*heads, layers=1)
    tc = J.Model.from_config(cfg, 3, mxfp4=True, kv_dtype=J.KV_BF16)
    cc = J.Model.from_config(cfg, 3, mxfp4=True, kv_dtype=J.KV_BF16)
    assert tc.prompt_attention(True) and not cc.prompt_attention(False)
    prompt = O.prompt_ids(n, cfg.vocab, 8)
    ids, lg = tc.predict(prompt, tc.cache(), all=True, logits=True)
    cids, clg = cc.predict(prompt, cc.cache(), all=True, logits=True)
    assert rel_l2(lg, clg) < KERNEL_AB
    check_rows(ids, lg, cids, clg)
    ref = O.Model.synthetic(cfg, 3, mxfp4=True)
    rids, rlg = ref.predict(prompt, ref.cache(round_bf16=True), all=True, logits=True)
    assert rel_l2(lg, rlg) < ORACLE_BF16


def test_f32_pool_keeps_the_cuda_core_kernel():
    m = J.Model.from_config(grouped(8, 2), 3, mxfp4=True, kv_dtype=J.KV_F32)
    assert not m.prompt_attention(True)
