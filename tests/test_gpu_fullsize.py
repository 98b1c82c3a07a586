"""Full-size BASELINE.json architectures on the GPU.

The CPU oracle checks the first decoder layer of every architecture (its
tensors are the same whatever the layer count), the whole 0.6B model, the
64-token greedy streams of Qwen3-1.7B bf16 and MXFP4 (configs 1 and 2, the
reference's own acceptance test: engine/tests/generation.rs:6-28), and the
8B model at full depth (last-row logits and the first greedy tokens).  The
8B speculative loop is also checked through size-independent properties:
speculative output equals greedy output, oracle-draft p=0 accepts every
proposal.
"""
import numpy as np
import pytest

import jalapeno as J
import oracle as O
from gpu_util import HIDDEN_REL_L2, assert_stream_matches, first_layers, logits_close, rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.slow]

PROMPT = O.prompt_ids(32, 151936, 2)


@pytest.mark.parametrize("preset,mxfp4", [("qwen3-0.6b", True), ("qwen3-1.7b", False),
                                          ("qwen3-1.7b", True), ("qwen3-8b", True)])
def test_first_layer_matches_oracle(preset, mxfp4):
    cfg = O.PRESETS[preset]
    one = first_layers(cfg, 1)
    seed = 1 if preset == "qwen3-0.6b" else 0
    ref = O.Model.synthetic(one, seed, mxfp4=mxfp4)
    m = J.Model.from_config(one, seed, mxfp4=mxfp4, kv_dtype=J.KV_F32, kv_pool_tokens=1024,
                            max_pass_rows=64)
    got = m.hidden(PROMPT[:8], 1)
    assert rel_l2(got, ref.hidden(PROMPT[:8], 1)) < HIDDEN_REL_L2


def test_qwen3_0_6b_mxfp4_logits_match_oracle():
    cfg = O.PRESETS["qwen3-0.6b"]
    ref = O.Model.synthetic(cfg, 1, mxfp4=True)
    m = J.Model.from_config(cfg, 1, mxfp4=True, kv_dtype=J.KV_F32, kv_pool_tokens=1024,
                            max_pass_rows=64)
    prompt = PROMPT[:8]
    ids, lg = m.predict(prompt, m.cache(), logits=True)
    rids, rlg = ref.predict(prompt, ref.cache(), logits=True)
    assert logits_close(lg, rlg)
    assert rel_l2(lg, rlg) < 1e-4
    assert ids == rids


@pytest.mark.parametrize("mxfp4", [False, True])
def test_qwen3_1_7b_greedy_stream_matches_oracle_full_depth(mxfp4):
    """BASELINE configs 1 and 2: 32-token prompt, 64 greedy tokens, every one
    equal to the oracle's (f32 KV, the reference's precision)."""
    cfg = O.PRESETS["qwen3-1.7b"]
    ref = O.Model.synthetic(cfg, 0, mxfp4=mxfp4)
    m = J.Model.from_config(cfg, 0, mxfp4=mxfp4, kv_dtype=J.KV_F32, kv_pool_tokens=1024)
    ids, lg = m.predict(PROMPT, m.cache(), logits=True)
    rids, rlg = ref.predict(PROMPT, ref.cache(), logits=True)
    assert logits_close(lg, rlg) and rel_l2(lg, rlg) < 1e-4 and ids == rids
    assert_stream_matches(m.generate(PROMPT, 64), ref, PROMPT, 64)


def test_qwen3_8b_full_depth_matches_oracle():
    """The headline target at full depth: last-row logits of the 32-token
    prompt and the first 8 greedy tokens against the oracle."""
    cfg = O.PRESETS["qwen3-8b"]
    ref = O.Model.synthetic(cfg, 0, mxfp4=True)
    m = J.Model.from_config(cfg, 0, mxfp4=True, kv_dtype=J.KV_F32, kv_pool_tokens=1024)
    ids, lg = m.predict(PROMPT, m.cache(), logits=True)
    rids, rlg = ref.predict(PROMPT, ref.cache(), logits=True)
    assert logits_close(lg, rlg), "logits outside 2e-2 abs/rel"
    assert rel_l2(lg, rlg) < 1e-4 and ids == rids
    assert_stream_matches(m.generate(PROMPT, 8), ref, PROMPT, 8)


def test_qwen3_8b_speculative_properties():
    target = J.Model.from_config(O.PRESETS["qwen3-8b"], 0, mxfp4=True, kv_pool_tokens=4096)
    draft = J.Model.from_config(O.PRESETS["qwen3-0.6b"], 1, mxfp4=True, kv_pool_tokens=4096)
    greedy = target.generate(PROMPT, 24)
    assert len(greedy) == len(PROMPT) + 24
    r = J.generate_speculative(target, draft, PROMPT, 24, 4)
    assert r.tokens == greedy
    r = J.generate_speculative(target, draft, PROMPT, 24, 4, oracle_stream=greedy)
    assert r.tokens == greedy and r.accepted == r.drafted
    _, lg = target.predict(PROMPT[:4], target.cache(), logits=True)
    assert np.isfinite(lg).all()


def test_long_context_draft_and_verify_attention():
    """A 600-token context: the draft's one-row steps (CUDA-core projections,
    attention on raw q|k|v) and the target's 5-row verify passes both split
    each row's attention over 128-position windows; speculative output must
    still equal greedy output, and the 0.6B's own greedy stream must agree
    with the draft path's proposals when p = 0 (every proposal accepted)."""
    target = J.Model.from_config(O.PRESETS["qwen3-8b"], 0, mxfp4=True, kv_pool_tokens=2048)
    draft = J.Model.from_config(O.PRESETS["qwen3-0.6b"], 1, mxfp4=True, kv_pool_tokens=2048)
    prompt = O.prompt_ids(600, 151936, 3)
    greedy = target.generate(prompt, 16)
    r = J.generate_speculative(target, draft, prompt, 16, 4, oracle_stream=greedy, oracle_p=0.25,
                               oracle_seed=5)
    assert r.tokens == greedy
    r = J.generate_speculative(target, draft, prompt, 16, 4)
    assert r.tokens == greedy


def test_draft_step_path_proposes_the_models_own_greedy_tokens():
    """The draft-step kernels (CUDA-core MXFP4 projections, attention on raw
    q|k|v, the RMSNorm division applied to the dot products) against the
    tensor-core path the greedy loop takes: with the same Qwen3-0.6B MXFP4
    weights as target and draft, the real draft's proposals are the target's
    own greedy tokens except at a near tie of the two paths' roundings, so
    almost every proposal is accepted."""
    cfg = O.PRESETS["qwen3-0.6b"]
    target = J.Model.from_config(cfg, 1, mxfp4=True, kv_pool_tokens=1024)
    draft = J.Model.from_config(cfg, 1, mxfp4=True, kv_pool_tokens=1024)
    greedy = target.generate(PROMPT, 40)
    r = J.generate_speculative(target, draft, PROMPT, 40, 4)
    assert r.tokens == greedy
    assert r.drafted > 0 and r.accepted >= 0.9 * r.drafted, (r.accepted, r.drafted)
