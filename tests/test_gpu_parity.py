"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Tolerances: hidden-state relative L2 < 1e-5 with an f32 KV cache (the
reference's own MXFP4 tolerance, engine/tests/mxfp4.rs:84); logits within
2e-2 abs/rel of the oracle (north star) -- in practice far tighter, so the
tests also bound the relative L2 of the logits; greedy tokens equal
token-for-token over the whole generated stream (a near-tie escape is
allowed only where the oracle's top-2 margin is below 1e-3, and is reported;
see gpu_util.compare_streams).
"""
import dataclasses

import numpy as np
import pytest

import checkpoint as CK
import jalapeno as J
import oracle as O
from gpu_util import (HIDDEN_REL_L2, LOGIT_TOL, assert_stream_matches, compare_streams,
                      first_layers, logits_close, rel_l2)

pytestmark = pytest.mark.gpu

TINY = O.PRESETS["tiny"]
TINY_U = O.PRESETS["tiny-untied"]
DRAFT = O.PRESETS["tiny-draft"]


@pytest.fixture(scope="module")
def oracles():
    return {
        ("tiny", False): O.Model.synthetic(TINY, 0),
        ("tiny", True): O.Model.synthetic(TINY, 0, mxfp4=True),
        ("tiny-untied", False): O.Model.synthetic(TINY_U, 0),
        ("tiny-draft", False): O.Model.synthetic(DRAFT, 1),
        ("tiny-draft", True): O.Model.synthetic(DRAFT, 1, mxfp4=True),
    }


def gpu_model(cfg, seed, mxfp4=False, **kw):
    return J.Model.from_config(cfg, seed, mxfp4=mxfp4, **kw)


PROMPT = O.prompt_ids(20, 1000, 2)


# -- weights -------------------------------------------------------------------

@pytest.mark.parametrize("mxfp4", [False, True])
def test_synthesized_weights_match_oracle_bit_exact(oracles, mxfp4):
    ref = oracles[("tiny", mxfp4)]
    m = gpu_model(TINY, 0, mxfp4)
    for name, key in [("model.embed_tokens.weight", "embed"),
                      ("model.layers.1.mlp.down_proj.weight", "1.down"),
                      ("model.layers.0.self_attn.q_proj.weight", "0.q")]:
        t = ref.tensors[key]
        if t.mxfp4:
            want = np.concatenate([t.packed.reshape(-1), t.scales.reshape(-1)])
        else:
            want = t.bf16.reshape(-1).view(np.uint8)
        got = m.read_tensor(name, want.size)
        np.testing.assert_array_equal(got, want, err_msg=name)


def test_quantizer_on_gpu_matches_reference_restatement():
    # 0.6B gate projection: 3.1M weights through the GPU quantizer
    cfg = O.PRESETS["qwen3-0.6b"]
    one = first_layers(cfg, 1)
    m = J.Model.from_config(one, 1, mxfp4=True, kv_pool_tokens=256, max_pass_rows=64)
    bits = O.synth_tensor(cfg, 1, "gate", 0)
    packed, scales = O.mxfp4_quantize(O.bf16_to_f32(bits).reshape(bits.shape))
    got = m.read_tensor("model.layers.0.mlp.gate_proj.weight", packed.size + scales.size)
    np.testing.assert_array_equal(got[: packed.size], packed.reshape(-1))
    np.testing.assert_array_equal(got[packed.size:], scales.reshape(-1))


# -- forward pass ---------------------------------------------------------------

@pytest.mark.parametrize("key", [("tiny", False), ("tiny", True), ("tiny-untied", False)])
def test_hidden_states_match_oracle(oracles, key):
    ref = oracles[key]
    m = gpu_model(O.PRESETS[key[0]], 0, key[1], kv_dtype=J.KV_F32)
    for layers in (1, ref.cfg.layers):
        got = m.hidden(PROMPT, layers)
        want = ref.hidden(PROMPT, layers)
        assert rel_l2(got, want) < HIDDEN_REL_L2, layers


@pytest.mark.parametrize("kv", [J.KV_F32, J.KV_BF16])
@pytest.mark.parametrize("key", [("tiny", False), ("tiny", True)])
def test_logits_match_oracle(oracles, key, kv):
    ref = oracles[key]
    m = gpu_model(TINY, 0, key[1], kv_dtype=kv)
    ids, lg = m.predict(PROMPT, m.cache(), all=True, logits=True)
    # the reference path (f32 KV) within the north-star tolerance
    rids, rlg = ref.predict(PROMPT, ref.cache(), all=True, logits=True)
    assert logits_close(lg, rlg)
    # against an oracle that rounds K/V like the cache under test: much tighter
    # (a bf16 cache can round a last-bit difference of K to the next bf16
    # value, so its bound is looser than the f32 cache's)
    bids, blg = ref.predict(PROMPT, ref.cache(round_bf16=kv == J.KV_BF16), all=True, logits=True)
    assert rel_l2(lg, blg) < (1e-5 if kv == J.KV_F32 else 1e-4)
    assert ids == bids


@pytest.mark.parametrize("n", [66, 96, 200])
@pytest.mark.parametrize("key", [("tiny", False), ("tiny", True)])
def test_multi_chunk_prefill_matches_oracle(oracles, key, n):
    """One predict call over several passes (16-row chunks), spanning KV pages:
    each pass's row descriptors reach the GPU intact although the host queues
    the next pass's before the earlier ones have run."""
    ref = oracles[key]
    m = gpu_model(TINY, 0, key[1], kv_dtype=J.KV_F32)
    prompt = O.prompt_ids(n, 1000, 3)
    for _ in range(3):  # the host runs ahead of the device differently each time
        ids, lg = m.predict(prompt, m.cache(), all=False, logits=True)
        rids, rlg = ref.predict(prompt, ref.cache(), all=False, logits=True)
        assert rel_l2(lg, rlg) < 1e-5 and ids == rids


@pytest.mark.parametrize("n", [300, 480])
@pytest.mark.parametrize("key", [("tiny", False), ("tiny", True)])
def test_long_context_attention_windows_match_oracle(oracles, key, n):
    """Rows past 128 positions: one CTA per 128-position window, partial
    softmax sums merged by the last window to finish.  Logits of the prompt's
    last row, then greedy decoding on top of the long context."""
    ref = oracles[key]
    m = gpu_model(TINY, 0, key[1], kv_dtype=J.KV_F32)
    prompt = O.prompt_ids(n, 1000, 4)
    ids, lg = m.predict(prompt, m.cache(), all=False, logits=True)
    rids, rlg = ref.predict(prompt, ref.cache(), all=False, logits=True)
    assert rel_l2(lg, rlg) < 1e-5 and ids == rids
    assert_stream_matches(m.generate(prompt, 12), ref, prompt, 12)


def test_long_context_speculative_equals_greedy():
    target = gpu_model(TINY, 0, True)
    draft = gpu_model(DRAFT, 1, True)
    prompt = O.prompt_ids(300, 1000, 4)
    greedy = target.generate(prompt, 24)
    for p in (0.0, 0.5):
        r = J.generate_speculative(target, draft, prompt, 24, 3, oracle_stream=greedy, oracle_p=p,
                                   oracle_seed=7)
        assert r.tokens == greedy


def test_decode_after_prefill_matches_oracle(oracles):
    ref = oracles[("tiny", True)]
    m = gpu_model(TINY, 0, True, kv_dtype=J.KV_F32)
    c, rc = m.cache(), ref.cache()
    m.predict(PROMPT, c)
    ref.predict(PROMPT, rc)
    for tok in (5, 17, 999, 0):
        ids, lg = m.predict([tok], c, logits=True)
        rids, rlg = ref.predict([tok], rc, logits=True)
        assert rel_l2(lg, rlg) < 1e-5
    assert c.len == rc.len == len(PROMPT) + 4


@pytest.mark.parametrize("key", [("tiny", False), ("tiny", True), ("tiny-untied", False)])
def test_greedy_matches_oracle_token_for_token(oracles, key):
    ref = oracles[key]
    m = gpu_model(O.PRESETS[key[0]], 0, key[1], kv_dtype=J.KV_F32)
    tokens = m.generate(PROMPT, 24)
    assert tokens[:20] == PROMPT
    assert_stream_matches(tokens, ref, PROMPT, 24)


def test_greedy_with_bf16_kv_matches_rounded_oracle(oracles):
    ref = oracles[("tiny", True)]
    m = gpu_model(TINY, 0, True, kv_dtype=J.KV_BF16)
    tokens = m.generate(PROMPT, 24)
    assert_stream_matches(tokens, ref, PROMPT, 24, round_bf16=True)


def test_rows_are_batch_invariant():
    # a row's logits do not depend on how many rows share its pass
    m = gpu_model(TINY, 0, True)
    c1 = m.cache()
    m.predict(PROMPT, c1)
    c5 = m.cache()
    m.predict(PROMPT, c5)
    extra = [3, 44, 555, 6, 77]
    one = []
    for t in extra:
        _, lg = m.predict([t], c1, logits=True)
        one.append(lg[0])
    _, five = m.predict(extra, c5, all=True, logits=True)
    np.testing.assert_array_equal(np.array(one), five)


def test_next_token_and_cache_truncation():
    m = gpu_model(TINY, 0, True)
    c = m.cache()
    first = m.predict(PROMPT, c)[0]
    assert m.next_token(PROMPT) == first
    m.predict([1, 2, 3], c)
    c.truncate(len(PROMPT))  # roll back like KvCache::truncate
    after = m.predict([first], c, logits=True)[1]
    fresh = m.cache()
    m.predict(PROMPT, fresh)
    np.testing.assert_array_equal(after, m.predict([first], fresh, logits=True)[1])
    with pytest.raises(J.JlError):
        c.truncate(c.len + 1)


# -- checkpoints through the loader -------------------------------------------

@pytest.mark.parametrize("quantized", [False, True])
def test_loaded_checkpoint_equals_synthesized_model(tmp_path, oracles, quantized):
    ref = oracles[("tiny", quantized)]
    CK.write_model(ref, tmp_path, quantized=quantized)
    loaded = J.Model.load(tmp_path)
    synth = gpu_model(TINY, 0, quantized)
    a = loaded.predict(PROMPT, loaded.cache(), all=True, logits=True)[1]
    b = synth.predict(PROMPT, synth.cache(), all=True, logits=True)[1]
    np.testing.assert_array_equal(a, b)
    assert loaded.info.mxfp4_projections == int(quantized)


def test_reference_converter_layout_with_mxfp4_head(tmp_path):
    # python/quantize_mxfp4.py:74-86 quantizes embed and lm_head too
    ref = O.Model.synthetic(TINY_U, 4, mxfp4=True, mxfp4_embed=True)
    CK.write_model(ref, tmp_path, quantized=True)
    m = J.Model.load(tmp_path, kv_dtype=J.KV_F32)
    assert m.info.mxfp4_head == 1
    got = m.hidden(PROMPT, 1)
    assert rel_l2(got, ref.hidden(PROMPT, 1)) < HIDDEN_REL_L2
    ids, lg = m.predict(PROMPT, m.cache(), all=True, logits=True)
    rids, rlg = ref.predict(PROMPT, ref.cache(), all=True, logits=True)
    assert rel_l2(lg, rlg) < 1e-5


# -- speculative decoding --------------------------------------------------------

@pytest.fixture(scope="module")
def pair():
    target = gpu_model(TINY, 0, True)
    draft = gpu_model(DRAFT, 1, True)
    return target, draft


@pytest.mark.parametrize("mode", [J.SPEC_DEVICE, J.SPEC_HOST])
def test_speculative_equals_greedy_with_rejections(pair, mode):
    # engine/tests/generation.rs:69-92
    target, draft = pair
    greedy = target.generate(PROMPT, 40)
    for schedule in (J.DraftSchedule.fixed(5), J.DraftSchedule.adaptive(5, 8),
                     J.DraftSchedule.fixed(1), J.DraftSchedule.fixed(4)):
        r = J.generate_scheduled(target, draft, PROMPT, 40, schedule, mode=mode)
        assert r.tokens == greedy
        assert r.accepted < r.drafted


def test_device_loop_matches_host_loop_bookkeeping(pair):
    target, draft = pair
    for schedule in (J.DraftSchedule.fixed(4), J.DraftSchedule.adaptive(2, 8)):
        d = J.generate_scheduled(target, draft, PROMPT, 30, schedule, mode=J.SPEC_DEVICE)
        h = J.generate_scheduled(target, draft, PROMPT, 30, schedule, mode=J.SPEC_HOST)
        assert d.tokens == h.tokens
        assert (d.drafted, d.accepted, d.rounds) == (h.drafted, h.accepted, h.rounds)
        assert d.round_stats == h.round_stats
        assert d.draft.passes == h.draft.passes and d.verify.passes == h.verify.passes


def test_speculative_control_flow_matches_oracle_loop(oracles):
    # same predictions -> same rounds, acceptance and pass counts as
    # engine/src/speculative.rs (restated in oracle.generate_scheduled)
    t_ref, d_ref = oracles[("tiny", False)], oracles[("tiny-draft", False)]
    target = gpu_model(TINY, 0, False, kv_dtype=J.KV_F32)
    draft = gpu_model(DRAFT, 1, False, kv_dtype=J.KV_F32)
    greedy = target.generate(PROMPT, 30)
    chk = assert_stream_matches(greedy, t_ref, PROMPT, 30)
    assert not chk.escapes, "streams diverged at a near tie; control-flow comparison needs equal streams"
    stream = greedy
    for p in (0.0, 0.25, 0.5):
        g = J.generate_scheduled(target, draft, PROMPT, 30, J.DraftSchedule.adaptive(4, 8),
                                 oracle_stream=stream, oracle_p=p, oracle_seed=11)
        o = O.generate_scheduled(t_ref, d_ref, PROMPT, 30, O.DraftSchedule.adaptive_(4, 8),
                                 oracle_stream=stream, oracle_p=p, oracle_seed=11)
        assert g.tokens == o.tokens
        assert (g.drafted, g.accepted, g.rounds) == (o.drafted, o.accepted, o.rounds)
        assert g.round_stats == [tuple(s) for s in o.round_stats]
        assert g.draft.passes == o.draft.passes


@pytest.mark.parametrize("p", [0.0, 0.25, 0.5])
def test_oracle_draft_sweeps_acceptance(pair, p):
    target, draft = pair
    greedy = target.generate(PROMPT, 40)
    r = J.generate_speculative(target, draft, PROMPT, 40, 4, oracle_stream=greedy, oracle_p=p,
                               oracle_seed=3)
    assert r.tokens == greedy
    if p == 0.0:
        assert r.accepted == r.drafted
    else:
        assert 0 < r.accepted < r.drafted


def test_adaptive_bookkeeping_on_gpu(pair):
    # engine/tests/generation.rs:128-202
    target, draft = pair
    greedy = target.generate(PROMPT, 15)
    for count in (0, 1, 15):
        r = J.generate_scheduled(target, draft, PROMPT, count, J.DraftSchedule.adaptive(5, 8))
        assert r.tokens == greedy[: len(PROMPT) + count]
        assert r.rounds == r.verify.passes == len(r.round_stats)
        assert r.drafted == sum(s[1] for s in r.round_stats)
        assert r.accepted == sum(s[2] for s in r.round_stats)
        assert all(1 <= s[0] <= 8 for s in r.round_stats)
        if count > 0:
            assert r.prefill.passes == 2
            assert r.draft.passes < r.drafted + r.rounds
        else:
            assert r.prefill.passes == 0
    # self-draft (a second handle of the same weights): everything accepted
    twin = gpu_model(TINY, 0, True)
    r = J.generate_scheduled(target, twin, PROMPT, 6, J.DraftSchedule.adaptive(2, 4))
    assert r.tokens == greedy[: len(PROMPT) + 6]
    assert r.round_stats[0][3] == 3
    assert r.draft.passes == 4


def test_eos_stops_greedy_and_speculative():
    base = gpu_model(TINY, 0, True)
    greedy = base.generate(PROMPT, 30)
    eos = greedy[len(PROMPT) + 5]
    stop = greedy.index(eos, len(PROMPT)) + 1
    cfg = dataclasses.replace(TINY, eos=eos)
    target = gpu_model(cfg, 0, True)
    draft = gpu_model(dataclasses.replace(DRAFT, eos=eos), 1, True)
    assert target.generate(PROMPT, 30) == greedy[:stop]
    for mode in (J.SPEC_DEVICE, J.SPEC_HOST):
        r = J.generate_speculative(target, draft, PROMPT, 30, 4, mode=mode)
        assert r.tokens == greedy[:stop]
        r = J.generate_speculative(target, draft, PROMPT, 30, 4, mode=mode, oracle_stream=greedy)
        assert r.tokens == greedy[:stop]


def test_context_limit_bounds_generation():
    cfg = dataclasses.replace(TINY, max_positions=len(PROMPT) + 3)
    target = gpu_model(cfg, 0, True)
    draft = gpu_model(dataclasses.replace(DRAFT, max_positions=len(PROMPT) + 3), 1, True)
    g = target.generate(PROMPT, 20)
    assert len(g) == len(PROMPT) + 3
    for mode in (J.SPEC_DEVICE, J.SPEC_HOST):
        r = J.generate_speculative(target, draft, PROMPT, 20, 5, mode=mode)
        assert r.tokens == g
    with pytest.raises(J.JlError):
        target.predict(list(range(len(PROMPT) + 4)), target.cache())


def test_invalid_tokens_are_rejected_on_the_host():
    m = gpu_model(TINY, 0, True)
    with pytest.raises(J.JlError) as e:
        m.predict([1000], m.cache())
    assert e.value.status == J.JL_ERR_INVALID_ARG
