"""Batched generation through the C ABI (jl_generate_batch,
jl_generate_speculative_batch): every sequence of a batch gets exactly the
tokens and counters that the single-sequence call gives it
(model.rs:268-285, speculative.rs:43-143), whatever the batch size, the
split of passes over 16 rows into chunks, prompt lengths, schedules, oracle
settings, end-of-sequence and context limits."""
import dataclasses

import numpy as np
import pytest

import jalapeno as J
import oracle as O

pytestmark = pytest.mark.gpu

TINY = O.PRESETS["tiny"]
DRAFT = O.PRESETS["tiny-draft"]
POOL = 16384  # KV pool tokens: room for every sequence of the largest batch


def model(cfg, seed, mxfp4=True, **kw):
    kw.setdefault("kv_pool_tokens", POOL)
    return J.Model.from_config(cfg, seed, mxfp4=mxfp4, **kw)


@pytest.fixture(scope="module")
def pair():
    return model(TINY, 0), model(DRAFT, 1)


def prompts(B, seed=7, longest=40):
    rng = np.random.default_rng(seed)
    return [O.prompt_ids(int(rng.integers(1, longest)), 1000, 100 + i) for i in range(B)]


def same_counters(a, b):
    assert a.tokens == b.tokens
    assert (a.drafted, a.accepted, a.rounds) == (b.drafted, b.accepted, b.rounds)
    assert a.round_stats == b.round_stats
    assert (a.prefill.passes, a.draft.passes, a.verify.passes) == (b.prefill.passes, b.draft.passes,
                                                                   b.verify.passes)


@pytest.mark.parametrize("mxfp4", [False, True])
@pytest.mark.parametrize("B", [1, 3, 17, 40])
def test_greedy_batch_equals_single(mxfp4, B):
    m = model(TINY, 0, mxfp4)
    ps = prompts(B)
    r = J.generate_batch(m, ps, 12)
    assert len(r.results) == B
    for p, s in zip(ps, r.results):
        assert s.tokens == m.generate(p, 12)
    # one round per generated token after the prefill's, every chunk of 16 rows a pass
    assert r.rounds == max(len(s.tokens) - len(p) for p, s in zip(ps, r.results)) - 1
    assert r.rounds <= r.target_passes <= r.rounds * ((B + 15) // 16)
    assert r.decode_ms > 0 and r.prefill_ms > 0


@pytest.mark.parametrize("B", [1, 2, 5, 20])
def test_speculative_batch_equals_single(pair, B):
    target, draft = pair
    ps = prompts(B)
    greedy = [target.generate(p, 40) for p in ps]
    p_of = [(0.0, 0.25, 0.5, 1.0)[i % 4] for i in range(B)]
    seeds = [11 + i for i in range(B)]
    r = J.generate_speculative_batch(target, draft, ps, 24, J.DraftSchedule.fixed(4), oracle_streams=greedy,
                                     oracle_p=p_of, oracle_seeds=seeds)
    for i, s in enumerate(r.results):
        one = J.generate_speculative(target, draft, ps[i], 24, 4, oracle_stream=greedy[i], oracle_p=p_of[i],
                                     oracle_seed=seeds[i])
        assert one.tokens == greedy[i][: len(ps[i]) + 24]
        same_counters(s, one)
    assert r.rounds == max(s.rounds for s in r.results)
    # verifies run as chunks of at most 16 rows
    assert r.rounds <= r.target_passes <= r.rounds * ((5 * B + 15) // 16)
    assert r.draft_passes > 0


def test_real_draft_and_mixed_schedules(pair):
    target, draft = pair
    ps = prompts(6, seed=3)
    scheds = [J.DraftSchedule.fixed(1), J.DraftSchedule.adaptive(2, 6), J.DraftSchedule.fixed(3),
              J.DraftSchedule.adaptive(5, 8), J.DraftSchedule.fixed(8), J.DraftSchedule.adaptive(1, 2)]
    greedy = [target.generate(p, 30) for p in ps]
    streams = [greedy[0], None, greedy[2], greedy[3], None, greedy[5]]
    r = J.generate_speculative_batch(target, draft, ps, 20, scheds, oracle_streams=streams, oracle_p=0.2,
                                     oracle_seeds=5)
    for i, s in enumerate(r.results):
        one = J.generate_scheduled(target, draft, ps[i], 20, scheds[i], oracle_stream=streams[i], oracle_p=0.2,
                                   oracle_seed=5)
        assert one.tokens == greedy[i][: len(ps[i]) + 20]
        same_counters(s, one)


def test_self_draft_accepts_everything():
    target = model(TINY, 0)
    twin = model(TINY, 0)
    ps = prompts(18, seed=4)
    r = J.generate_speculative_batch(target, twin, ps, 10, J.DraftSchedule.fixed(4))
    for p, s in zip(ps, r.results):
        assert s.tokens == target.generate(p, 10)
        assert s.accepted == s.drafted


def test_eos_stops_each_sequence_on_its_own():
    base = model(TINY, 0)
    ps = prompts(9, seed=5)
    g = [base.generate(p, 30) for p in ps]
    eos = g[0][len(ps[0]) + 5]
    target = model(dataclasses.replace(TINY, eos=eos), 0)
    draft = model(dataclasses.replace(DRAFT, eos=eos), 1)
    want = [target.generate(p, 30) for p in ps]
    assert len(set(len(w) - len(p) for w, p in zip(want, ps))) > 1  # sequences stop at different lengths
    assert [s.tokens for s in J.generate_batch(target, ps, 30).results] == want
    for streams in (None, g):
        r = J.generate_speculative_batch(target, draft, ps, 30, J.DraftSchedule.fixed(4), oracle_streams=streams)
        assert [s.tokens for s in r.results] == want


def test_context_limit_and_empty_counts():
    limit = 30
    target = model(dataclasses.replace(TINY, max_positions=limit), 0)
    draft = model(dataclasses.replace(DRAFT, max_positions=limit), 1)
    ps = [O.prompt_ids(n, 1000, 40 + n) for n in (3, 17, 27, 29, 30, 31)]
    for count in (0, 1, 20):
        g = J.generate_batch(target, ps, count)
        s = J.generate_speculative_batch(target, draft, ps, count, J.DraftSchedule.fixed(4))
        for i, p in enumerate(ps):
            want = target.generate(p, count)
            assert len(want) == max(len(p), min(len(p) + count, limit))
            assert g.results[i].tokens == want
            one = J.generate_speculative(target, draft, p, count, 4)
            same_counters(s.results[i], one)


def test_pool_exhaustion_is_an_error():
    target = model(TINY, 0, kv_pool_tokens=256)
    draft = model(DRAFT, 1, kv_pool_tokens=256)
    ps = prompts(12, seed=6)
    with pytest.raises(J.JlError) as e:
        J.generate_speculative_batch(target, draft, ps, 60, J.DraftSchedule.fixed(4))
    assert e.value.status == J.JL_ERR_OOM
    # the models stay usable
    assert J.generate_batch(target, ps[:1], 5).results[0].tokens == target.generate(ps[0], 5)


def test_argument_errors(pair):
    target, draft = pair
    ps = prompts(3)
    with pytest.raises(J.JlError):
        J.generate_batch(target, [], 5)
    with pytest.raises(J.JlError):
        J.generate_batch(target, [[1, 2]] * 65, 5)
    with pytest.raises(J.JlError):
        J.generate_batch(target, [[1, 2], []], 5)
    with pytest.raises(J.JlError):
        J.generate_batch(target, [[1, 5000]], 5)  # id outside the vocabulary
    with pytest.raises(J.JlError):
        J.generate_speculative_batch(target, target, ps, 5, J.DraftSchedule.fixed(4))
    with pytest.raises(J.JlError):  # 64 x (8 + 1) rows exceed the 512 a round may verify
        J.generate_speculative_batch(target, draft, [[1, 2]] * 64, 5, J.DraftSchedule.fixed(8))
    with pytest.raises(J.JlError):
        J.generate_speculative_batch(target, draft, ps, 5, J.DraftSchedule.fixed(4), oracle_streams=[[1]] * 3,
                                     oracle_p=1.5)
