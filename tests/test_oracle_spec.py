"""Pins the oracle's speculative loop and scheduler to the reference's tests.

engine/src/speculative.rs:145-190, engine/src/scheduler.rs:47-76 and the
bookkeeping invariants of engine/tests/generation.rs:94-183 (re-pointed at
seeded synthetic models, since the reference's checkpoints are not shipped).
"""
import pytest

import oracle as O
from oracle import DraftSchedule, constant_for_test, generate_scheduled, generate_speculative


# -- engine/src/speculative.rs tests -----------------------------------------

def test_accepted_and_corrected_eos_stop_generation():
    target = constant_for_test(3)
    for draft_token in (1, 3):
        draft = constant_for_test(draft_token)
        r = generate_scheduled(target, draft, [0], 5, DraftSchedule.adaptive_(3, 5))
        assert r.tokens == [0, 3]
        assert r.rounds == 1


def test_rejected_draft_eos_and_gamma_one_preserve_target_output():
    target = constant_for_test(2)
    draft = constant_for_test(3)
    for gamma in (1, 5):
        r = generate_scheduled(target, draft, [0], 20, DraftSchedule.fixed(gamma))
        assert r.tokens == target.generate([0], 20)
        assert len(r.tokens) == 6
        assert r.accepted == 0


def test_zero_budget_and_context_boundary_do_not_overrun():
    target = constant_for_test(2)
    empty = generate_scheduled(target, target, [0], 0, DraftSchedule.fixed(5))
    assert empty.tokens == [0]
    assert empty.prefill.passes == 0
    r = generate_scheduled(target, target, [0] * 5, 20, DraftSchedule.fixed(5))
    assert r.tokens == [0, 0, 0, 0, 0, 2]
    assert r.draft.passes == 0


# -- engine/src/scheduler.rs tests --------------------------------------------

def test_feedback_increases_and_decreases_budget_within_bounds():
    s = DraftSchedule.adaptive_(4, 5)
    s.observe(4, 4)
    assert s.gamma == 5
    s.observe(5, 5)
    assert s.gamma == 5
    s.observe(1, 5)
    assert s.gamma == 2
    s.observe(0, 2)
    assert s.gamma == 1
    s.observe(0, 1)
    assert s.gamma == 1


def test_fixed_and_truncated_rounds_keep_the_budget():
    f = DraftSchedule.fixed(5)
    f.observe(0, 5)
    assert f.gamma == 5
    a = DraftSchedule.adaptive_(5, 8)
    a.observe(1, 1)
    assert a.gamma == 5
    with pytest.raises(ValueError):
        DraftSchedule.adaptive_(0, 8)
    with pytest.raises(ValueError):
        DraftSchedule.adaptive_(9, 8)


# -- engine/tests/generation.rs invariants on synthetic models ---------------

@pytest.fixture(scope="module")
def models():
    target = O.Model.synthetic("tiny", 0)
    draft = O.Model.synthetic("tiny-draft", 1)
    target_q = O.Model.synthetic("tiny", 0, mxfp4=True)
    draft_q = O.Model.synthetic("tiny-draft", 1, mxfp4=True)
    return {"": (target, draft), "-MXFP4": (target_q, draft_q)}


def test_speculative_matches_greedy_with_rejections(models):
    prompt = O.prompt_ids(20, 1000, 2)
    for suffix, (target, draft) in models.items():
        greedy = target.generate(prompt, 15)
        for schedule in (DraftSchedule.fixed(5), DraftSchedule.adaptive_(5, 8)):
            r = generate_scheduled(target, draft, prompt, 15, schedule)
            assert r.tokens == greedy, suffix
            assert r.accepted < r.drafted


def test_self_draft_accepts_everything(models):
    # engine/tests/generation.rs:122-125
    target, _ = models[""]
    prompt = O.prompt_ids(20, 1000, 2)
    expected = target.generate(prompt, 3)
    r = generate_speculative(target, target, prompt, 3, 2)
    assert r.tokens == expected
    assert r.accepted == 2
    assert r.rounds == 1


def test_adaptive_scheduler_bookkeeping(models):
    # engine/tests/generation.rs:128-202
    prompt = O.prompt_ids(20, 1000, 2)
    for suffix, (target, draft) in models.items():
        greedy = target.generate(prompt, 15)
        for count in (0, 1, 15):
            r = generate_scheduled(target, draft, prompt, count, DraftSchedule.adaptive_(5, 8))
            assert r.tokens == greedy[: len(prompt) + count]
            assert r.rounds == r.verify.passes == len(r.round_stats)
            assert r.drafted == sum(s[1] for s in r.round_stats)
            assert r.accepted == sum(s[2] for s in r.round_stats)
            assert all(1 <= s[0] <= 8 for s in r.round_stats)
            if count > 0:
                assert r.prefill.passes == 2
                assert r.draft.passes < r.drafted + r.rounds
            if count == 15:
                assert any(s[3] != s[0] for s in r.round_stats)
        r = generate_scheduled(target, target, prompt, 6, DraftSchedule.adaptive_(2, 4))
        assert r.tokens == greedy[: len(prompt) + 6]
        assert r.round_stats[0][3] == 3
        assert r.draft.passes == 4


@pytest.mark.parametrize("p", [0.0, 0.25, 0.5])
def test_oracle_draft_mode_sweeps_acceptance(models, p):
    target, draft = models[""]
    prompt = O.prompt_ids(20, 1000, 2)
    greedy = target.generate(prompt, 24)
    r = generate_speculative(target, draft, prompt, 24, 4, oracle_stream=greedy,
                             oracle_p=p, oracle_seed=7)
    assert r.tokens == greedy
    if p == 0.0:
        assert r.accepted == r.drafted
    else:
        assert 0 < r.accepted < r.drafted


def test_bf16_kv_rounding_changes_little(models):
    target, _ = models[""]
    prompt = O.prompt_ids(20, 1000, 2)
    a, la = target.predict(prompt, target.cache(False), all=True, logits=True)
    b, lb = target.predict(prompt, target.cache(True), all=True, logits=True)
    assert abs(la - lb).max() < 2e-2
