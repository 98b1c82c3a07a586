"""Draft steps against the CPU oracle.

A speculative loop's draft passes of one or two rows run kernels of their own
on a model whose layer projections are all MXFP4 (CUDA-core projections,
attention on raw q|k|v): the reference's draft proposals are ordinary
Model::predict calls (engine/src/speculative.rs:84-92, 136-138), so their
logits are held to the same oracle as every other pass, through
jl_predict_draft.  The real-draft loop (no oracle stream) is then compared
with the oracle's restatement of generate_scheduled: tokens, drafted,
accepted, rounds and per-round statistics (engine/tests/generation.rs:52-73).

Tolerances: logits within 2e-2 abs/rel (north star), ids equal, and a
relative L2 below 1e-4 against the oracle with f32 K/V (1e-3 with a bf16
cache: the draft kernels round differently from the oracle, and a last-bit
difference in K or V can move its bf16 rounding by a whole bf16 step).
"""
import numpy as np
import pytest

import jalapeno as J
import oracle as O
from gpu_util import assert_stream_matches, logits_close, rel_l2

pytestmark = pytest.mark.gpu

DEC = O.PRESETS["tiny-dec"]
PROMPT = O.prompt_ids(20, DEC.vocab, 2)
REL = 1e-4
REL_BF16_KV = 1e-3


@pytest.fixture(scope="module")
def dec_oracle():
    return O.Model.synthetic(DEC, 1, mxfp4=True)


def dec_model(seed=1, **kw):
    kw.setdefault("kv_dtype", J.KV_F32)
    return J.Model.from_config(DEC, seed, mxfp4=True, **kw)


def check_step(got, want, what, rel=REL):
    ids, lg = got
    rids, rlg = want
    assert logits_close(lg, rlg), what
    err = rel_l2(lg, rlg)
    assert err < rel, f"{what}: logits relative L2 {err:.3g}"
    assert ids == rids, f"{what}: {ids} != {rids}"


def test_tiny_dec_takes_the_draft_path():
    m = dec_model()
    assert m.has_draft_path
    assert not J.Model.from_config(O.PRESETS["tiny"], 0, mxfp4=True).has_draft_path


@pytest.mark.parametrize("kv", [J.KV_F32, J.KV_BF16])
def test_draft_step_logits_match_oracle(dec_oracle, kv):
    m = dec_model(kv_dtype=kv)
    c, rc = m.cache(), dec_oracle.cache(round_bf16=kv == J.KV_BF16)
    assert m.predict(PROMPT, c) == dec_oracle.predict(PROMPT, rc)
    rel = REL if kv == J.KV_F32 else REL_BF16_KV
    for toks in ([5], [17, 999], [0], [3, 4], [123], [999]):
        check_step(m.predict_draft(toks, c, logits=True), dec_oracle.predict(toks, rc, logits=True),
                   f"draft step {toks}", rel)
    assert c.len == rc.len == len(PROMPT) + 8


def test_draft_step_stream_matches_oracle(dec_oracle):
    """The draft path used as a greedy decoder, one row per step."""
    m = dec_model()
    c = m.cache()
    tokens = list(PROMPT)
    nxt = m.predict(PROMPT, c)[0]
    for _ in range(24):
        tokens.append(nxt)
        if nxt == DEC.eos:
            break
        nxt = m.predict_draft([nxt], c)[0]
    assert_stream_matches(tokens, dec_oracle, PROMPT, len(tokens) - len(PROMPT))


def test_draft_step_rejects_other_row_counts():
    m = dec_model()
    c = m.cache()
    m.predict(PROMPT, c)
    with pytest.raises(J.JlError):
        m.predict_draft([1, 2, 3], c)


@pytest.mark.parametrize("n", [2048, 4096, 9000])
def test_long_context_passes_match_oracle(dec_oracle, n):
    """Past 128 positions every decode, verify and draft-step row splits its
    attention into 128-position windows (one CTA each, partial softmax sums
    merged in window order); past 64 windows (8192 positions) each CTA takes
    several windows.  The prompt is prefilled by multi-chunk passes; then a
    5-row verify pass, one- and two-row draft steps and greedy one-row
    passes on top of the long context."""
    ref = dec_oracle
    m = dec_model()
    prompt = O.prompt_ids(n, DEC.vocab, 5)
    c, rc = m.cache(), ref.cache()
    check_step(m.predict(prompt, c, logits=True), ref.predict(prompt, rc, logits=True), "prefill")
    verify = [7, 77, 777, 1, 2]
    ids, lg = m.predict(verify, c, all=True, logits=True)
    rids, rlg = ref.predict(verify, rc, all=True, logits=True)
    check_step((ids, lg), (rids, rlg), "verify pass")
    c.truncate(n)
    rc.truncate(n)
    check_step(m.predict_draft([7], c, logits=True), ref.predict([7], rc, logits=True), "draft 1 row")
    check_step(m.predict_draft([77, 777], c, logits=True), ref.predict([77, 777], rc, logits=True),
               "draft 2 rows")
    c.truncate(n)
    rc.truncate(n)
    tok = 7
    for i in range(6):
        got = m.predict([tok], c, logits=True)
        want = ref.predict([tok], rc, logits=True)
        check_step(got, want, f"greedy step {i}")
        tok = want[0][0]


@pytest.mark.slow
def test_qwen3_0_6b_draft_steps_match_oracle():
    """The benchmark's draft model at full size: the draft-step kernels
    against the oracle on Qwen3-0.6B MXFP4 (seed 1)."""
    cfg = O.PRESETS["qwen3-0.6b"]
    ref = O.Model.synthetic(cfg, 1, mxfp4=True)
    m = J.Model.from_config(cfg, 1, mxfp4=True, kv_dtype=J.KV_F32, kv_pool_tokens=1024)
    assert m.has_draft_path
    prompt = O.prompt_ids(32, cfg.vocab, 2)
    c, rc = m.cache(), ref.cache()
    ids = m.predict(prompt, c)
    assert ids == ref.predict(prompt, rc)
    tok = ids[0]
    for i in range(6):
        got = m.predict_draft([tok], c, logits=True)
        want = ref.predict([tok], rc, logits=True)
        check_step(got, want, f"draft step {i}")
        tok = want[0][0]
    check_step(m.predict_draft([tok, 11], c, logits=True), ref.predict([tok, 11], rc, logits=True),
               "two-row draft step")


@pytest.mark.parametrize("target_seed", [1, 0])
def test_real_draft_loop_matches_oracle_loop(dec_oracle, target_seed):
    """generate_scheduled with a real draft on the draft-step kernels and no
    oracle stream, against the oracle's loop on the same weights: the target
    of seed 1 has the draft's own weights (nearly every proposal accepted),
    the target of seed 0 unrelated ones (nearly every proposal rejected)."""
    t_ref = dec_oracle if target_seed == 1 else O.Model.synthetic(DEC, 0, mxfp4=True)
    target = dec_model(target_seed)
    draft = dec_model(1)
    for gpu_sched, ref_sched in ((J.DraftSchedule.fixed(4), O.DraftSchedule.fixed(4)),
                                 (J.DraftSchedule.adaptive(2, 8), O.DraftSchedule.adaptive_(2, 8))):
        g = J.generate_scheduled(target, draft, PROMPT, 40, gpu_sched)
        o = O.generate_scheduled(t_ref, dec_oracle, PROMPT, 40, ref_sched)
        assert g.tokens == o.tokens
        assert (g.drafted, g.accepted, g.rounds) == (o.drafted, o.accepted, o.rounds)
        assert g.round_stats == [tuple(s) for s in o.round_stats]
        assert g.draft.passes == o.draft.passes and g.verify.passes == o.verify.passes
        if target_seed == 1:
            assert g.accepted >= 0.9 * g.drafted

