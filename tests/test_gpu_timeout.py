"""The bounded-wait timeout path, on the GPU and without a fault.

Every wait of a pass kernel (a weight, activation or KV page copy, a split-K
reduction) polls an mbarrier a bounded number of times, then sets a bit in
the model's device error flag and returns; the host turns the bit into
JL_ERR_TIMEOUT after the pass.  jl_wait_probe runs that same poll loop on a
barrier nothing completes, with a short bound, so the path is exercised end
to end: no trap, no unbounded loop, and the context stays usable.
"""
import pytest

import jalapeno as J
import oracle as O

pytestmark = pytest.mark.gpu

CFG = O.PRESETS["tiny"]
PROMPT = O.prompt_ids(8, CFG.vocab, 2)


def test_a_wait_nothing_completes_returns_timeout_and_the_model_stays_usable():
    m = J.Model.from_config(CFG, 0, mxfp4=True)
    before = m.predict(PROMPT, m.cache())
    with pytest.raises(J.JlError) as e:
        m.wait_probe(1000)
    assert e.value.status == J.JL_ERR_TIMEOUT
    assert "bounded device wait gave up" in e.value.message
    # the flag is cleared when it is reported: the next pass succeeds
    assert m.predict(PROMPT, m.cache()) == before
    with pytest.raises(J.JlError) as e:
        m.wait_probe(1)
    assert e.value.status == J.JL_ERR_TIMEOUT
    assert m.generate(PROMPT, 4)[: len(PROMPT)] == list(PROMPT)


@pytest.mark.parametrize("polls", [0, (1 << 20) + 1])
def test_wait_probe_bounds(polls):
    m = J.Model.from_config(CFG, 0, mxfp4=True)
    with pytest.raises(J.JlError) as e:
        m.wait_probe(polls)
    assert e.value.status == J.JL_ERR_INVALID_ARG
