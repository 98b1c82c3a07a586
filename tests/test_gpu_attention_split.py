"""Decode attention over long contexts: a row's result does not depend on
the pass that computes it.

A row whose context spans several windows of 128 positions gets one CTA per
window (several consecutive windows per CTA past 64 windows), and the last
CTA to finish merges the windows' partial softmax sums in window order; the
split depends only on the row's position.  So a row computed inside a 5-row
verify pass must equal, bit for bit, the same row computed alone, at
contexts of 3, 33 and 71 windows, and both must match the oracle."""
import numpy as np
import pytest

import jalapeno as J
import oracle as O
from gpu_util import logits_close, rel_l2

pytestmark = pytest.mark.gpu

DEC = O.PRESETS["tiny-dec"]
ROWS = [7, 77, 777, 1, 2]


@pytest.fixture(scope="module")
def dec_oracle():
    return O.Model.synthetic(DEC, 1, mxfp4=True)


@pytest.mark.parametrize("n", [300, 4096, 9000])
def test_rows_equal_alone_and_in_a_verify_pass(dec_oracle, n):
    m = J.Model.from_config(DEC, 1, mxfp4=True, kv_dtype=J.KV_F32)
    prompt = O.prompt_ids(n, DEC.vocab, 5)
    c = m.cache()
    m.predict(prompt, c)
    ids5, lg5 = m.predict(ROWS, c, all=True, logits=True)
    c.truncate(n)
    for i, t in enumerate(ROWS):
        ids1, lg1 = m.predict([t], c, logits=True)
        assert ids1[0] == ids5[i], f"row {i}"
        assert np.array_equal(lg1[0], lg5[i]), f"row {i}: logits differ between a 1-row and a 5-row pass"
    # and the verify pass matches the oracle
    rc = dec_oracle.cache()
    dec_oracle.predict(prompt, rc)
    rids, rlg = dec_oracle.predict(ROWS, rc, all=True, logits=True)
    assert ids5 == rids
    assert logits_close(lg5, rlg) and rel_l2(lg5, rlg) < 1e-4
