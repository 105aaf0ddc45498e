"""CPU: the sampling restatement (oracle/sampling.py) against the reference's
own sample_next (src/chat.py:46-75), whose candidate ids and final
probabilities tests/golden/make_golden.py captured."""

from __future__ import annotations

from pathlib import Path

import numpy as np

from oracle import sampling as osamp

GOLDEN = Path(__file__).resolve().parent / "golden" / "sampling.npz"


def test_oracle_matches_reference_sample_next():
    z = np.load(GOLDEN)
    n_cases = len([k for k in z.files if k.startswith("args")])
    assert n_cases >= 4
    for ci in range(n_cases):
        temp, top_k, top_p, rep = z[f"args{ci}"]
        logits, seen = z[f"logits{ci}"], z[f"seen{ci}"]
        if temp <= 0:
            assert osamp.sample_token(logits, seen, temp, int(top_k), top_p, rep, 0.5) == int(z[f"token{ci}"][0])
            continue
        idx, p = osamp.sample_probs(logits, seen, temp, int(top_k), top_p, rep)
        np.testing.assert_array_equal(idx, z[f"idx{ci}"])
        np.testing.assert_allclose(p, z[f"probs{ci}"], rtol=0, atol=2e-6)
        # the reference's multinomial draw is one of the tokens with probability > 0
        assert p[list(idx).index(int(z[f"token{ci}"][0]))] > 0


def test_inverse_cdf_pick():
    logits = np.zeros(10, np.float16)
    logits[[3, 7, 1]] = [2.0, 1.0, 0.5]
    idx, p = osamp.sample_probs(logits, None, 1.0, 3, 1.0, 1.0)
    assert list(idx) == [3, 7, 1]
    c = np.cumsum(p)
    assert osamp.sample_token(logits, None, 1.0, 3, 1.0, 1.0, 0.0) == 3
    assert osamp.sample_token(logits, None, 1.0, 3, 1.0, 1.0, float(c[0]) + 1e-4) == 7
    assert osamp.sample_token(logits, None, 1.0, 3, 1.0, 1.0, 0.99999) == 1
    assert osamp.sample_token(logits, None, 0.0, 3, 1.0, 1.0, 0.3) == 3
