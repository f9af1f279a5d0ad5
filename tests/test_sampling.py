"""The host sampler (GSDLQModel.sample_token: greedy, temperature + top-p) against picks made by the
reference's own sample_token (gsd_lq_cpu_runtime.py:422-443) on the same logits under the same
np.random seeds (tests/golden/sampling_ref.npz, written by make_golden.py).  No GPU needed: the method
reads only its arguments and NumPy's global generator."""
import os

import numpy as np

from conftest import GOLDEN


def _sample(logits, t, p):
    from gsdlq_b200.model import GSDLQModel
    return GSDLQModel.sample_token(None, logits, temperature=t, top_p=p)


def test_sampling_matches_reference_picks():
    g = np.load(os.path.join(GOLDEN, "sampling_ref.npz"))
    logits, cases, seeds, picks = g["logits"], g["cases"], g["seeds"], g["picks"]
    state = np.random.get_state()
    try:
        for i, lg in enumerate(logits):
            for j, (t, p) in enumerate(cases):
                for k, seed in enumerate(seeds):
                    np.random.seed(int(seed))
                    got = _sample(lg.copy(), float(t), float(p))
                    assert got == picks[i, j, k], (i, (t, p), int(seed), got, picks[i, j, k])
    finally:
        np.random.set_state(state)


def test_sampling_edge_rules():
    # greedy: NaN is never picked, +inf counts as 100 and wins, the first of tied maxima wins
    z = np.zeros(16, np.float32)
    z[3], z[9] = np.nan, np.inf
    assert _sample(z, 0.0, 0.9) == 9
    z = np.zeros(16, np.float32)
    z[[4, 11]] = 2.0
    assert _sample(z, 0.0, 0.9) == 4
    # a single-token nucleus: with top_p below the top probability only the top token can be drawn
    z = np.zeros(16, np.float32)
    z[6] = 5.0
    for seed in range(4):
        np.random.seed(seed)
        assert _sample(z, 1.0, 0.5) == 6
    # the logits passed in are not modified
    z = np.linspace(-1, 1, 32).astype(np.float32)
    before = z.copy()
    _sample(z, 0.8, 0.9)
    np.testing.assert_array_equal(z, before)
