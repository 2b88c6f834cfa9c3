"""The sampling restatement (oracle/port/sample.c) pinned to the reference's
own sample_top_p (src/compute/sampler_topp.c:113) through the committed
vectors of tests/golden/make_sample_golden.py, and directly against
oracle/_ref where it is built.  No GPU."""
import os
import sys

import numpy as np

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_sample_golden import PENALTY, cases  # noqa: E402

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "sample_vectors.npz"))


def port_top_p(P, lg, hist, temp, top_p, r):
    lg = lg.copy()
    cut = np.zeros(1, np.int32)
    cum = np.zeros(1, np.float32)
    h = np.ascontiguousarray(hist, np.int32)
    tok = P.port_sample_top_p(lg, lg.size, h, h.size, temp, top_p, PENALTY, 1, np.float32(r),
                              cut, cum)
    return tok, lg


def test_cases_regenerate():
    cs = cases()
    assert len(cs) == G["token"].size
    for (lg, *_), head in zip(cs, G["logits_head"]):
        assert int.from_bytes(lg[:64].tobytes()[:8], "little") == int(head)


def test_port_top_p_matches_reference_vectors(oracle):
    P = oracle.port()
    for k, (lg, hist, temp, top_p, _) in enumerate(cases()):
        tok, _ = port_top_p(P, lg, hist, temp, top_p, G["draw"][k])
        assert tok == int(G["token"][k]), k


def test_port_top_p_matches_reference_live(ref):
    """Fresh seeds straight through the reference's sampler."""
    P, R = ref.port(), ref.ref()
    rng = np.random.default_rng(5)
    for k in range(40):
        n = int(rng.choice([50, 1000, 32000]))
        lg = (float(rng.uniform(0.5, 8)) * rng.standard_normal(n)).astype(np.float32)
        lg[0] = np.float32(-1e9)
        temp = np.float32(rng.uniform(0.2, 1.5))
        top_p = np.float32(rng.choice([0.5, 0.9, 0.95, 1.0]))
        seed = int(rng.integers(1, 2**31 - 1))
        want = R.refd_sample_top_p(lg, n, temp, top_p, seed)
        r = R.refd_first_rand(seed)
        got = P.port_sample_top_p(lg.copy(), n, np.zeros(1, np.int32), 0, temp, top_p,
                                  np.float32(1), 0, np.float32(r), np.zeros(1, np.int32),
                                  np.zeros(1, np.float32))
        assert got == want, k


def test_port_temperature_cdf(oracle):
    """sample_from_probs: the first index whose running sum exceeds r."""
    P = oracle.port()
    lg = np.array([0.0, 1.0, -2.0, 3.0, 0.5], np.float32)
    p = np.exp((lg - lg.max()) / 0.7)
    c = np.cumsum(p / p.sum())
    for r in np.linspace(0.0, 0.999, 57, dtype=np.float32):
        want = int(np.searchsorted(c, r, side="right"))
        if np.min(np.abs(c - r)) < 1e-5:
            continue
        assert P.port_sample_temperature(lg, lg.size, np.float32(0.7), r) == want
