"""Device sampling (ec_op_sample_top_p / ec_op_sample_temperature, through
the C ABI) against the reference's own sample_top_p (golden vectors from
tests/golden/make_sample_golden.py) and the C restatement
(oracle/port/sample.c).

Bit-exact: the repetition-penalised logits, and the token wherever the draw
and top_p are not within float rounding (1e-5) of a running-sum boundary.
The device sums probabilities in exact fixed point, the reference in float,
so a draw within rounding of a boundary may legitimately pick the
neighbouring token; those few cases are counted, not compared.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from conftest import load_pkg_module  # noqa: E402
from make_sample_golden import PENALTY, SHAPES, PER_SHAPE, cases  # noqa: E402

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "sample_vectors.npz"))


@pytest.fixture(scope="module")
def eng():
    return load_pkg_module("engine")


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _probs32(lg, temp):
    """The reference's softmax in float32 (compute_softmax,
    sampler_topp.c:82-108): the sum accumulated in index order."""
    lg = np.asarray(lg, np.float32)
    e = np.exp((lg - lg.max()) / np.float32(temp)).astype(np.float32)
    total = np.cumsum(e, dtype=np.float32)[-1]
    return (e / total).astype(np.float32)


TOL = 2e-4  # probability mass: above the reference's own float32 drift


def top_p_check(lg, temp, top_p, r, tok, ref_tok=None):
    """Asserts that `tok` is the token the reference's top-p step picks for
    draw r, up to float rounding: in the descending order of the
    probabilities (ties by index) with exact running sums cs, tok lies in
    the nucleus and its interval [cs_before, cs_after] contains r times the
    nucleus' mass, each within TOL.  The reference's float32 running sums
    drift from exact ones by up to 1.2e-4 over the golden cases.  Where the
    draw is farther than TOL from both ends of an interval and top_p farther
    than TOL from every running sum, the token must equal ref_tok exactly.
    Returns True when the exact comparison was made."""
    p = _probs32(lg, temp)
    order = np.lexsort((np.arange(p.size), -p))
    cs = np.cumsum(p[order].astype(np.float64))
    above = np.nonzero(cs > float(top_p))[0]
    cut = int(above[0]) + 1 if above.size else cs.size
    target = float(r) * cs[cut - 1]
    q = int(np.nonzero(order == tok)[0][0])
    lo = cs[q - 1] if q else 0.0
    assert q == 0 or lo <= float(top_p) + TOL, ("outside the nucleus", q, cut)
    assert lo - TOL <= target <= cs[q] + TOL, ("draw outside the token's interval", q)
    je = min(int(np.searchsorted(cs[:cut], target, side="right")), cut - 1)
    lo_e = cs[je - 1] if je else 0.0
    clear = (target - lo_e > TOL and cs[je] - target > TOL
             and np.abs(cs - float(top_p)).min() > TOL)
    if clear and ref_tok is not None:
        assert tok == ref_tok, (tok, ref_tok)
    return clear


def penalise(lg, hist):
    lg = lg.copy()
    for t in hist:
        lg[t] = lg[t] / PENALTY if lg[t] > 0 else lg[t] * PENALTY
    lg[0] = np.float32(-1e9)
    return lg


def run_top_p(eng, torch, rows, hists, temp, top_p, r, penalty=PENALTY, block0=1):
    L = eng.lib()
    lg = torch.from_numpy(np.stack(rows)).cuda()
    n = lg.shape[1]
    hl = np.array([h.size for h in hists], np.int32)
    stride = max(1, int(hl.max()) if hl.size else 1)
    hb = np.zeros((len(rows), stride), np.int32)
    for k, h in enumerate(hists):
        hb[k, :h.size] = h
    hd = torch.from_numpy(hb).cuda()
    hld = torch.from_numpy(hl).cuda()
    rd = torch.from_numpy(np.asarray(r, np.float32)).cuda()
    out = torch.full((len(rows),), -7, dtype=torch.int32, device="cuda")
    eng.check(L.ec_op_sample_top_p(lg.data_ptr(), n, len(rows), hd.data_ptr(), hld.data_ptr(),
                                   stride, float(temp), float(top_p), float(penalty), block0,
                                   rd.data_ptr(), out.data_ptr(), None))
    torch.cuda.synchronize()
    return out.cpu().numpy(), lg.cpu().numpy()


def test_top_p_matches_reference_vectors(eng, torch):
    cs = cases()
    exact = 0
    for s_, (n, _, temp, top_p) in enumerate(SHAPES):
        ks = range(s_ * PER_SHAPE, (s_ + 1) * PER_SHAPE)
        rows = [cs[k][0] for k in ks]
        hists = [cs[k][1] for k in ks]
        toks, got_lg = run_top_p(eng, torch, rows, hists, temp, top_p, G["draw"][list(ks)])
        for j, k in enumerate(ks):
            want_lg = penalise(rows[j], hists[j])
            assert np.array_equal(got_lg[j].view(np.uint32), want_lg.view(np.uint32)), k
            # the reference's own token passes the same check
            top_p_check(want_lg, temp, top_p, G["draw"][k], int(G["token"][k]))
            exact += top_p_check(want_lg, temp, top_p, G["draw"][k], int(toks[j]),
                                 int(G["token"][k]))
    assert exact >= 20  # 24 of the 48 golden draws are clear of rounding


def test_top_p_matches_restatement_many_draws(eng, torch, oracle):
    """One logits row, 256 draws spread over [0, 1]: every token within
    tolerance of the restatement's, equal to it where rounding cannot
    matter."""
    P = oracle.port()
    rng = np.random.default_rng(11)
    lg = (3.0 * rng.standard_normal(32000)).astype(np.float32)
    draws = np.linspace(0, 1, 256, dtype=np.float32)
    toks, _ = run_top_p(eng, torch, [lg] * 256, [np.zeros(0, np.int32)] * 256,
                        0.7, 0.9, draws, block0=0)
    z = np.zeros(1, np.int32)
    exact = 0
    for j, r in enumerate(draws):
        want = P.port_sample_top_p(lg.copy(), lg.size, z, 0, np.float32(0.7), np.float32(0.9),
                                   np.float32(1), 0, r, np.zeros(1, np.int32),
                                   np.zeros(1, np.float32))
        exact += top_p_check(lg, 0.7, 0.9, r, int(toks[j]), want)
    assert exact >= 200


def test_top_p_edges(eng, torch, oracle):
    P = oracle.port()
    z = np.zeros(1, np.int32)

    def port(lg, temp, top_p, r, block0=0):
        return P.port_sample_top_p(lg.copy(), lg.size, z, 0, np.float32(temp),
                                   np.float32(top_p), np.float32(1), block0, np.float32(r),
                                   np.zeros(1, np.int32), np.zeros(1, np.float32))
    # one token
    t, _ = run_top_p(eng, torch, [np.array([0.3], np.float32)], [np.zeros(0, np.int32)],
                     0.7, 0.9, [0.5], block0=0)
    assert t[0] == 0
    # all equal: the nucleus is the first ceil(top_p * n) ids (ties by index)
    n = 1000
    eq = np.zeros(n, np.float32)
    draws = np.array([0.0, 0.2511, 0.5013, 0.9005], np.float32)
    t, _ = run_top_p(eng, torch, [eq] * 4, [np.zeros(0, np.int32)] * 4, 1.0, 0.5005, draws,
                     block0=0)
    for j, r in enumerate(draws):
        assert t[j] == port(eq, 1.0, 0.5005, r), (r, t[j])
    # a tiny top_p keeps only the most probable token
    rng = np.random.default_rng(3)
    lg = rng.standard_normal(5000).astype(np.float32)
    t, _ = run_top_p(eng, torch, [lg] * 3, [np.zeros(0, np.int32)] * 3, 0.7, 1e-6,
                     [0.0, 0.5, 1.0], block0=0)
    assert set(t.tolist()) == {int(np.argmax(lg))}
    # top_p = 1: the whole vocabulary; draw 0 is the most probable token
    t, _ = run_top_p(eng, torch, [lg], [np.zeros(0, np.int32)], 0.7, 1.0, [0.0], block0=0)
    assert t[0] == int(np.argmax(lg))
    # a long history with repeats: the penalty applied once per occurrence
    lg = (2.0 * rng.standard_normal(128256)).astype(np.float32)
    hist = rng.integers(0, 50, size=3000).astype(np.int32)
    t, got = run_top_p(eng, torch, [lg], [hist], 0.7, 0.9, [0.3])
    assert np.array_equal(got[0].view(np.uint32), penalise(lg, hist).view(np.uint32))


def test_temperature_matches_restatement(eng, torch, oracle):
    P = oracle.port()
    L = eng.lib()
    rng = np.random.default_rng(9)
    n, rows = 32000, 128
    lg = (2.0 * rng.standard_normal((rows, n))).astype(np.float32)
    r = rng.uniform(0, 1, rows).astype(np.float32)
    r[:3] = [0.0, 0.999999, 1.0]
    lgd = torch.from_numpy(lg).cuda()
    rd = torch.from_numpy(r).cuda()
    out = torch.zeros(rows, dtype=torch.int32, device="cuda")
    eng.check(L.ec_op_sample_temperature(lgd.data_ptr(), n, rows, 0.8, rd.data_ptr(),
                                         out.data_ptr(), None))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    exact = 0
    for k in range(rows):
        p = _probs32(lg[k], 0.8)
        c = np.cumsum(p.astype(np.float64))
        q = int(got[k])
        lo = c[q - 1] if q else 0.0
        if r[k] >= c[-1]:
            assert q == n - 1
            continue
        assert lo - TOL <= float(r[k]) <= c[q] + TOL, k
        je = int(np.searchsorted(c, float(r[k]), side="right"))
        if float(r[k]) - (c[je - 1] if je else 0.0) > TOL and c[je] - float(r[k]) > TOL:
            assert q == P.port_sample_temperature(lg[k], n, np.float32(0.8), r[k]), k
            exact += 1
    assert exact >= 48  # 59 of the 128 draws are clear of rounding
    assert 0 <= got.min() and got.max() < n


def test_engine_sample_device(eng, torch, oracle, tiny_model):
    """After each decode step, the server's sampling on the context's own
    device logits (the history so far penalised): the same token as the
    restatement on the logits the step returned."""
    P = oracle.port()
    e = eng.Engine(tiny_model.cfg, use_paged_kv=True, sparse_k=64)
    e.load(tiny_model)
    hist = np.array([5, 9, 9, 17, 300, 41, 9, 77], np.int32)
    hd = torch.from_numpy(hist).cuda()
    draws = np.linspace(0.05, 0.95, hist.size, dtype=np.float32)
    for pos, t in enumerate(hist):
        lg, _ = e.step([int(t)], [pos])
        hl = torch.tensor([pos + 1], dtype=torch.int32, device="cuda")
        rd = torch.tensor([draws[pos]], dtype=torch.float32, device="cuda")
        out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        e.sample_device(1, rd.data_ptr(), out.data_ptr(), hd.data_ptr(), hl.data_ptr(),
                        hist.size)
        e.sync()
        row = lg[0]
        want = P.port_sample_top_p(row.copy(), row.size, np.ascontiguousarray(hist[:pos + 1]),
                                   pos + 1, np.float32(0.7), np.float32(0.9), PENALTY, 1,
                                   draws[pos], np.zeros(1, np.int32), np.zeros(1, np.float32))
        top_p_check(penalise(row, hist[:pos + 1]), 0.7, 0.9, draws[pos],
                    int(out.item()), want)
    e.close()
