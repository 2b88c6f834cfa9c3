"""Tensor-core batched GEMM (ec_op_gemm_tc) against two references.

1. Bit-exact against a numpy restatement of its own arithmetic: each
   activation row rounded to 21-bit fixed point against its max |x|
   (x' = rint(x * 2080768 / max)), the exact int64 dot with the INT8 rows,
   then float32(float64(dot) * (max / 2080768 * scale)).  This pins the
   tensor-core layout, the digit planes, the stream-K split and the combine.
2. Within tolerance of the reference's op_matmul (the oracle restatement,
   fp32, per row): |y - y_ref| <= 2e-5 * max |y_ref| per row.
"""
import numpy as np
import pytest

from conftest import load_pkg_module

pytestmark = pytest.mark.gpu

FULL = 2080768.0  # 127 * 2^14


@pytest.fixture(scope="module")
def eng():
    return load_pkg_module("engine")


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def emulate(q, s, xs):
    """The GEMM's arithmetic in numpy (exact integers, the same roundings)."""
    out = np.zeros((xs.shape[0], q.shape[0]), np.float32)
    q64 = q.astype(np.int64)
    for b, x in enumerate(xs):
        mx = np.float32(np.abs(x).max())
        if mx == 0:
            continue
        xv = np.rint(x.astype(np.float64) * (FULL / np.float64(mx))).astype(np.int64)
        tot = q64 @ xv
        out[b] = (tot.astype(np.float64) * ((np.float64(mx) / FULL) * s.astype(np.float64))).astype(
            np.float32)
    return out


@pytest.mark.parametrize("m,k,nb", [(1000, 2048, 16), (300, 512, 1), (4096, 4096, 64), (128, 14336, 5),
                                    (2816, 512, 33), (130, 1408, 80), (777, 1024, 100)])
def test_gemm_tc(eng, torch, synth, m, k, nb):
    rng = np.random.default_rng(m + k + nb)
    w = rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.02)
    q, s = synth.quant_int8_rows(w, pow2=False)
    xs = rng.standard_normal((nb, k), dtype=np.float32)
    xs[0, :7] = 0.0
    if nb > 2:
        xs[2] *= np.float32(1e-3)  # rows with very different ranges
    L = eng.lib()
    dq = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    ds = torch.from_numpy(s).cuda()
    dx = torch.from_numpy(xs).cuda()
    wt = torch.zeros(L.ec_gemm_tc_bytes(m, k), dtype=torch.uint8, device="cuda")
    eng.check(L.ec_gemm_tc_pack(dq.data_ptr(), wt.data_ptr(), m, k, None))
    dy = torch.full((nb, m), float("nan"), dtype=torch.float32, device="cuda")
    eng.check(L.ec_op_gemm_tc(wt.data_ptr(), ds.data_ptr(), dx.data_ptr(), dy.data_ptr(), m, k, nb,
                              None))
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    want = emulate(q, s, xs)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), \
        f"max |d| = {np.abs(got - want).max()}"
    exact = (q.astype(np.float64) @ xs.astype(np.float64).T).T * s.astype(np.float64)
    for b in range(nb):
        tol = 2e-5 * np.abs(exact[b]).max()
        assert np.abs(got[b] - exact[b]).max() <= tol, f"row {b}"


def test_gemm_tc_zero_rows_and_errors(eng, torch):
    L = eng.lib()
    m, k, nb = 256, 256, 3
    wt = torch.zeros(L.ec_gemm_tc_bytes(m, k), dtype=torch.uint8, device="cuda")
    s = torch.ones(m, device="cuda")
    x = torch.zeros((nb, k), device="cuda")
    y = torch.full((nb, m), 7.0, device="cuda")
    eng.check(L.ec_op_gemm_tc(wt.data_ptr(), s.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, nb,
                              None))
    torch.cuda.synchronize()
    assert float(y.abs().max()) == 0.0
    assert L.ec_gemm_tc_bytes(m, 100) == 0
    assert L.ec_op_gemm_tc(wt.data_ptr(), s.data_ptr(), x.data_ptr(), y.data_ptr(), m, 100, nb,
                           None) == eng.EC_ERR_ARG


@pytest.mark.parametrize("B,steps", [(16, 72), (85, 6)])
def test_tensor_core_decode_matches_oracle(eng, torch, oracle, synth, B, steps):
    """Steps of at least tensor_min_batch sequences run every projection on the
    tensor cores (85 = a pass of 80 and a pass of 5).  Against each sequence's
    own restatement model: logits within 2e-2 of their range (BASELINE's bar)
    at every step, and the greedy token of every step equal -- the GPU's
    token is fed back to both for 64 steps after an 8-token prompt.  The
    projections differ from the reference by about 1e-6 relative, but the
    INT8 KV cache rounds: a key or value element that lands on a rounding
    boundary moves by one step (1/127 of its row's max), so single logits
    can differ by ~1e-3 of the range."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1408, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=4096, seq_len=512, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=29)
    e = eng.Engine(cfg, max_batch=B, tensor_min_batch=16)
    e.load(model)
    passes = (B + 79) // 80
    assert e.launches_per_step(B) == 1 + 3 * passes + 2 * (2 + 12 * passes) + 1
    pms = [oracle.PortModel(model) for _ in range(B)]
    prompts = [synth.prompt(cfg, 8, seed=60 + b) for b in range(B)]
    toks = [int(p[0]) for p in prompts]
    worst = 0.0
    for t in range(steps):
        lg, am = e.step(toks, [t] * B, want_logits=True)
        for b in range(B):
            want = pms[b].forward(toks[b], t)
            rng_ = float(want.max() - want.min())
            d = float(np.abs(lg[b] - want).max())
            worst = max(worst, d / rng_)
            assert d <= 2e-2 * rng_, f"step {t} sequence {b}: |d| {d} of range {rng_}"
            assert am[b] == oracle.port().port_argmax(want, want.size), f"step {t} sequence {b}"
        toks = [int(prompts[b][t + 1]) if t + 1 < 8 else int(am[b]) for b in range(B)]
    e.close()
    print(f"worst |d| / range = {worst:.2e}")


@pytest.mark.parametrize("mode", ["paged", "linear"])
def test_tensor_core_prefill(eng, torch, oracle, synth, mode):
    """ec_prefill with tensor_min_batch: chunks of >= 16 rows run their
    projections on the tensor cores (the last chunk of 7 rows on the exact
    chain), in both KV modes.  The prompt's last logits within 2e-2 of the
    range of the restatement's, its greedy token equal, and decode steps
    after it still within tolerance with equal greedy tokens."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=4096, seq_len=512, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=37)
    if mode == "paged":
        kw = dict(sparse_blocks_k=4)
    else:
        kw = dict(use_paged_kv=False, sparse_k=32)
    e = eng.Engine(cfg, max_batch=32, tensor_min_batch=16, **kw)
    e.load(model)
    pm = oracle.PortModel(model, **kw)
    P = oracle.port()
    prompt = [int(t) for t in synth.prompt(cfg, 135, seed=12)]
    lg, tok = e.prefill(0, prompt)
    for p, t in enumerate(prompt):
        want = pm.forward(t, p)
    assert np.abs(lg - want).max() <= 2e-2 * (want.max() - want.min())
    assert tok == P.port_argmax(want, want.size)
    for p in range(135, 160):
        lgs, am = e.step([tok], [p])
        want = pm.forward(tok, p)
        assert np.abs(lgs[0] - want).max() <= 2e-2 * (want.max() - want.min()), f"step {p}"
        assert int(am[0]) == P.port_argmax(want, want.size), f"step {p}"
        tok = int(am[0])
    e.close()
