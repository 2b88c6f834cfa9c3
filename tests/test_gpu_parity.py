"""GPU parity: the CUDA library (through its C ABI) against the oracle.

Bit-exact: GEMV (INT8 / FP8 / BF16), RMSNorm, RoPE, SwiGLU, INT8 quantisation,
argmax, and the whole decode step of the tiny model (every step's logits and
the greedy tokens) in both KV modes, checked against digests produced by the
reference engine itself (tests/golden) and against the C restatement.
Beyond SPARSE_BLOCKS_K blocks the block-sparse path is checked the same way,
including the order of the selected blocks (the reference's min-heap array
order), which matters: its online softmax uses an approximate exp, so the
result depends on the order tokens are visited in.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from conftest import load_pkg_module  # noqa: E402
from make_golden import digest  # noqa: E402

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_vectors.npz"))


@pytest.fixture(scope="module")
def eng():
    return load_pkg_module("engine")


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def bits(a):
    return np.asarray(a).view(np.uint32)


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("kind", ["int8", "fp8", "bf16"])
@pytest.mark.parametrize("m,k", [(37, 64), (300, 512), (4096, 4096), (1000, 14336),
                                 (2816, 1408)])
def test_gemv(eng, torch, synth, oracle, kind, m, k):
    rng = np.random.default_rng(m * 7 + k)
    w = rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.02)
    x = rng.standard_normal(k, dtype=np.float32)
    y = np.zeros(m, np.float32)
    P = oracle.port()
    if kind == "int8":
        q, s = synth.quant_int8_rows(w, pow2=False)
        P.port_gemv_q8(y, q, s, x, m, k)
        wk, scale = eng.EC_W_INT8, s
    elif kind == "fp8":
        q, s = synth.quant_fp8_tensor(w)
        P.port_gemv_fp8(y, q, np.float32(s[0]), x, m, k)
        wk, scale = eng.EC_W_FP8, s
    else:
        q, scale = synth.f32_to_bf16(w), None
        P.port_gemv_bf16(y, q, x, m, k)
        wk = eng.EC_W_BF16
    dq, dx = dev(torch, q), dev(torch, x)
    ds = dev(torch, scale) if scale is not None else None
    dy = torch.zeros(m, dtype=torch.float32, device="cuda")
    eng.check(eng.lib().ec_op_gemv(wk, dq.data_ptr(), ds.data_ptr() if ds is not None else None,
                                   dx.data_ptr(), dy.data_ptr(), m, k, None))
    torch.cuda.synchronize()
    assert np.array_equal(bits(dy.cpu().numpy()), bits(y))


@pytest.mark.parametrize("rows_per_thread", ["0", "1", "2"])
@pytest.mark.parametrize("kind", ["int8", "fp8"])
@pytest.mark.parametrize("m,k", [(37, 64), (6, 1024), (300, 512), (4096, 4096), (1000, 14336),
                                 (2816, 1408), (130, 4096), (6144, 4096)])
def test_gemv_packed(eng, torch, synth, oracle, monkeypatch, rows_per_thread, kind, m, k):
    """The decode step's GEMV (packed weight layout, chunks of 512 or 32
    columns, 1 or 2 rows per thread, ragged last row quad) == the
    restatement of op_matmul, bit for bit."""
    monkeypatch.setenv("EC_GEMV_ROWS_PER_THREAD", rows_per_thread)
    rng = np.random.default_rng(m * 11 + k)
    w = rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.02)
    x = rng.standard_normal(k, dtype=np.float32)
    y = np.zeros(m, np.float32)
    P = oracle.port()
    if kind == "int8":
        q, s = synth.quant_int8_rows(w, pow2=False)
        P.port_gemv_q8(y, q, s, x, m, k)
        wk = eng.EC_W_INT8
    else:
        q, s = synth.quant_fp8_tensor(w)
        P.port_gemv_fp8(y, q, np.float32(s[0]), x, m, k)
        wk = eng.EC_W_FP8
    L = eng.lib()
    dq, dx, ds = dev(torch, q), dev(torch, x), dev(torch, s)
    packed = torch.full((L.ec_gemv_packed_bytes(m, k),), 7, dtype=torch.uint8, device="cuda")
    eng.check(L.ec_gemv_pack(dq.data_ptr(), packed.data_ptr(), m, k, None))
    dy = torch.full((m,), float("nan"), dtype=torch.float32, device="cuda")
    eng.check(L.ec_op_gemv_packed(wk, packed.data_ptr(), ds.data_ptr(), dx.data_ptr(),
                                  dy.data_ptr(), m, k, None))
    torch.cuda.synchronize()
    assert np.array_equal(bits(dy.cpu().numpy()), bits(y))


@pytest.mark.parametrize("nb", [1, 3, 8, 11])
def test_gemv_packed_batch(eng, torch, synth, oracle, nb):
    """nb activation vectors through one weight pass: each result bit-identical
    to the restatement of op_matmul on that vector."""
    m, k = 1000, 2048
    rng = np.random.default_rng(nb)
    w = rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.02)
    xs = rng.standard_normal((nb, k), dtype=np.float32)
    q, s = synth.quant_int8_rows(w, pow2=False)
    P = oracle.port()
    L = eng.lib()
    dq, ds, dx = dev(torch, q), dev(torch, s), dev(torch, xs)
    packed = torch.empty(L.ec_gemv_packed_bytes(m, k), dtype=torch.uint8, device="cuda")
    eng.check(L.ec_gemv_pack(dq.data_ptr(), packed.data_ptr(), m, k, None))
    dy = torch.full((nb, m), float("nan"), dtype=torch.float32, device="cuda")
    eng.check(L.ec_op_gemv_packed_batch(eng.EC_W_INT8, packed.data_ptr(), ds.data_ptr(),
                                        dx.data_ptr(), dy.data_ptr(), m, k, nb, None))
    torch.cuda.synchronize()
    got = dy.cpu().numpy()
    for b in range(nb):
        y = np.zeros(m, np.float32)
        P.port_gemv_q8(y, q, s, np.ascontiguousarray(xs[b]), m, k)
        assert np.array_equal(bits(got[b]), bits(y)), f"vector {b}"


def test_small_ops(eng, torch):
    L = eng.lib()
    # RMSNorm
    x, w, want = G["norm_x"], G["norm_w"], G["norm_y"]
    dx, dw = dev(torch, x), dev(torch, w)
    out = torch.zeros_like(dx)
    eng.check(L.ec_op_rmsnorm(out.data_ptr(), dx.data_ptr(), dw.data_ptr(), x.size,
                              np.float32(1e-5), None))
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))
    # RoPE
    q = dev(torch, G["rope_in"])
    ct, st = dev(torch, G["rope_cos"]), dev(torch, G["rope_sin"])  # keep alive
    eng.check(L.ec_op_rope(q.data_ptr(), 8, 128, 311, ct.data_ptr(), st.data_ptr(), 512, None))
    torch.cuda.synchronize()
    assert np.array_equal(bits(q.cpu().numpy()), bits(G["rope_out"]))
    # SwiGLU
    g, u = dev(torch, G["silu_g"]), dev(torch, G["silu_u"])
    o = torch.zeros_like(g)
    eng.check(L.ec_op_silu_mul(o.data_ptr(), g.data_ptr(), u.data_ptr(), g.numel(), None))
    torch.cuda.synchronize()
    assert np.array_equal(bits(o.cpu().numpy()), bits(G["silu_y"]))
    # INT8 quantisation
    vin = dev(torch, G["quant_in"])
    qo = torch.zeros(vin.shape, dtype=torch.int8, device="cuda")
    so = torch.zeros(vin.shape[0], dtype=torch.float32, device="cuda")
    eng.check(L.ec_op_quant_int8(qo.data_ptr(), so.data_ptr(), vin.data_ptr(), vin.shape[0],
                                 vin.shape[1], None))
    torch.cuda.synchronize()
    assert np.array_equal(qo.cpu().numpy(), G["quant_q"])
    assert np.array_equal(bits(so.cpu().numpy()), bits(G["quant_s"]))
    # argmax (with ties)
    lg = dev(torch, G["argmax_in"])
    am = torch.zeros(1, dtype=torch.int32, device="cuda")
    eng.check(L.ec_op_argmax(lg.data_ptr(), lg.numel(), 1, am.data_ptr(), None))
    torch.cuda.synchronize()
    assert int(am.item()) == int(G["argmax_out"])


@pytest.mark.parametrize("mode", ["paged", "linear"])
def test_tiny_decode_matches_reference(eng, torch, tiny_model, mode):
    """64-token prompt + 128 greedy steps of the tiny model: every step's
    logits bit-identical to the reference engine's (digests from
    tests/golden), same greedy tokens, same LSH counters."""
    paged = mode == "paged"
    e = eng.Engine(tiny_model.cfg, use_paged_kv=paged, sparse_k=64 if paged else 32)
    e.load(tiny_model)
    toks = G[f"tiny_{mode}_tokens"]
    dg = G[f"tiny_{mode}_digests"]
    for pos in range(dg.size):
        lg, am = e.step([toks[pos]], [pos])
        assert digest(lg[0]) == dg[pos], f"step {pos}"
        if pos >= 63:
            assert am[0] == toks[pos + 1], f"greedy token at step {pos}"
    assert np.array_equal(np.array(e.counters()), G[f"tiny_{mode}_counters"])
    e.close()


def test_tiny_lsh_index_matches_oracle(eng, torch, oracle, tiny_model):
    """Layer-0 LSH index after 192 tokens: unit hashes, bucket heads, chains."""
    e = eng.Engine(tiny_model.cfg, use_paged_kv=False, sparse_k=32)
    e.load(tiny_model)
    pm = oracle.PortModel(tiny_model, use_paged_kv=False, sparse_k=32)
    toks = G["tiny_linear_tokens"]
    for pos in range(192):
        e.step([toks[pos]], [pos], want_logits=False)
        pm.forward(int(toks[pos]), pos)
    got = e.lsh()
    L = pm.lsh()
    n = L.n_units
    assert got["n_units"] == n == 3
    assert np.array_equal(got["unit_hash"][0, :n], np.ctypeslib.as_array(L.unit_hash, (n,)))
    assert np.array_equal(got["heads"][0], np.ctypeslib.as_array(L.heads, (65536,)))
    assert np.array_equal(got["next"][0, :n], np.ctypeslib.as_array(L.next, (n,)))
    e.close()


def test_tiny_lsh_4x8(eng, torch, oracle, tiny_model):
    """LSH with 4 tables x 8 bits, top-K 32, unit 64: the
    CUDA path against the restatement, every step bit-exact."""
    lsh = dict(lsh_tables=4, lsh_bits=8)
    e = eng.Engine(tiny_model.cfg, use_paged_kv=False, sparse_k=32, **lsh)
    e.load(tiny_model)
    pm = oracle.PortModel(tiny_model, use_paged_kv=False, sparse_k=32, **lsh)
    toks = list(np.load(os.path.join(os.path.dirname(__file__), "golden",
                                     "ref_vectors.npz"))["tiny_linear_tokens"][:64])
    for pos in range(64 + 128):
        lg, am = e.step([toks[pos]], [pos])
        want = pm.forward(int(toks[pos]), pos)
        assert np.array_equal(bits(lg[0]), bits(want)), f"step {pos}"
        if pos >= 63:
            toks.append(int(am[0]))
    assert e.counters() == pm.counters()
    e.close()


@pytest.mark.parametrize("sparse_k,steps", [(37, 200), (511, 640)])
def test_linear_topk_not_multiple_of_4(eng, torch, oracle, tiny_model, sparse_k, steps):
    """Linear-mode top-K sizes that are not a multiple of 4 (BASELINE config
    5 attends 511-512 tokens): the attention's per-token arrays are padded;
    every checked step bit-exact against the restatement."""
    e = eng.Engine(tiny_model.cfg, use_paged_kv=False, sparse_k=sparse_k)
    e.load(tiny_model)
    pm = oracle.PortModel(tiny_model, use_paged_kv=False, sparse_k=sparse_k)
    toks = list(G["tiny_linear_tokens"][:64])
    for pos in range(steps):
        check = pos % 40 == 0 or pos >= steps - 8
        lg, am = e.step([toks[pos]], [pos], want_logits=True)
        want = pm.forward(int(toks[pos]), pos)
        if check:
            assert np.array_equal(bits(lg[0]), bits(want)), f"step {pos}"
        if pos >= 63:
            toks.append(int(am[0]))
    e.close()


def test_paged_block_sparse(eng, torch, oracle, synth):
    """Context beyond SPARSE_BLOCKS_K * 16 = 1024 tokens: block-centroid
    scoring, first + last + min-heap top-62 selection in the reference's heap
    array order, sparse attention: every step bit-exact, and the selected
    blocks of the last layer identical (same order) to the restatement's."""
    import ctypes as C
    cfg = synth.ModelConfig(dim=256, hidden_dim=512, n_layers=2, n_heads=4, n_kv_heads=2,
                            vocab_size=2048, seq_len=2048, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=11)
    e = eng.Engine(cfg)
    e.load(model)
    pm = oracle.PortModel(model)
    P = oracle.port()
    toks = synth.prompt(cfg, 1200, seed=4)
    for pos in range(1200):
        lg, _ = e.step([toks[pos]], [pos], want_logits=pos >= 1000)
        want = pm.forward(int(toks[pos]), pos)
        if pos < 1000:
            continue
        assert np.array_equal(bits(lg[0]), bits(want)), f"step {pos}"
        if pos < 1024:
            continue
        pp = pm.paged(cfg.n_layers - 1)
        nb = pp.n_blocks
        q = np.ctypeslib.as_array(P.port_model_state(pm.h, 2), (cfg.n_heads * cfg.head_dim,))
        sc = np.zeros(nb, np.float32)
        P.port_paged_scores(C.byref(pp), np.ascontiguousarray(q), sc)
        sel = np.zeros(70, np.int32)
        ns = P.port_select_blocks(sc, nb, 64, sel)
        got = e.state(8, n=80)
        gn = int(got[0])
        assert gn == ns and np.array_equal(got[1:1 + gn].astype(np.int32), sel[:ns])
    e.close()


def test_host_transformer_api(eng, torch, tiny_model):
    """ec_transformer_forward (the reference-facing API) == golden digests."""
    t = eng.HostTransformer(tiny_model.cfg)
    t.load(tiny_model)
    toks = G["tiny_paged_tokens"]
    dg = G["tiny_paged_digests"]
    for pos in range(80):
        lg = t.forward(toks[pos], pos)
        assert digest(lg) == dg[pos]
    t.close()


def paged_view(eng, torch, kv_heads, hd, max_blocks, seed=5):
    """A paged cache in torch-allocated device memory whose page table is a
    seeded permutation (logical block b lives in physical block perm[b])."""
    perm = np.random.default_rng(seed).permutation(max_blocks).astype(np.int32)
    bufs = dict(
        k=torch.zeros(max_blocks * kv_heads * 16 * hd, dtype=torch.int8, device="cuda"),
        v=torch.zeros(max_blocks * kv_heads * 16 * hd, dtype=torch.int8, device="cuda"),
        ks=torch.zeros(max_blocks * kv_heads * 16, dtype=torch.float32, device="cuda"),
        vs=torch.zeros(max_blocks * kv_heads * 16, dtype=torch.float32, device="cuda"),
        c=torch.zeros(max_blocks * hd, dtype=torch.float32, device="cuda"),
        pt=dev(torch, perm))
    pv = eng.PagedView(bufs["k"].data_ptr(), bufs["v"].data_ptr(), bufs["ks"].data_ptr(),
                       bufs["vs"].data_ptr(), bufs["c"].data_ptr(), bufs["pt"].data_ptr(),
                       kv_heads, hd, max_blocks)
    return pv, bufs


def golden_paged_view(eng, torch):
    """The golden paged cache (KV=2, hd=64, 1100 tokens of seed 31) filled
    through ec_op_paged_append."""
    import ctypes as C
    from make_golden import paged_inputs
    KV, hd, T = 2, 64, 1100
    pv, bufs = paged_view(eng, torch, KV, hd, 128)
    kk, vv = paged_inputs(T, KV * hd)
    dk, dv = dev(torch, kk), dev(torch, vv)
    L = eng.lib()
    for p in range(T):
        eng.check(L.ec_op_paged_append(C.byref(pv), dk[p].data_ptr(), dv[p].data_ptr(), p, None))
    bufs["kk"], bufs["vv"] = dk, dv
    return pv, bufs


def test_paged_ops_match_reference(eng, torch):
    """ec_op_paged_append + ec_op_paged_attention on a permuted page table:
    dense (op_paged_attention) and block-sparse (score, heap top-K, sparse
    attention) outputs and the selected logical blocks, bit-identical to the
    reference engine's (tests/golden)."""
    import ctypes as C
    H, hd, T = 8, 64, 1100
    pv, bufs = golden_paged_view(eng, torch)
    L = eng.lib()
    q = dev(torch, G["paged_q"])
    out = torch.zeros(H * hd, dtype=torch.float32, device="cuda")
    sel = torch.full((80,), -7, dtype=torch.int32, device="cuda")
    ns = torch.zeros(1, dtype=torch.int32, device="cuda")
    eng.check(L.ec_op_paged_attention(C.byref(pv), q.data_ptr(), out.data_ptr(), H, T, 0,
                                      sel.data_ptr(), ns.data_ptr(), None))
    torch.cuda.synchronize()
    assert np.array_equal(bits(out.cpu().numpy()), bits(G["paged_dense"]))
    nb = (T + 15) // 16
    assert int(ns.item()) == nb
    assert np.array_equal(sel.cpu().numpy()[:nb], np.arange(nb))
    out.zero_()
    eng.check(L.ec_op_paged_attention(C.byref(pv), q.data_ptr(), out.data_ptr(), H, T, 64,
                                      sel.data_ptr(), ns.data_ptr(), None))
    torch.cuda.synchronize()
    assert np.array_equal(bits(out.cpu().numpy()), bits(G["paged_sparse"]))
    want = G["paged_sel"]
    assert int(ns.item()) == want.size
    assert np.array_equal(sel.cpu().numpy()[:want.size], want)


def test_paged_ops_argument_errors(eng, torch):
    import ctypes as C
    L = eng.lib()
    pv, bufs = paged_view(eng, torch, 2, 64, 8)
    x = torch.zeros(512, dtype=torch.float32, device="cuda")
    assert L.ec_op_paged_append(C.byref(pv), x.data_ptr(), x.data_ptr(), 8 * 16, None) == \
        eng.EC_ERR_ARG
    assert L.ec_op_paged_attention(C.byref(pv), x.data_ptr(), x.data_ptr(), 3, 16, 0,
                                   None, None, None) == eng.EC_ERR_ARG
    assert L.ec_op_paged_attention(C.byref(pv), x.data_ptr(), x.data_ptr(), 8, 16, 65,
                                   None, None, None) == eng.EC_ERR_UNSUPPORTED


@pytest.mark.parametrize("chain", [True, False])
def test_layer_chain_matches_oracle(eng, torch, oracle, synth, monkeypatch, chain):
    """Every matrix width a multiple of 512: each layer's o, gate/up, down and
    the next QKV (the LM head after the last layer) run as one persistent
    kernel.  1100 tokens (past the block-sparse threshold) bit-identical to
    the restatement, with the chain and with one launch per matrix."""
    monkeypatch.setenv("EC_NO_CHAIN", "0" if chain else "1")
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=3, n_heads=8, n_kv_heads=4,
                            vocab_size=4096, seq_len=2048, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=21)
    e = eng.Engine(cfg)
    e.load(model)
    # embed + QKV(0) + 3 per layer + argmax with the chain, 6 per layer without
    assert e.launches_per_step(1) == (3 + 3 * 3 if chain else 3 + 6 * 3)
    pm = oracle.PortModel(model)
    toks = synth.prompt(cfg, 1100, seed=5)
    for pos in range(1100):
        check = pos % 50 == 0 or pos >= 1090
        lg, _ = e.step([toks[pos]], [pos], want_logits=check)
        want = pm.forward(int(toks[pos]), pos)
        if check:
            assert np.array_equal(bits(lg[0]), bits(want)), f"step {pos}"
    e.close()


@pytest.mark.parametrize("B", [3, 9])
def test_batched_chain_matches_oracle(eng, torch, oracle, synth, B):
    """B sequences per decode step: the sequence-parallel kernels run once for
    all B, the weight-streaming GEMVs as one batched chain per pack of up to 8
    sequences (B = 9: a pack of 8 and a pack of 1).  Every sequence's logits
    bit-identical to its own restatement model, and the greedy tokens."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=4096, seq_len=2048, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=23)
    e = eng.Engine(cfg, max_batch=B)
    e.load(model)
    packs = (B + 7) // 8
    assert e.launches_per_step(B) == 1 + packs + 2 * (2 + packs) + 1
    pms = [oracle.PortModel(model) for _ in range(B)]
    prompts = [synth.prompt(cfg, 70, seed=40 + b) for b in range(B)]
    for t in range(70):
        check = t % 10 == 0 or t >= 66
        lg, am = e.step([int(p[t]) for p in prompts], [t] * B, want_logits=check)
        for b in range(B):
            want = pms[b].forward(int(prompts[b][t]), t)
            if check:
                assert np.array_equal(bits(lg[b]), bits(want)), f"step {t} sequence {b}"
                assert am[b] == oracle.port().port_argmax(want, want.size)
    e.close()


@pytest.mark.parametrize("heads,hd", [(4, 128), (8, 64)])
def test_group_attention_sparse(eng, torch, oracle, synth, heads, hd):
    """Batched steps (B >= 4) run one attention CTA per (KV head, sequence)
    for all query heads of the group.  Llama-like geometry (4 query heads per
    KV head, head_dim 128) and the 70B shape's 8 query heads per KV head,
    past SPARSE_BLOCKS_K blocks so the block-sparse order matters: every
    checked step's logits bit-identical per sequence."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=heads, n_kv_heads=1,
                            vocab_size=2048, seq_len=2048, head_dim=hd, rope_theta=5e5)
    model = synth.make_model(cfg, seed=31)
    B = 4
    e = eng.Engine(cfg, max_batch=B)
    e.load(model)
    pms = [oracle.PortModel(model) for _ in range(B)]
    prompts = [synth.prompt(cfg, 1060, seed=80 + b) for b in range(B)]
    for t in range(1060):
        check = t % 100 == 0 or t >= 1050
        lg, _ = e.step([int(p[t]) for p in prompts], [t] * B, want_logits=check)
        for b in range(B):
            want = pms[b].forward(int(prompts[b][t]), t)
            if check:
                assert np.array_equal(bits(lg[b]), bits(want)), f"step {t} sequence {b}"
    e.close()


@pytest.mark.parametrize("max_batch", [16, 5])
def test_linear_prefill_matches_sequential_decode(eng, torch, oracle, synth, max_batch):
    """ec_prefill in linear KV mode: a 400-token prompt as rows of batched
    steps into one sequence's BF16 cache.  Past the 128-token window the
    rows select top-32 keys from LSH candidates; the layer-0 index is built
    for the whole chunk before the rows query it, and each row sees only the
    units that end by its own position (as decode would).  The last token's
    logits, every decode step after it and the sparse-query counters are
    bit-identical to feeding the tokens one at a time and to the
    restatement."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=2048, seq_len=512, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=43)
    a = eng.Engine(cfg, use_paged_kv=False, sparse_k=32, max_batch=max_batch)
    b = eng.Engine(cfg, use_paged_kv=False, sparse_k=32, max_batch=1)
    a.load(model)
    b.load(model)
    pm = oracle.PortModel(model, use_paged_kv=False, sparse_k=32)
    n = 400
    prompt = [int(t) for t in synth.prompt(cfg, n, seed=10)]
    lg_a, tok_a = a.prefill(0, prompt)
    for p, t in enumerate(prompt):
        lg_b, am_b = b.step([t], [p])
        want = pm.forward(t, p)
    assert np.array_equal(bits(lg_a), bits(lg_b[0])), "prompt logits"
    assert np.array_equal(bits(lg_a), bits(want)), "prompt logits against the restatement"
    assert tok_a == int(am_b[0])
    assert a.counters(0) == b.counters(0)
    assert a.counters(0)[0] > 0, "the sparse path ran"
    la_idx, lb_idx = a.lsh(0), b.lsh(0)
    assert la_idx["n_units"] == lb_idx["n_units"] == n // 64
    nu = la_idx["n_units"]
    for key in ("unit_hash", "next"):
        assert np.array_equal(la_idx[key][:, :nu], lb_idx[key][:, :nu]), key
    assert np.array_equal(la_idx["heads"], lb_idx["heads"])
    tok = tok_a
    for p in range(n, n + 6):
        la, _ = a.step([tok], [p])
        lb, amb = b.step([tok], [p])
        want = pm.forward(tok, p)
        assert np.array_equal(bits(la[0]), bits(lb[0])), f"decode step {p}"
        assert np.array_equal(bits(la[0]), bits(want)), f"decode step {p} against the restatement"
        tok = int(amb[0])
    assert a.counters(0) == b.counters(0)
    a.close()
    b.close()


@pytest.mark.parametrize("max_batch", [8, 3])
def test_prefill_matches_sequential_decode(eng, torch, oracle, synth, max_batch):
    """ec_prefill runs a 150-token prompt as rows of batched steps (chunks of
    max_batch rows into one sequence's paged cache; the block selection is
    active past 4 blocks) -- the last token's logits, and every decode step
    after it, bit-identical to feeding the tokens one at a time and to the
    restatement.  The layer-0 LSH index (lsh_update runs on every token in
    paged mode as well, inference.c:177-191) is built for the prefilled
    sequence in token order and leaves the other sequences untouched."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=2048, seq_len=512, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=41)
    a = eng.Engine(cfg, max_batch=max_batch, sparse_blocks_k=4)
    b = eng.Engine(cfg, max_batch=1, sparse_blocks_k=4)
    a.load(model)
    b.load(model)
    pm = oracle.PortModel(model, sparse_blocks_k=4)
    n = 150
    prompt = [int(t) for t in synth.prompt(cfg, n, seed=9)]
    other_before = a.lsh(1)
    lg_a, tok_a = a.prefill(0, prompt)
    for p, t in enumerate(prompt):
        lg_b, am_b = b.step([t], [p])
        want = pm.forward(t, p)
    assert np.array_equal(bits(lg_a), bits(lg_b[0])), "prompt logits"
    assert np.array_equal(bits(lg_a), bits(want)), "prompt logits against the restatement"
    assert tok_a == int(am_b[0])
    la_idx, lb_idx = a.lsh(0), b.lsh(0)
    assert la_idx["n_units"] == lb_idx["n_units"] == n // 64
    nu = la_idx["n_units"]  # unit slots past n_units are never written
    for key in ("unit_start", "unit_len"):
        assert np.array_equal(la_idx[key][:nu], lb_idx[key][:nu]), key
    for key in ("unit_hash", "next"):
        assert np.array_equal(la_idx[key][:, :nu], lb_idx[key][:, :nu]), key
    assert np.array_equal(la_idx["heads"], lb_idx["heads"])
    po = pm.lsh()
    assert po.n_units == la_idx["n_units"]
    for u in range(po.n_units):
        assert po.unit_hash[u] == la_idx["unit_hash"][0, u]
        assert po.unit_start[u] == la_idx["unit_start"][u]
    other_after = a.lsh(1)
    for key in ("unit_hash", "unit_start", "unit_len", "heads", "next"):
        assert np.array_equal(np.asarray(other_before[key]), np.asarray(other_after[key])), key
    assert other_after["n_units"] == other_before["n_units"]
    assert a.counters(0) == b.counters(0)
    tok = tok_a
    for p in range(n, n + 6):
        la, ama = a.step([tok], [p])
        lb, amb = b.step([tok], [p])
        want = pm.forward(tok, p)
        assert np.array_equal(bits(la[0]), bits(lb[0])), f"decode step {p}"
        assert np.array_equal(bits(la[0]), bits(want)), f"decode step {p} against the restatement"
        tok = int(ama[0])
    a.close()
    b.close()
