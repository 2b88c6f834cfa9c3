"""Pins the C restatement (oracle/port) to vectors produced by the reference
engine itself (tests/golden/make_golden.py).  Runs anywhere: no reference
sources and no GPU needed.  Everything is bit-exact."""
import os
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import digest, lsh_keys, paged_inputs  # noqa: E402

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_vectors.npz"))


def same_bits(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_gemv(oracle):
    w, x = G["gemv_w"], G["gemv_x"]
    y = np.zeros(w.shape[0], np.float32)
    oracle.port().port_gemv_bf16(y, w, x, w.shape[0], w.shape[1])
    assert same_bits(y, G["gemv_y"])


def test_rmsnorm(oracle):
    y = np.zeros_like(G["norm_x"])
    oracle.port().port_rmsnorm(y, G["norm_x"], G["norm_w"], y.size, np.float32(1e-5))
    assert same_bits(y, G["norm_y"])


def test_rope(oracle):
    P = oracle.port()
    ct = np.zeros_like(G["rope_cos"])
    st = np.zeros_like(G["rope_sin"])
    P.port_rope_tables(ct, st, 128, 512, np.float32(5e5))
    assert same_bits(ct, G["rope_cos"]) and same_bits(st, G["rope_sin"])
    q = G["rope_in"].copy()
    P.port_rope(q, 8, 128, 311, ct, st, 512)
    assert same_bits(q, G["rope_out"])


def test_silu(oracle):
    y = np.zeros_like(G["silu_g"])
    oracle.port().port_silu_mul(y, G["silu_g"], G["silu_u"], y.size)
    assert same_bits(y, G["silu_y"])


def test_quant_int8(oracle):
    for i, row in enumerate(G["quant_in"]):
        q = np.zeros(row.size, np.int8)
        s = oracle.port().port_quant_int8(q, np.ascontiguousarray(row), row.size)
        assert np.float32(s) == G["quant_s"][i]
        assert np.array_equal(q, G["quant_q"][i])


def test_heap_and_argmax(oracle):
    P = oracle.port()
    out = np.zeros(37, np.int32)
    n = P.port_heap_topk(G["heap_scores"], G["heap_idx"], 300, 37, out)
    assert np.array_equal(out[:n], G["heap_out"])
    lg = G["argmax_in"]
    assert P.port_argmax(lg, lg.size) == int(G["argmax_out"])


def test_paged(oracle):
    P = oracle.port()
    KV, H, hd, T = 2, 8, 64, 1100
    kk, vv = paged_inputs(T, KV * hd)
    pp = P.port_paged_create(KV, hd, 2048)
    for p in range(T):
        P.port_paged_append(pp, np.ascontiguousarray(kk[p]), np.ascontiguousarray(vv[p]), p)
    q = G["paged_q"]
    nb = pp.contents.n_blocks
    o = np.zeros(H * hd, np.float32)
    P.port_paged_attention(o, q, pp, np.arange(nb, dtype=np.int32), nb, H)
    assert same_bits(o, G["paged_dense"])
    sc = np.zeros(nb, np.float32)
    P.port_paged_scores(pp, q, sc)
    sel = np.zeros(70, np.int32)
    ns = P.port_select_blocks(sc, nb, 64, sel)
    assert np.array_equal(sel[:ns], G["paged_sel"])
    P.port_paged_attention(o, q, pp, sel, ns, H)
    assert same_bits(o, G["paged_sparse"])
    P.port_paged_free(pp)


def test_lsh(oracle):
    P = oracle.port()
    hd = 64
    pl = P.port_lsh_create(1, 16, hd, 64, 4096, 4, 42)
    hp = np.ctypeslib.as_array(pl.contents.hp, (16 * hd,)).reshape(16, hd)
    assert same_bits(hp, G["lsh_hp"])
    h = [P.port_lsh_hash(pl, 0, np.ascontiguousarray(v)) for v in G["lsh_vecs"]]
    assert np.array_equal(np.array(h, np.int32), G["lsh_hashes"])
    _, keys = lsh_keys(hd, 64 * 200)
    for p in range(keys.shape[0]):
        P.port_lsh_update(pl, np.ascontiguousarray(keys[p]), p)
    L = pl.contents
    n = L.n_units
    assert n == G["lsh_block_hashes"].size
    assert np.array_equal(np.ctypeslib.as_array(L.unit_hash, (n,)).astype(np.int32),
                          G["lsh_block_hashes"])
    assert np.array_equal(np.ctypeslib.as_array(L.heads, (65536,)), G["lsh_heads"])
    assert np.array_equal(np.ctypeslib.as_array(L.next, (n,)), G["lsh_next"])
    for qh, want in zip(G["lsh_qhash"], G["lsh_cands"]):
        o = np.zeros(64, np.int32)
        c = P.port_lsh_find(pl, np.array([qh], np.uint32), o, 64)
        assert np.array_equal(o[:c], want[want >= 0])
    P.port_lsh_free(pl)


@pytest.mark.parametrize("mode", ["paged", "linear"])
def test_tiny_decode_trace(oracle, tiny_model, mode):
    """64-token prompt + 128 greedy steps: every step's logits bit-identical to
    the reference's, same greedy tokens, same LSH query counters."""
    paged = mode == "paged"
    pm = oracle.PortModel(tiny_model, use_paged_kv=paged, sparse_k=64 if paged else 32)
    toks = G[f"tiny_{mode}_tokens"]
    dg = G[f"tiny_{mode}_digests"]
    P = oracle.port()
    for pos in range(dg.size):
        lg = pm.forward(int(toks[pos]), pos)
        assert digest(lg) == dg[pos], f"step {pos}"
        if pos >= 63:
            assert P.port_argmax(lg, lg.size) == toks[pos + 1]
    assert np.array_equal(np.array(pm.counters()), G[f"tiny_{mode}_counters"])


def test_reference_context_fill(ref, synth):
    """The CPU baseline's context fill: positions 0..n-1 of the reference's
    paged cache through its own paged_kv_append / lsh_update, then decode
    steps at position n (finite logits, the block-sparse path active past
    1024 tokens)."""
    cfg = synth.ModelConfig(dim=256, hidden_dim=512, n_layers=2, n_heads=4, n_kv_heads=2,
                            vocab_size=512, seq_len=2048, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=2)
    m = ref.RefModel(model, use_paged_kv=True, sparse_k=64)
    m.fill_context(1100, seed=3)
    for p in range(1100, 1103):
        lg = m.forward(5, p)
        assert np.all(np.isfinite(lg))
    kb = np.zeros(cfg.n_kv_heads * 16 * cfg.head_dim, np.int8)
    vb = np.zeros_like(kb)
    ks = np.zeros(cfg.n_kv_heads * 16, np.float32)
    vs = np.zeros_like(ks)
    cen = np.zeros(cfg.head_dim, np.float32)
    assert ref.ref().refd_paged_block(m.h, 1, 68, kb, vb, ks, vs, cen) == 15
    assert ref.ref().refd_paged_block(m.h, 1, 67, kb, vb, ks, vs, cen) == 16
    assert np.abs(cen).max() > 0
