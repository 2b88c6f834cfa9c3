"""Generate tests/golden/ref_vectors.npz from the reference engine itself.

Run in a container that has the reference sources (the oracle/_ref library is
built from them by `make -C oracle ref`):

    python tests/golden/make_golden.py

Every input is drawn from a fixed numpy seed and stored next to the output
(or, for the synthetic models, regenerated from the seed by synth.make_model),
so tests/test_golden.py can check the C restatement -- and through it the CUDA
library -- on machines where the reference is absent.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.dirname(HERE))
import oracle as O  # noqa: E402
from conftest import load_pkg_module  # noqa: E402

S = load_pkg_module("synth")


def paged_inputs(T, width):
    """K and V rows for the paged-cache vectors (seed 31)."""
    r = np.random.default_rng(31)
    return (r.standard_normal((T, width), dtype=np.float32),
            r.standard_normal((T, width), dtype=np.float32))


def lsh_keys(hd, n):
    """Clustered keys for the LSH index vectors (seed 32)."""
    r = np.random.default_rng(32)
    base = r.standard_normal((8, hd), dtype=np.float32)
    keys = (base[(np.arange(n) // 64) % 8]
            + np.float32(0.3) * r.standard_normal((n, hd), dtype=np.float32)).astype(np.float32)
    return base, keys


def digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()[:16]


def decode_trace(model, paged, sparse_k, n_prompt, n_gen):
    """Prompt of n_prompt seeded ids, then greedy decode with the reference's
    own argmax (sample_argmax).  Returns tokens and per-step logits digests."""
    rm = O.RefModel(model, use_paged_kv=paged, sparse_k=sparse_k)
    toks = [int(t) for t in S.prompt(model.cfg, n_prompt)]
    digests, logits_keep = [], []
    R = O.ref()
    for pos in range(n_prompt + n_gen):
        lg = rm.forward(toks[pos], pos)
        digests.append(digest(lg))
        if pos in (n_prompt - 1, n_prompt + n_gen - 1):
            logits_keep.append(lg.copy())
        if pos >= n_prompt - 1:
            toks.append(int(R.refd_argmax(lg, lg.size)))
    return np.array(toks, np.int32), np.array(digests), np.stack(logits_keep), rm.counters()


def main():
    R = O.ref()
    rng = np.random.default_rng(2024)
    g = {}
    # GEMV (op_matmul, batch 1)
    m, k = 48, 4096 + 40
    w = S.f32_to_bf16(rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.02))
    x = rng.standard_normal(k, dtype=np.float32)
    y = np.zeros(m, np.float32)
    R.refd_matmul(y, w, x, m, k)
    g.update(gemv_w=w, gemv_x=x, gemv_y=y)
    # RMSNorm
    n = 4096 + 4
    x = rng.standard_normal(n, dtype=np.float32)
    wn = S.f32_to_bf16(1 + 0.1 * rng.standard_normal(n, dtype=np.float32))
    y = np.zeros(n, np.float32)
    R.refd_rmsnorm(y, x, wn, n, np.float32(1e-5))
    g.update(norm_x=x, norm_w=wn, norm_y=y)
    # RoPE (tables + rotation)
    hd, seq = 128, 512
    rc = R.refd_rope_create(hd, seq, np.float32(5e5))
    ct = np.ctypeslib.as_array(R.refd_rope_table(rc, 0), (seq * hd // 2,)).copy()
    st = np.ctypeslib.as_array(R.refd_rope_table(rc, 1), (seq * hd // 2,)).copy()
    qv = rng.standard_normal(8 * hd, dtype=np.float32)
    qr = qv.copy()
    R.refd_rope_apply(rc, qr, 8, 311)
    g.update(rope_cos=ct, rope_sin=st, rope_in=qv, rope_out=qr)
    # SiLU * up
    n = 1408 + 3
    gt = (rng.standard_normal(n, dtype=np.float32) * 4).astype(np.float32)
    up = rng.standard_normal(n, dtype=np.float32)
    y = np.zeros(n, np.float32)
    R.refd_silu_mul(y, gt, up, n)
    g.update(silu_g=gt, silu_u=up, silu_y=y)
    # INT8 KV quantisation
    v = (rng.standard_normal((64, 128), dtype=np.float32)
         * rng.uniform(0.01, 10, (64, 1)).astype(np.float32)).astype(np.float32)
    v[3] = 0
    qs, ss = np.zeros_like(v, np.int8), np.zeros(64, np.float32)
    for i in range(64):
        row = np.zeros(128, np.int8)
        ss[i] = R.refd_quant_int8(row, np.ascontiguousarray(v[i]), 128)
        qs[i] = row
    g.update(quant_in=v, quant_q=qs, quant_s=ss)
    # heap top-K with ties
    sc = np.round(rng.standard_normal(300), 1).astype(np.float32)
    ix = (np.arange(300) * 7).astype(np.int32)
    out = np.zeros(37, np.int32)
    nk = R.refd_heap_topk(sc, ix, 300, 37, out)
    g.update(heap_scores=sc, heap_idx=ix, heap_out=out[:nk])
    # argmax with ties
    lg = np.round(rng.standard_normal(32003), 2).astype(np.float32)
    g.update(argmax_in=lg, argmax_out=np.int32(R.refd_argmax(lg, lg.size)))
    # paged INT8 KV: append, dense and block-sparse attention
    KV, H, hd, T = 2, 8, 64, 1100
    kk, vv = paged_inputs(T, KV * hd)
    rp = R.refd_paged_create(KV, hd, 2048)
    for p in range(T):
        R.refd_paged_append(rp, np.ascontiguousarray(kk[p]), np.ascontiguousarray(vv[p]), p)
    q = rng.standard_normal(H * hd, dtype=np.float32)
    od = np.zeros(H * hd, np.float32)
    R.refd_paged_attention(rp, od, q, H, KV, hd)
    osp = np.zeros(H * hd, np.float32)
    sel = np.zeros(70, np.int32)
    ns = R.refd_paged_sparse(rp, osp, q, H, KV, hd, 64, sel)
    nb = R.refd_paged_nblocks(rp)
    phys2log = {R.refd_paged_phys(rp, b): b for b in range(nb)}
    g.update(paged_q=q, paged_dense=od, paged_sparse=osp,
             paged_sel=np.array([phys2log[s] for s in sel[:ns]], np.int32))
    # LSH: hyperplanes, hashes, index and multiprobe candidates (1 x 16 bits)
    hd = 64
    lc = R.refd_lsh_ctx_create(hd, 42)
    hp = np.ctypeslib.as_array(R.refd_lsh_hyperplanes(lc), (16 * 256,)).reshape(16, 256)[:, :hd]
    vecs = rng.standard_normal((256, hd), dtype=np.float32)
    vecs[7] = 0
    hashes = np.array([R.refd_lsh_hash(lc, np.ascontiguousarray(r)) for r in vecs], np.int32)
    li = R.refd_lsh_index_create()
    base, keys = lsh_keys(hd, 64 * 200)
    for p in range(keys.shape[0]):
        R.refd_lsh_update(li, lc, np.ascontiguousarray(keys[p]), hd, p)
    idx = O.C.cast(li, O.C.POINTER(O.LshIndex)).contents
    nbk = idx.n_blocks
    qh = np.array([R.refd_lsh_hash(lc, np.ascontiguousarray(base[i % 8] + np.float32(0.5) * r))
                   for i, r in enumerate(rng.standard_normal((40, hd), dtype=np.float32))],
                  np.int32)
    cands = np.full((40, 64), -1, np.int32)
    for i, h in enumerate(qh):
        o = np.zeros(64, np.int32)
        c = R.refd_lsh_find(li, int(h), o, 64)
        cands[i, :c] = o[:c]
    g.update(lsh_hp=hp.copy(), lsh_vecs=vecs, lsh_hashes=hashes, 
             lsh_block_hashes=np.array(idx.block_hashes[:nbk], np.int32),
             lsh_heads=np.array(idx.bucket_heads[:], np.int32),
             lsh_next=np.array(idx.chain_next[:nbk], np.int32),
             lsh_qhash=qh, lsh_cands=cands)
    # tiny model: 64-token prompt + greedy decode, both KV modes
    model = S.make_model(S.TINY, seed=7)
    for name, paged, sk in (("paged", True, 64), ("linear", False, 32)):
        toks, dg, keep, cnt = decode_trace(model, paged, sk, 64, 128)
        g[f"tiny_{name}_tokens"] = toks
        g[f"tiny_{name}_digests"] = dg
        g[f"tiny_{name}_logits"] = keep
        g[f"tiny_{name}_counters"] = np.array(cnt, np.int64)
    path = os.path.join(HERE, "ref_vectors.npz")
    np.savez_compressed(path, **g)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
