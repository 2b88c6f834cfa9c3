"""Isolated LSH sparse attention through the C ABI
against the restatement (oracle/port/lsh_attn.c), bit for bit: the selected
positions in the reference's heap order and every head's output.  Cases:
per-key units with and without the candidate cut-off, 16-token units, and
the reference's own setting (1 table x 16 bits x 64-token units); and the
same cache as paged 16-token blocks under a shuffled page table
(ec_lsh_attn_build_paged), which must give the identical result."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def bf16_to_f32(u):
    return (u.astype(np.uint32) << 16).view(np.float32)


def planted_case(synth, T, H, KV, hd, window, seed):
    """BF16 K/V N(0,1); 64 keys before the window set to q + N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    base = rng.standard_normal(hd, dtype=np.float32)
    q = (base[None, :] + np.float32(0.1) * rng.standard_normal((H, hd), dtype=np.float32))
    q = q.astype(np.float32)
    k = rng.standard_normal((T, KV, hd), dtype=np.float32)
    v = rng.standard_normal((T, KV, hd), dtype=np.float32)
    planted = rng.choice(T - window, 64, replace=False)
    grp = H // KV
    for p in planted:
        for kv in range(KV):
            k[p, kv] = q[kv * grp] + np.float32(0.1) * rng.standard_normal(hd, dtype=np.float32)
    return q, synth.f32_to_bf16(k), synth.f32_to_bf16(v), np.sort(planted)


@pytest.mark.parametrize("tables,bits,unit,max_cand", [(4, 8, 1, 4096), (4, 8, 1, 40),
                                                       (4, 8, 16, 64), (1, 16, 64, 64)])
def test_lsh_attention_matches_oracle(torch, oracle, synth, tables, bits, unit, max_cand):
    from conftest import load_pkg_module
    eng = load_pkg_module("engine")
    H, KV, hd, T, window, top_k, radius = 8, 2, 64, 3000, 128, 64, 4
    q, k, v, planted = planted_case(synth, T, H, KV, hd, window, seed=tables * 100 + unit)
    # oracle
    P = oracle.port()
    lsh = P.port_lsh_create(tables, bits, hd, unit, T // unit + 1, radius, 42)
    k0 = bf16_to_f32(k[:, 0, :]).astype(np.float32)
    for t in range(T):
        P.port_lsh_update(lsh, np.ascontiguousarray(k0[t]), t)
    want_sel = np.zeros(T, np.int32)
    want_out = np.zeros(H * hd, np.float32)
    n = P.port_lsh_attend(lsh, np.ascontiguousarray(k.reshape(-1)),
                          np.ascontiguousarray(v.reshape(-1)), T, np.ascontiguousarray(q.reshape(-1)),
                          H, KV, hd, window, max_cand, top_k, want_sel, want_out)
    P.port_lsh_free(lsh)
    # device
    L = eng.lib()
    cfg = eng.LshAttnConfig(H, KV, hd, T, tables, bits, unit, radius, max_cand, window, top_k, 1)
    h = C.c_void_p()
    eng.check(L.ec_lsh_attn_create(C.byref(cfg), 0, C.byref(h)))
    try:
        dk = torch.from_numpy(k.reshape(-1)).cuda()
        dv = torch.from_numpy(v.reshape(-1)).cuda()
        dq = torch.from_numpy(q.reshape(-1)).cuda()
        out = torch.full((H * hd,), float("nan"), device="cuda")
        sel = torch.full((top_k,), -7, dtype=torch.int32, device="cuda")
        ns = torch.zeros(1, dtype=torch.int32, device="cuda")
        eng.check(L.ec_lsh_attn_build(h, dk.data_ptr(), dv.data_ptr(), T, None))
        eng.check(L.ec_lsh_attn_query(h, dq.data_ptr(), 1, out.data_ptr(), sel.data_ptr(),
                                      ns.data_ptr(), None))
        torch.cuda.synchronize()
        assert int(ns.item()) == n
        assert np.array_equal(sel.cpu().numpy()[:n], want_sel[:n])
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want_out.view(np.uint32))
        if unit == 1 and max_cand >= 4096:
            # the planted keys are found (recall of the configuration's check)
            assert len(set(planted) & set(want_sel[:n].tolist())) >= 32
    finally:
        L.ec_lsh_attn_destroy(h)


@pytest.mark.parametrize("T,top_k", [(3000, 64), (100, 256)])
def test_lsh_attention_paged_cache(torch, oracle, synth, T, top_k):
    """The cache as paged blocks ([block][16][KV][hd], blocks shuffled by a
    page table): selection and output bit-identical to the restatement over
    the linear cache -- the sparse case, and a context shorter than top_k
    (every position attended, in order, through the page table)."""
    from conftest import load_pkg_module
    eng = load_pkg_module("engine")
    H, KV, hd, window, tables, bits, unit, max_cand, radius = 8, 2, 64, 128, 4, 8, 16, 64, 4
    q, k, v, _ = planted_case(synth, max(T, 300), H, KV, hd, window, seed=T)
    k, v = k[:T], v[:T]
    P = oracle.port()
    lsh = P.port_lsh_create(tables, bits, hd, unit, T // unit + 1, radius, 42)
    k0 = bf16_to_f32(k[:, 0, :]).astype(np.float32)
    for t in range(T):
        P.port_lsh_update(lsh, np.ascontiguousarray(k0[t]), t)
    want_sel = np.zeros(T, np.int32)
    want_out = np.zeros(H * hd, np.float32)
    n = P.port_lsh_attend(lsh, np.ascontiguousarray(k.reshape(-1)),
                          np.ascontiguousarray(v.reshape(-1)), T, np.ascontiguousarray(q.reshape(-1)),
                          H, KV, hd, window, max_cand, top_k, want_sel, want_out)
    P.port_lsh_free(lsh)
    nblk = (T + 15) // 16
    rng = np.random.default_rng(3)
    pt = rng.permutation(nblk + 5)[:nblk].astype(np.int32)   # logical -> physical
    kp = np.zeros((nblk + 5, 16, KV, hd), np.uint16)
    vp = np.zeros_like(kp)
    for lb in range(nblk):
        m = min(16, T - lb * 16)
        kp[pt[lb], :m] = k[lb * 16:lb * 16 + m]
        vp[pt[lb], :m] = v[lb * 16:lb * 16 + m]
    L = eng.lib()
    cfg = eng.LshAttnConfig(H, KV, hd, (nblk + 5) * 16, tables, bits, unit, radius, max_cand,
                            window, top_k, 1)
    h = C.c_void_p()
    eng.check(L.ec_lsh_attn_create(C.byref(cfg), 0, C.byref(h)))
    try:
        dk = torch.from_numpy(kp.reshape(-1)).cuda()
        dv = torch.from_numpy(vp.reshape(-1)).cuda()
        dpt = torch.from_numpy(pt).cuda()
        dq = torch.from_numpy(q.reshape(-1)).cuda()
        out = torch.full((H * hd,), float("nan"), device="cuda")
        sel = torch.full((top_k,), -7, dtype=torch.int32, device="cuda")
        ns = torch.zeros(1, dtype=torch.int32, device="cuda")
        eng.check(L.ec_lsh_attn_build_paged(h, dk.data_ptr(), dv.data_ptr(), dpt.data_ptr(), T,
                                            None))
        eng.check(L.ec_lsh_attn_query(h, dq.data_ptr(), 1, out.data_ptr(), sel.data_ptr(),
                                      ns.data_ptr(), None))
        torch.cuda.synchronize()
        if n < T:
            assert int(ns.item()) == n
            assert np.array_equal(sel.cpu().numpy()[:n], want_sel[:n])
        else:
            assert int(ns.item()) == -1  # dense: every position
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want_out.view(np.uint32))
    finally:
        L.ec_lsh_attn_destroy(h)
