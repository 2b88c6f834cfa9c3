"""ec_op_paged_attention_static -- the entry point that allocates nothing --
against ec_op_paged_attention on the same paged cache.  Collected last so it
also runs after every other GPU test in one process; it passes alone too.

Two calls in a row (block-sparse, then dense) check that the shared fixed
scratch left by one call does not leak into the next; results must be
bit-identical to the allocating entry point's, the tolerance every parity
test here uses."""
import ctypes as C
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from conftest import load_pkg_module  # noqa: E402
from make_golden import paged_inputs  # noqa: E402


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def test_static_scratch_matches_allocating_op(torch):
    eng = load_pkg_module("engine")
    L = eng.lib()
    KV, H, hd, T, MB = 2, 8, 64, 1100, 128
    perm = np.random.default_rng(9).permutation(MB).astype(np.int32)
    k = torch.zeros(MB * KV * 16 * hd, dtype=torch.int8, device="cuda")
    v = torch.zeros_like(k)
    ks = torch.zeros(MB * KV * 16, dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    cen = torch.zeros(MB * hd, dtype=torch.float32, device="cuda")
    pt = torch.from_numpy(perm).cuda()
    pv = eng.PagedView(k.data_ptr(), v.data_ptr(), ks.data_ptr(), vs.data_ptr(),
                       cen.data_ptr(), pt.data_ptr(), KV, hd, MB)
    kk, vv = (torch.from_numpy(a).cuda() for a in paged_inputs(T, KV * hd))
    for p in range(T):
        eng.check(L.ec_op_paged_append(C.byref(pv), kk[p].data_ptr(), vv[p].data_ptr(), p, None))
    q = torch.from_numpy(np.random.default_rng(3).standard_normal(
        H * hd, dtype=np.float32)).cuda()

    def run(fn, sbk):
        out = torch.full((H * hd,), float("nan"), device="cuda")
        sel = torch.full((80,), -7, dtype=torch.int32, device="cuda")
        ns = torch.full((1,), -7, dtype=torch.int32, device="cuda")
        eng.check(fn(C.byref(pv), q.data_ptr(), out.data_ptr(), H, T, sbk,
                     sel.data_ptr(), ns.data_ptr(), None))
        torch.cuda.synchronize()
        n = int(ns.item())
        return out.cpu().numpy(), sel.cpu().numpy()[:n], n

    for sbk in (64, 0):  # two calls in a row on the shared scratch
        got = run(L.ec_op_paged_attention_static, sbk)
        want = run(L.ec_op_paged_attention, sbk)
        assert got[2] == want[2] == (64 if sbk else (T + 15) // 16)
        assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32))
        assert np.array_equal(got[1], want[1])


def test_static_scratch_rejects_oversize(torch):
    eng = load_pkg_module("engine")
    L = eng.lib()
    x = torch.zeros(4096, dtype=torch.float32, device="cuda")
    pt = torch.zeros(4096, dtype=torch.int32, device="cuda")
    pv = eng.PagedView(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(),
                       pt.data_ptr(), 1, 64, 4096)
    rc = L.ec_op_paged_attention_static(C.byref(pv), x.data_ptr(), x.data_ptr(), 1,
                                        2049 * 16, 64, None, None, None)
    assert rc == eng.EC_ERR_UNSUPPORTED
    assert b"fixed scratch" in L.ec_last_error()
