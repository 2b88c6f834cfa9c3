"""The drop-in, end to end: the reference's own transformer_forward
(src/inference/inference.c, compiled from a copy patched by oracle/dropin.py
with the hook INTEGRATION.md shows) runs the decode step on libengine_cuda.so
once a context is attached -- and its logits match the digests the
unmodified reference produced on the CPU (tests/golden), bit for bit, over
the tiny model's 64-token prompt and greedy continuation."""
import os
import sys

import pytest

from conftest import load_pkg_module

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from make_golden import digest  # noqa: E402

import numpy as np  # noqa: E402

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_vectors.npz"))


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def test_reference_transformer_forward_through_the_hook(torch, oracle, tiny_model):
    if not oracle.dropin_available():
        pytest.skip("oracle/_ref/libref_dropin.so not built (make -C oracle dropin)")
    eng = load_pkg_module("engine")
    e = eng.Engine(tiny_model.cfg)  # loads libengine_cuda.so before the drop-in build
    e.load(tiny_model)
    lib = oracle.dropin()
    m = oracle.RefModel(tiny_model, use_paged_kv=True, sparse_k=64, lib=lib)
    lib.refd_attach_gpu(m.h, e.h)
    toks = G["tiny_paged_tokens"]
    dg = G["tiny_paged_digests"]
    for pos in range(96):
        lg = m.forward(int(toks[pos]), pos)
        assert digest(lg) == dg[pos], f"step {pos}"
    lib.refd_attach_gpu(m.h, None)
    e.close()
