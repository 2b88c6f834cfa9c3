"""Failure detection without a GPU fault: every wait inside the kernels is
bounded and ends in EC_ERR_TIMEOUT instead of a hang.

A test-only wait limit (ec_model_config.wait_limit < 0) makes the GEMV
chain's grid-wide phase wait look for a count that no CTA ever reaches; the
wait gives up after a few hundred polls, the CTA drains its in-flight copies
and stops computing, and ec_decode_step returns EC_ERR_TIMEOUT.  A fresh
context on the same device then decodes normally, bit-identical to the
restatement.  Nothing here traps, faults or spins without a limit.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import load_pkg_module

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def eng():
    return load_pkg_module("engine")


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _cfg(synth):
    return synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                             vocab_size=2048, seq_len=256, head_dim=64, rope_theta=1e4)


def test_chain_wait_times_out_then_fresh_context_works(eng, torch, oracle, synth):
    cfg = _cfg(synth)
    model = synth.make_model(cfg, seed=3)
    bad = eng.Engine(cfg, wait_limit=-500)
    bad.load(model)
    tok = np.array([5], np.int32)
    pos = np.array([0], np.int32)
    am = np.zeros(1, np.int32)
    rc = eng.lib().ec_decode_step(bad.h, C.c_void_p(tok.ctypes.data), C.c_void_p(pos.ctypes.data),
                                  1, None, C.c_void_p(am.ctypes.data))
    assert rc == eng.EC_ERR_TIMEOUT, eng.lib().ec_last_error()
    assert b"timed out" in eng.lib().ec_last_error()
    bad.close()
    good = eng.Engine(cfg)
    good.load(model)
    pm = oracle.PortModel(model)
    for p, t in enumerate(synth.prompt(cfg, 6, seed=1)):
        lg, _ = good.step([int(t)], [p])
        want = pm.forward(int(t), p)
        assert np.array_equal(lg[0].view(np.uint32), want.view(np.uint32)), f"step {p}"
    good.close()


def test_wait_limit_default_and_positive(eng, torch, oracle, synth):
    """A positive limit (polls) is only a bound: steps that never wait that
    long decode as with the default."""
    cfg = _cfg(synth)
    model = synth.make_model(cfg, seed=4)
    e = eng.Engine(cfg, wait_limit=1 << 22)
    e.load(model)
    pm = oracle.PortModel(model)
    for p, t in enumerate(synth.prompt(cfg, 4, seed=2)):
        lg, _ = e.step([int(t)], [p])
        assert np.array_equal(lg[0].view(np.uint32), pm.forward(int(t), p).view(np.uint32))
    e.close()
