"""Tensor parallelism (ec_create_tp) on 2 GPUs, one process per GPU.

Each rank holds half of the heads, KV heads, FFN rows and vocabulary rows;
the row-split projections are gathered and added in rank order, the
reference's cross-head quantities (LSH query mean, candidate scores summed
over KV heads, the paged block selection from query head 0, the layer-0 LSH
key) are exchanged.  Against the restatement of the whole model: every
step's logits within BASELINE's 2e-2 of the logit range, every greedy token
equal, and both ranks holding bit-identical logits.  Skipped with fewer
than 2 GPUs (the round-end suite runs on one)."""
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _cfg(synth):
    # H * hd / 2 and F / 2 multiples of 512: the GEMV chain on each rank
    return synth.ModelConfig(dim=1024, hidden_dim=1024, n_layers=2, n_heads=16, n_kv_heads=2,
                             vocab_size=2048, seq_len=512, head_dim=64, rope_theta=1e4)


def _worker(rank, world, uid, kind, paged, n_prompt, n_greedy, out_q):
    sys.path.insert(0, HERE)
    from conftest import load_pkg_module
    eng, synth = load_pkg_module("engine"), load_pkg_module("synth")
    cfg = _cfg(synth)
    model = synth.make_model(cfg, seed=13, kind=kind)
    e = eng.Engine(cfg, device=rank, tp=(rank, world, uid),
                   weight_kind=eng.EC_W_INT8 if kind == "int8" else eng.EC_W_FP8,
                   use_paged_kv=paged, sparse_k=64 if paged else 32, sparse_blocks_k=4)
    e.load(model)
    toks = [int(t) for t in synth.prompt(cfg, n_prompt, seed=21)]
    fed, logits = [], []
    tok = toks[0]
    for p in range(n_prompt + n_greedy):
        lg, am = e.step([tok], [p])
        fed.append(tok)
        logits.append(lg[0].copy())
        tok = toks[p + 1] if p + 1 < n_prompt else int(am[0])
    out_q.put((rank, fed, np.stack(logits)))
    e.close()


@pytest.mark.parametrize("kind,paged", [("int8", True), ("fp8", False)])
def test_tp2_matches_restatement(oracle, synth, kind, paged):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    sys.path.insert(0, HERE)
    from conftest import load_pkg_module
    eng = load_pkg_module("engine")
    uid = eng.tp_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n_prompt, n_greedy = 200, 64
    procs = [ctx.Process(target=_worker, args=(r, 2, uid, kind, paged, n_prompt, n_greedy, q))
             for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            r, fed, lgs = q.get(timeout=300)
            res[r] = (fed, lgs)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    for p in procs:
        assert p.exitcode == 0
    fed0, lg0 = res[0]
    fed1, lg1 = res[1]
    assert fed0 == fed1
    assert np.array_equal(lg0.view(np.uint32), lg1.view(np.uint32)), "ranks disagree"
    cfg = _cfg(synth)
    model = synth.make_model(cfg, seed=13, kind=kind)
    pm = oracle.PortModel(model, use_paged_kv=paged, sparse_k=64 if paged else 32,
                          sparse_blocks_k=4)
    P = oracle.port()
    for p, t in enumerate(fed0):
        want = pm.forward(t, p)
        d = float(np.abs(lg0[p] - want).max())
        assert d <= 2e-2 * float(want.max() - want.min()), f"step {p}: |d| {d}"
        if p + 1 >= n_prompt and p + 1 < len(fed0):
            assert fed0[p + 1] == P.port_argmax(want, want.size), f"greedy token after step {p}"
