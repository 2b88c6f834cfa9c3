"""The split decode attention (attention_mode EC_ATTN_SPLIT /
EC_ATTN_SPLIT_EXACT_EXP, csrc/attn_fast.cu) against the restatement.

The top-K block set is selected by ranks over the reference's block scores,
so it must equal select_top_k_blocks' set (paged.c:439-495) exactly; the
attention is split over many CTAs per KV head and merged, so its rounding
differs from the reference's sequential online softmax: logits must agree
within BASELINE's 2e-2 of the logit range and greedy tokens must be equal.
"""
import numpy as np
import pytest

from conftest import load_pkg_module

pytestmark = pytest.mark.gpu
TOL = 2e-2


@pytest.fixture(scope="module")
def eng():
    return load_pkg_module("engine")


@pytest.fixture(scope="module")
def torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def within(got, want):
    return float(np.abs(got - want).max()) <= TOL * float(want.max() - want.min())


def selection_matches(e, cfg, P, pos):
    """The engine's selected block SET equals select_top_k_blocks
    (paged.c:439-495) run on the engine's own query head 0 and block
    centroids of the last layer (score_blocks' dot, paged.c:401-431)."""
    hd = cfg.head_dim
    nb = (pos + 1 + 15) // 16
    q0 = e.state(2)[:hd].copy()
    mb = (cfg.seq_len + 15) // 16
    cen = e.state(9, n=mb * hd)[:nb * hd].reshape(nb, hd)
    sc = np.array([P.port_dot_f32(q0, np.ascontiguousarray(cen[i]), hd) for i in range(nb)],
                  np.float32)
    sel = np.zeros(70, np.int32)
    ns = P.port_select_blocks(sc, nb, 64, sel)
    got = e.state(8, n=80)
    return int(got[0]) == ns and np.array_equal(np.sort(got[1:1 + ns].astype(np.int32)),
                                                np.sort(sel[:ns]))


@pytest.mark.parametrize("heads,kvh,hd", [(4, 2, 64), (8, 2, 128), (8, 8, 64), (16, 2, 128)])
def test_split_decode_b1(eng, torch, oracle, synth, heads, kvh, hd):
    """Past SPARSE_BLOCKS_K blocks: every checked step's selected block set
    equal to select_top_k_blocks' on the same scores; logits within tolerance
    of the restatement (bit-identical weights, reordered additions; from 1024
    tokens on the visiting order differs), then 64 greedy steps with equal
    tokens."""
    mode = 1
    cfg = synth.ModelConfig(dim=256, hidden_dim=512, n_layers=2, n_heads=heads, n_kv_heads=kvh,
                            vocab_size=2048, seq_len=2048, head_dim=hd, rope_theta=1e4)
    model = synth.make_model(cfg, seed=11)
    e = eng.Engine(cfg, attention_mode=mode)
    e.load(model)
    pm = oracle.PortModel(model)
    P = oracle.port()
    toks = synth.prompt(cfg, 1100, seed=4)
    for pos in range(1100):
        check = pos % 100 == 0 or pos >= 1030
        lg, _ = e.step([toks[pos]], [pos], want_logits=check)
        want = pm.forward(int(toks[pos]), pos)
        if not check:
            continue
        assert within(lg[0], want), f"step {pos}"
        if pos >= 1024:
            assert selection_matches(e, cfg, P, pos), f"selection at {pos}"
    tok = P.port_argmax(want, want.size)
    for i in range(64):
        lg, am = e.step([tok], [1100 + i])
        want = pm.forward(tok, 1100 + i)
        assert within(lg[0], want), f"greedy step {i}"
        ref_tok = P.port_argmax(want, want.size)
        assert int(am[0]) == ref_tok, f"greedy token {i}"
        tok = ref_tok
    e.close()


@pytest.mark.parametrize("B", [3, 9])
def test_split_decode_batched(eng, torch, oracle, synth, B):
    """B sequences per step (B = 3: the split attention, 8 CTAs per KV head;
    B = 9: split mode keeps the grouped reference-order attention; both on
    the exact batched chain): every sequence within tolerance of its own
    restatement model past the block-sparse threshold."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=2,
                            vocab_size=2048, seq_len=2048, head_dim=128, rope_theta=5e5)
    model = synth.make_model(cfg, seed=23)
    e = eng.Engine(cfg, max_batch=B, attention_mode=1)
    e.load(model)
    pms = [oracle.PortModel(model) for _ in range(B)]
    prompts = [synth.prompt(cfg, 1060, seed=40 + b) for b in range(B)]
    for t in range(1060):
        check = t % 200 == 0 or t >= 1050
        lg, am = e.step([int(p[t]) for p in prompts], [t] * B, want_logits=check)
        for b in range(B):
            want = pms[b].forward(int(prompts[b][t]), t)
            if check:
                assert within(lg[b], want), f"step {t} sequence {b}"
    e.close()


def test_split_tensor_core_step(eng, torch, oracle, synth):
    """The tensor-core batched step (B >= tensor_min_batch) with the split
    attention, on the tensor-core decode test's model and prompts: 16
    sequences within tolerance of the restatement at every step and every
    greedy token equal, the GPU's token fed back to both for 64 steps."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1408, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=4096, seq_len=512, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=29)
    B = 16
    P = oracle.port()
    e = eng.Engine(cfg, max_batch=B, tensor_min_batch=16, attention_mode=1)
    e.load(model)
    pms = [oracle.PortModel(model) for _ in range(B)]
    prompts = [synth.prompt(cfg, 8, seed=60 + b) for b in range(B)]
    toks = [int(p[0]) for p in prompts]
    for t in range(72):
        lg, am = e.step(toks, [t] * B)
        for b in range(B):
            want = pms[b].forward(toks[b], t)
            assert within(lg[b], want), f"step {t} sequence {b}"
            assert am[b] == P.port_argmax(want, want.size), f"step {t} sequence {b}"
        toks = [int(prompts[b][t + 1]) if t + 1 < 8 else int(am[b]) for b in range(B)]
    e.close()


def test_split_rejects_unsupported_geometry(eng, torch, synth):
    """Three query heads per KV head is outside the split kernels' shapes:
    ec_create refuses instead of running another path."""
    cfg = synth.ModelConfig(dim=384, hidden_dim=512, n_layers=1, n_heads=6, n_kv_heads=2,
                            vocab_size=512, seq_len=256, head_dim=64, rope_theta=1e4)
    with pytest.raises(eng.EngineError):
        eng.Engine(cfg, attention_mode=1)
