"""The final hidden adapter and logit bias (inference.c:583-651) against the
reference itself: transformer_forward of oracle/_ref with the same adapter
(bf16 [dim][dim], x += 16 * (A . x) after the final RMSNorm) and bias
(logits += bias) attached.

Bit-exact on the exact paths (batch 1 and the batched chain); within
BASELINE's 2e-2 of the logit range with equal greedy tokens on the
tensor-core batched step; an all-zero adapter and bias stay switched off
(the reference's zero-initialised tensors change nothing)."""
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


def _setup(synth, seed=5):
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=2048, seq_len=512, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=seed)
    rng = np.random.default_rng(seed)
    adapter = synth.f32_to_bf16(rng.standard_normal((cfg.dim, cfg.dim), dtype=np.float32)
                                * np.float32(0.002))
    bias = (rng.standard_normal(cfg.vocab_size, dtype=np.float32) * np.float32(0.5))
    return cfg, model, adapter, bias


@pytest.mark.parametrize("B,tmb", [(1, 0), (3, 0), (16, 16)])
def test_adapter_and_bias_match_reference(eng, torch, ref, synth, B, tmb):
    cfg, model, adapter, bias = _setup(synth)
    e = eng.Engine(cfg, max_batch=B, tensor_min_batch=tmb)
    e.load(model)
    e.set_final(adapter, bias)
    rms = []
    for _ in range(B):
        m = ref.RefModel(model, use_paged_kv=True, sparse_k=64)
        m.set_final(adapter, bias)
        rms.append(m)
    prompts = [synth.prompt(cfg, 40, seed=30 + b) for b in range(B)]
    toks = [int(p[0]) for p in prompts]
    P = ref.port()
    for t in range(48):
        lg, am = e.step(toks, [t] * B)
        for b in range(B):
            want = rms[b].forward(toks[b], t)
            if tmb:
                d = float(np.abs(lg[b] - want).max())
                assert d <= 2e-2 * float(want.max() - want.min()), f"step {t} sequence {b}"
            else:
                assert np.array_equal(lg[b].view(np.uint32), want.view(np.uint32)), \
                    f"step {t} sequence {b}"
            assert int(am[b]) == P.port_argmax(want, want.size), f"token {t} sequence {b}"
        toks = [int(prompts[b][t + 1]) if t + 1 < 40 else int(am[b]) for b in range(B)]
    e.close()


def test_zero_adapter_and_bias_stay_off(eng, torch, ref, synth):
    cfg, model, adapter, bias = _setup(synth, seed=6)
    e = eng.Engine(cfg)
    e.load(model)
    n0 = e.launches_per_step(1)
    e.set_final(np.zeros_like(adapter), np.zeros_like(bias))
    assert e.launches_per_step(1) == n0
    m = ref.RefModel(model, use_paged_kv=True, sparse_k=64)
    for p, t in enumerate(synth.prompt(cfg, 8, seed=2)):
        lg, _ = e.step([int(t)], [p])
        assert np.array_equal(lg[0].view(np.uint32), m.forward(int(t), p).view(np.uint32))
    e.set_final(adapter, bias)
    assert e.launches_per_step(1) == n0 + 4  # final norm, adapter, LM head, bias
    e.close()


def _fmix64(k):
    m = (1 << 64) - 1
    k ^= k >> 33
    k = (k * 0xff51afd7ed558ccd) & m
    k ^= k >> 33
    k = (k * 0xc4ceb9fe1a85ec53) & m
    k ^= k >> 33
    return k


def _context_table(cfg, prompts, size=97, seed=3):
    """A context bias table as the reference's training fills it: for a
    previous token key, linear probing from fmix64(key) % size to the first
    empty slot.  Keys: token 1 (position 0's key) and previous tokens of the
    prompts, enough of them to make probe chains collide."""
    rng = np.random.default_rng(seed)
    keys = np.zeros(size, np.uint64)
    tokens = np.zeros(size, np.int32)
    biases = np.zeros(size, np.float32)
    wanted = [1] + sorted({int(t) for p in prompts for t in p[:30]})[:40]
    for k in wanted:
        if k == 0:
            continue
        i = _fmix64(k) % size
        while keys[i] != 0:
            i = (i + 1) % size
        keys[i] = k
        tokens[i] = int(rng.integers(0, cfg.vocab_size))
        biases[i] = np.float32(rng.uniform(2.0, 9.0))
    return keys, tokens, biases


@pytest.mark.parametrize("B", [1, 3])
def test_context_bias_matches_reference(eng, torch, ref, synth, B):
    """The context-aware bias cache (inference.c:657-693): every step's logits
    bit-identical to the reference with the same table attached, including
    keys whose slots collide and greedy tokens the biases change; then a
    prompt prefilled as rows of one sequence."""
    cfg, model, _, _ = _setup(synth, seed=8)
    prompts = [synth.prompt(cfg, 40, seed=50 + b) for b in range(B)]
    keys, tokens, biases = _context_table(cfg, prompts)
    e = eng.Engine(cfg, max_batch=max(B, 8))
    e.load(model)
    n0 = e.launches_per_step(B)
    e.set_context_bias(keys, tokens, biases)
    assert e.launches_per_step(B) == n0 + 1
    rms = []
    for _ in range(B):
        m = ref.RefModel(model, use_paged_kv=True, sparse_k=64)
        m.set_context_bias(keys, tokens, biases)
        rms.append(m)
    toks = [int(p[0]) for p in prompts]
    P = ref.port()
    hits = 0
    for t in range(48):
        lg, am = e.step(toks, [t] * B)
        for b in range(B):
            want = rms[b].forward(toks[b], t)
            assert np.array_equal(lg[b].view(np.uint32), want.view(np.uint32)), \
                f"step {t} sequence {b}"
            assert int(am[b]) == P.port_argmax(want, want.size)
            hits += int(int(am[b]) in set(tokens[keys != 0].tolist()))
        toks = [int(prompts[b][t + 1]) if t + 1 < 40 else int(am[b]) for b in range(B)]
    assert hits > 0, "the biases reached a greedy token"
    # prefill: rows of one sequence read their predecessors' tokens
    e.reset(0)
    m = ref.RefModel(model, use_paged_kv=True, sparse_k=64)
    m.set_context_bias(keys, tokens, biases)
    lg, tok = e.prefill(0, prompts[0][:21])
    for p, t in enumerate(prompts[0][:21]):
        want = m.forward(int(t), p)
    assert np.array_equal(lg.view(np.uint32), want.view(np.uint32))
    e.close()
