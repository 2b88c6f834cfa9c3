"""Speculative decoding (speculate.c:93-258): a draft engine proposes greedy
tokens, the target verifies them in one ec_verify pass (its rows are the
ec_prefill path, bit-identical to decode steps) and keeps the accepted
prefix plus its correction.  The tokens must be exactly the target's own
greedy decode -- with a draft that always agrees (the target's own weights)
and with one that mostly disagrees (another model)."""
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


@pytest.mark.parametrize("same_draft", [True, False])
def test_speculative_tokens_equal_greedy(eng, torch, synth, same_draft):
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=2048, seq_len=1024, head_dim=64, rope_theta=1e4)
    target_model = synth.make_model(cfg, seed=51)
    draft_model = target_model if same_draft else synth.make_model(cfg, seed=52)
    n_draft, n_prompt, n_gen = 5, 90, 60
    prompt = [int(t) for t in synth.prompt(cfg, n_prompt, seed=4)]
    # the target alone, one greedy step at a time
    ref = eng.Engine(cfg, sparse_blocks_k=4)
    ref.load(target_model)
    for p, t in enumerate(prompt):
        _, am = ref.step([t], [p], want_logits=False)
    want = [int(am[0])]
    for p in range(n_prompt, n_prompt + n_gen):
        _, am = ref.step([want[-1]], [p], want_logits=False)
        want.append(int(am[0]))
    ref.close()
    # draft + verify bursts
    target = eng.Engine(cfg, max_batch=n_draft, sparse_blocks_k=4)
    draft = eng.Engine(cfg, sparse_blocks_k=4)
    target.load(target_model)
    draft.load(draft_model)
    _, tok = target.prefill(0, prompt)
    for p, t in enumerate(prompt):
        draft.step([t], [p], want_logits=False)
    got, pos, bursts = [tok], n_prompt, 0
    while len(got) < len(want):
        out = eng.speculate(target, draft, got[-1], pos, n_draft)
        got += out
        pos += len(out)
        bursts += 1
    got = got[:len(want)]
    assert got == want
    if same_draft:
        assert bursts <= (n_gen + n_draft - 1) // n_draft + 1  # every draft accepted
    target.close()
    draft.close()


def test_verify_matches_decode_steps(eng, torch, synth):
    """ec_verify's greedy token after each row == the decode step's."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=2048, seq_len=512, head_dim=64, rope_theta=1e4)
    model = synth.make_model(cfg, seed=53)
    toks = [int(t) for t in synth.prompt(cfg, 40, seed=6)]
    a = eng.Engine(cfg, max_batch=8, sparse_blocks_k=4)
    b = eng.Engine(cfg, sparse_blocks_k=4)
    a.load(model)
    b.load(model)
    got = a.verify(0, toks, 0)
    want = []
    for p, t in enumerate(toks):
        _, am = b.step([t], [p], want_logits=False)
        want.append(int(am[0]))
    assert [int(x) for x in got] == want
    a.close()
    b.close()
