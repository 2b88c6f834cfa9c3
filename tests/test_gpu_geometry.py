"""Parity at the benchmark's own geometry, against the reference engine.

The bench runs the Llama-3-8B shape (D 4096, 32/8 heads, head_dim 128,
F 14336, RoPE theta 5e5, INT8, paged KV) and the 70B shape (D 8192, 64/8
heads, F 28672, FP8 E4M3, linear KV with LSH top-K 511).  These tests run
two-layer slices of exactly those shapes (vocabulary cut to 8192 rows so
the reference's BF16 copy stays small) through the C ABI and compare every
checked step with ``transformer_forward`` of the reference itself
(oracle/_ref, its BF16 path on weights equal to the INT8 / FP8 weights):

* logits bit-identical at the checked steps of a prompt that takes the
  paged path past SPARSE_BLOCKS_K blocks (block-centroid selection active),
  then 64 greedy steps with identical tokens;
* the selected blocks of the last layer, in the reference's heap order,
  equal to select_top_k_blocks (paged.c:401-495) on the reference's own
  centroids and query;
* FP8 in linear mode: the LSH-routed top-511 path (inference.c:213-423).
"""
import ctypes as C
import os

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


def bits(a):
    return np.asarray(a).view(np.uint32)


class _HostBF16:
    """A config plus host BF16 weights, the form oracle.RefModel takes."""

    def __init__(self, cfg, bf):
        self.cfg, self._bf = cfg, bf

    def bf16_weights(self):
        return self._bf


def _load_device_model(eng, e, src):
    def sink(kind, layer, name, t, s):
        if kind == "emb":
            e.set_weight_device(-1, eng.EC_EMBEDDING, t.data_ptr(), 0)
        elif kind == "norm":
            which = {"attention_norm": eng.EC_ATTN_NORM, "ffn_norm": eng.EC_FFN_NORM,
                     "final_norm": eng.EC_FINAL_NORM}[name]
            e.set_weight_device(layer, which, t.data_ptr(), 0)
        else:
            which = eng.EC_LM_HEAD if layer < 0 else eng.MAT_IDS[name]
            e.set_weight_device(layer, which, t.data_ptr(), s.data_ptr())
    src.generate(sink)


def _slice(synth, base, **over):
    d = base.as_dict()
    d.update(n_layers=2, vocab_size=8192)
    d.update(over)
    return synth.ModelConfig(**d)


def close_enough(got, want):
    """BASELINE's tolerance: max |difference| <= 2e-2 of the logit range."""
    return float(np.abs(got - want).max()) <= TOL * float(want.max() - want.min())


TOL = 2e-2


def _run(eng, torch, ref, synth, cfg, kind, paged, sparse_k, n_prompt, n_greedy, check_every,
         check_from, sel_check=False, mode=0):
    """mode 0: the reference-order path, bit-exact; otherwise the split
    attention: logits within TOL of the range, the same selected block SET,
    equal greedy tokens."""
    src = synth.DeviceModel(cfg, seed=77, device=0, kind=kind)
    e = eng.Engine(cfg, device=0, weight_kind=eng.EC_W_FP8 if kind == "fp8" else eng.EC_W_INT8,
                   use_paged_kv=paged, sparse_k=sparse_k, attention_mode=mode)
    same = (lambda a, b: np.array_equal(bits(a), bits(b))) if mode == 0 else close_enough
    _load_device_model(eng, e, src)
    torch.cuda.synchronize()
    rm = ref.RefModel(_HostBF16(cfg, src.bf16_weights()), use_paged_kv=paged, sparse_k=sparse_k)
    del src
    torch.cuda.empty_cache()
    R = ref.ref()
    P = ref.port()
    toks = synth.prompt(cfg, n_prompt, seed=3)
    hd = cfg.head_dim
    n_sel_checked = 0
    for pos in range(n_prompt):
        check = pos % check_every == 0 or pos >= check_from
        lg, _ = e.step([int(toks[pos])], [pos], want_logits=check)
        want = rm.forward(int(toks[pos]), pos)
        if not check:
            continue
        assert same(lg[0], want), f"prompt step {pos}"
        if sel_check and pos >= 64 * 16 and pos % 8 == 0:
            if mode == 0:
                # select_top_k_blocks over the reference's centroids of the
                # last layer with its query head 0 (score_blocks, paged.c:401-431)
                q = np.ctypeslib.as_array(R.refd_state(rm.h, 2), (hd,)).copy()
                kb = np.zeros(cfg.n_kv_heads * 16 * hd, np.int8)
                vb = np.zeros_like(kb)
                ks = np.zeros(cfg.n_kv_heads * 16, np.float32)
                vs = np.zeros_like(ks)
                cen = np.zeros(hd, np.float32)
                scores = []
                while R.refd_paged_block(rm.h, cfg.n_layers - 1, len(scores), kb, vb, ks, vs,
                                         cen) >= 0:
                    scores.append(P.port_dot_f32(q, cen, hd))
            else:
                # the split path's caches drift from the reference's by
                # rounding: the same selection rule on the engine's own query
                # and centroids
                q = e.state(2)[:hd].copy()
                nb = (pos + 16) // 16
                mb = (cfg.seq_len + 15) // 16
                cens = e.state(9, n=mb * hd)[:nb * hd].reshape(nb, hd)
                scores = [P.port_dot_f32(q, np.ascontiguousarray(cens[i]), hd) for i in range(nb)]
            sc = np.asarray(scores, np.float32)
            sel = np.zeros(70, np.int32)
            ns = P.port_select_blocks(sc, sc.size, 64, sel)
            got = e.state(8, n=80)
            assert int(got[0]) == ns, f"selected count at {pos}"
            g = got[1:1 + ns].astype(np.int32)
            if mode:
                g, want_sel = np.sort(g), np.sort(sel[:ns])
            else:
                want_sel = sel[:ns]
            assert np.array_equal(g, want_sel), f"selection at {pos}"
            n_sel_checked += 1
    # greedy continuation: the GPU picks the token, the reference must agree
    tok = P.port_argmax(want, want.size)
    for i in range(n_greedy):
        pos = n_prompt + i
        lg, am = e.step([tok], [pos])
        want = rm.forward(tok, pos)
        assert same(lg[0], want), f"greedy step {i}"
        ref_tok = P.port_argmax(want, want.size)
        assert int(am[0]) == ref_tok, f"greedy token {i}"
        tok = ref_tok
    e.close()
    return n_sel_checked


@pytest.mark.parametrize("mode", [0, 1])
def test_llama8b_slice_int8_paged(eng, torch, ref, synth, mode):
    """Two layers of the Llama-3-8B shape, INT8, paged KV: 1100 prompt tokens
    (block-sparse past 1024) and 64 greedy steps against the reference:
    bit-exact on the reference-order path with the last layer's block
    selection in heap order; on the split attention within the tolerance,
    the same block set, equal tokens."""
    cfg = _slice(synth, synth.LLAMA3_8B)
    n = _run(eng, torch, ref, synth, cfg, "int8", True, 64, 1100, 64, 50, 1024, sel_check=True,
             mode=mode)
    assert n >= 9


def test_70b_slice_fp8_linear(eng, torch, ref, synth):
    """Two layers of the 70B shape, FP8 E4M3 per tensor, linear BF16 KV with
    the reference's LSH-routed top-511 selection: 600 prompt tokens (sparse
    past 511) and 64 greedy steps, bit-exact against the reference."""
    cfg = _slice(synth, synth.LLAMA_70B, seq_len=4096)
    _run(eng, torch, ref, synth, cfg, "fp8", False, 511, 600, 64, 50, 500)
