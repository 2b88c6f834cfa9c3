"""Quantise-at-load: the reference's weights are BF16 (loader_parse.c:35-49);
ec_set_weight_bf16 (and ec_transformer_set_tensor without scales) quantise
them on the device to the context's INT8 per-row or FP8 per-tensor format.

The rule is restated in numpy (synth.quant_int8_rows(pow2=False) and
synth.quant_fp8_tensor on the BF16 values); a model loaded from BF16 on the
device must decode bit-identically to the restatement running on the
numpy-quantised weights -- any differing code or scale would show in the
logits."""
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


def _bf16_model(synth, cfg, seed):
    """BF16 weights of a random model, and the synth.Model whose matrices are
    those BF16 values quantised by the numpy restatement."""
    rng = np.random.default_rng(seed)
    shapes = synth.mat_shapes(cfg)

    def bf(shape, sd=0.02):
        return synth.f32_to_bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(sd))

    def norm():
        return synth.f32_to_bf16(1.0 + 0.1 * rng.standard_normal(cfg.dim, dtype=np.float32))

    out = {"emb": bf((cfg.vocab_size, cfg.dim)), "layers": []}
    for _ in range(cfg.n_layers):
        lw = {n: bf(shapes[n]) for n in synth.MATS}
        lw["attention_norm"] = norm()
        lw["ffn_norm"] = norm()
        out["layers"].append(lw)
    out["final_norm"] = norm()
    out["lm"] = bf((cfg.vocab_size, cfg.dim))
    return out


def _quantised(synth, cfg, bfw, kind):
    def q(m):
        w = synth.bf16_to_f32(m)
        return synth.quant_int8_rows(w, pow2=False) if kind == "int8" else synth.quant_fp8_tensor(w)
    layers = []
    for lw in bfw["layers"]:
        d = {n: q(lw[n]) for n in synth.MATS}
        d["attention_norm"] = lw["attention_norm"]
        d["ffn_norm"] = lw["ffn_norm"]
        layers.append(d)
    return synth.Model(cfg, kind, bfw["emb"], bfw["final_norm"], q(bfw["lm"]), layers, 0)


@pytest.mark.parametrize("kind", ["int8", "fp8"])
def test_bf16_load_matches_restated_quantisation(eng, torch, oracle, synth, kind):
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=2048, seq_len=256, head_dim=64, rope_theta=1e4)
    bfw = _bf16_model(synth, cfg, seed=17)
    model = _quantised(synth, cfg, bfw, kind)
    e = eng.Engine(cfg, weight_kind=eng.EC_W_INT8 if kind == "int8" else eng.EC_W_FP8)
    e.load_bf16(bfw)
    pm = oracle.PortModel(model)
    for p, t in enumerate(synth.prompt(cfg, 12, seed=8)):
        lg, _ = e.step([int(t)], [p])
        want = pm.forward(int(t), p)
        assert np.array_equal(lg[0].view(np.uint32), want.view(np.uint32)), f"step {p}"
    e.close()


def test_host_transformer_quantises_bf16_tensors(eng, torch, oracle, synth):
    """ec_transformer_set_tensor with scales == NULL: the reference's BF16
    tensors by their HuggingFace names."""
    cfg = synth.ModelConfig(dim=512, hidden_dim=1024, n_layers=2, n_heads=8, n_kv_heads=4,
                            vocab_size=2048, seq_len=256, head_dim=64, rope_theta=1e4)
    bfw = _bf16_model(synth, cfg, seed=19)
    model = _quantised(synth, cfg, bfw, "int8")
    t = eng.HostTransformer(cfg)
    import ctypes as C
    L = eng.lib()
    hf = {"wq": "self_attn.q_proj", "wk": "self_attn.k_proj", "wv": "self_attn.v_proj",
          "wo": "self_attn.o_proj", "w1": "mlp.gate_proj", "w2": "mlp.down_proj",
          "w3": "mlp.up_proj"}
    for i, lw in enumerate(bfw["layers"]):
        for n, hn in hf.items():
            eng.check(L.ec_transformer_set_tensor(C.byref(t.t), f"model.layers.{i}.{hn}.weight".encode(),
                                                  eng._ptr(lw[n]), None))
        eng.check(L.ec_transformer_set_tensor(C.byref(t.t), f"model.layers.{i}.input_layernorm.weight".encode(),
                                              eng._ptr(lw["attention_norm"]), None))
        eng.check(L.ec_transformer_set_tensor(C.byref(t.t),
                                              f"model.layers.{i}.post_attention_layernorm.weight".encode(),
                                              eng._ptr(lw["ffn_norm"]), None))
    eng.check(L.ec_transformer_set_tensor(C.byref(t.t), b"model.embed_tokens.weight", eng._ptr(bfw["emb"]), None))
    eng.check(L.ec_transformer_set_tensor(C.byref(t.t), b"model.norm.weight", eng._ptr(bfw["final_norm"]), None))
    eng.check(L.ec_transformer_set_tensor(C.byref(t.t), b"lm_head.weight", eng._ptr(bfw["lm"]), None))
    pm = oracle.PortModel(model)
    for p, tok in enumerate(synth.prompt(cfg, 8, seed=9)):
        lg = t.forward(int(tok), p)
        want = pm.forward(int(tok), p)
        assert np.array_equal(np.asarray(lg).view(np.uint32), want.view(np.uint32)), f"step {p}"
    t.close()
