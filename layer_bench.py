"""Per-kernel timing of the decode step on a model with the 8B layer shapes
but few layers and a small vocabulary (a small case for profilers: a few
hundred MB on the device).

  python layer_bench.py [--layers 2] [--prompt 2048]
        [--steps 20] [--paged 1] [--vocab 4096] [--batch 1] [--tensor-min-batch 16]

Prints one JSON line: ms per step (graph replay, CUDA events) and the
per-kernel device time from the library's profiling mode.
"""
import argparse
import importlib.util
import json
import os
import sys

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "42-berlin-engine_b200")


def _load(name):
    key = "ec_" + name
    if key in sys.modules:
        return sys.modules[key]
    spec = importlib.util.spec_from_file_location(key, os.path.join(PKG, name + ".py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[key] = mod
    spec.loader.exec_module(mod)
    return mod


def load_device_model(eng, e, src):
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


def main():
    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--paged", type=int, default=1)
    ap.add_argument("--vocab", type=int, default=4096)
    ap.add_argument("--sparse-k", type=int, default=64)
    ap.add_argument("--batch", type=int, default=1, help="sequences per step")
    ap.add_argument("--tensor-min-batch", type=int, default=16)
    ap.add_argument("--attention", type=int, default=0, help="attention_mode (0 reference, 1 split)")
    args = ap.parse_args()
    B = args.batch
    eng, S = _load("engine"), _load("synth")
    base = S.LLAMA3_8B
    cfg = S.ModelConfig(dim=base.dim, hidden_dim=base.hidden_dim, n_layers=args.layers,
                        n_heads=base.n_heads, n_kv_heads=base.n_kv_heads,
                        vocab_size=args.vocab, seq_len=base.seq_len, head_dim=base.head_dim,
                        rope_theta=base.rope_theta)
    tmb = args.tensor_min_batch if B >= args.tensor_min_batch > 0 else 0
    e = eng.Engine(cfg, use_paged_kv=bool(args.paged), sparse_k=args.sparse_k, max_batch=B,
                   tensor_min_batch=tmb, attention_mode=args.attention)
    load_device_model(eng, e, S.DeviceModel(cfg, seed=3, device=0))
    torch.cuda.synchronize()
    toks = [S.prompt(cfg, args.prompt, seed=5 + b) for b in range(B)]
    for p in range(args.prompt):
        _, am = e.step([t[p] for t in toks], [p] * B, want_logits=False)
    tok = torch.tensor([int(a) for a in am], dtype=torch.int32, device="cuda")
    pos = torch.tensor([args.prompt] * B, dtype=torch.int32, device="cuda")
    stream = torch.cuda.ExternalStream(e.stream())
    for _ in range(3):
        e.step_device(tok.data_ptr(), pos.data_ptr(), B, True)
    e.sync()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    for _ in range(args.steps):
        e.step_device(tok.data_ptr(), pos.data_ptr(), B, True)
    ev[1].record(stream)
    e.sync()
    ms = ev[0].elapsed_time(ev[1]) / args.steps
    e.profile(True)
    cur, p = [int(v) for v in tok.cpu()], int(pos[0].item())
    for _ in range(3):
        _, am = e.step(cur, [p] * B, want_logits=False)
        cur, p = [int(a) for a in am], p + 1
    prof = e.profile_read()
    e.profile(False)
    out = {"layers": args.layers, "context": args.prompt, "paged": args.paged, "batch": B,
           "ms_per_step": round(ms, 4),
           "us_per_launch": {k: round(v["ms"] * 1e3 / v["launches"], 2)
                             for k, v in prof.items() if v["launches"]},
           "GBps": {k: round(v["bytes"] / (v["ms"] * 1e-3) / 1e9, 1)
                    for k, v in prof.items() if v["launches"] and v["bytes"]}}
    print(json.dumps(out), flush=True)
    e.close()


if __name__ == "__main__":
    main()
