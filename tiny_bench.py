"""The tiny correctness configuration's decode rate (D=512, 8 layers, 8 heads
of 64, F=1408, V=32000; INT8 weights with power-of-two row scales), batch 1:
a 64-token prompt, then 128 greedy tokens.  Paged KV (block selection) and
linear KV (LSH candidates, top-32).  The 42 MB of weights stay in L2, so the
step is bound by launch and synchronisation latency, not by HBM: tok/s only.

Device time per greedy step: CUDA events on the context's stream around the
128 steps (each step's graph replay feeds its own argmax back as the next
token, as the decode loop does).

  python tiny_bench.py
"""
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


def main():
    import torch
    eng, S = _load("engine"), _load("synth")
    model = S.make_model(S.TINY, seed=7)
    for mode, kw in (("paged", dict(use_paged_kv=True, sparse_k=64)),
                     ("linear", dict(use_paged_kv=False, sparse_k=32))):
        e = eng.Engine(S.TINY, **kw)
        e.load(model)
        prompt = [int(t) for t in S.prompt(S.TINY, 64, seed=3)]
        for p, t in enumerate(prompt):
            _, am = e.step([t], [p], want_logits=False)
        tok = torch.tensor([int(am[0])], dtype=torch.int32, device="cuda")
        pos = torch.tensor([64], dtype=torch.int32, device="cuda")
        stream = torch.cuda.ExternalStream(e.stream())
        for _ in range(3):  # warm-up (graph capture), positions 64..66
            e.step_device(tok.data_ptr(), pos.data_ptr(), 1, True)
        e.sync()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        ev[0].record(stream)
        n = 128
        for _ in range(n):
            e.step_device(tok.data_ptr(), pos.data_ptr(), 1, True)
        ev[1].record(stream)
        e.sync()
        ms = ev[0].elapsed_time(ev[1]) / n
        print(json.dumps({"config": "tiny", "kv": mode, "batch": 1, "prompt": 64,
                          "greedy_tokens": n, "ms_per_step": round(ms, 4),
                          "tok_s": round(1e3 / ms, 1)}), flush=True)
        e.close()


if __name__ == "__main__":
    main()
