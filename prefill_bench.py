"""Prompt prefill through ec_prefill (exact chain, and tensor cores with
tensor_min_batch 16) against token-by-token decode.

Llama-3-8B shape, INT8, paged KV: a P-token random prompt for sequence 0 run
(1) by ec_prefill with max_batch rows per weight pass (bit-identical to
decode), and (2) one token per ec_decode_step.  Prints one JSON line with
tokens/s of each and the check that the last logits agree bit for bit.

  python prefill_bench.py [--prompt 2048] [--rows 64]
"""
import argparse
import importlib.util
import json
import os
import sys
import time

import numpy as np

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
    ap = argparse.ArgumentParser()
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--rows", type=int, default=64, help="max_batch: rows per weight pass")
    args = ap.parse_args()
    eng, S = _load("engine"), _load("synth")
    import layer_bench as lb
    cfg = S.LLAMA3_8B
    prompt = [int(t) for t in S.prompt(cfg, args.prompt, seed=11)]
    out = {"workload": "llama3-8b-shape int8 prompt prefill", "prompt": args.prompt,
           "rows_per_pass": args.rows}
    res = {}
    for mode in ("prefill", "prefill_tc", "decode"):
        rows = args.rows if mode != "decode" else 1
        e = eng.Engine(cfg, max_batch=rows, tensor_min_batch=16 if mode == "prefill_tc" else 0)
        lb.load_device_model(eng, e, S.DeviceModel(cfg, seed=3, device=0))
        torch.cuda.synchronize()
        if mode != "decode":
            e.prefill(0, prompt[:64])  # warm-up (kernels, allocator)
            e.reset(0)
            t0 = time.perf_counter()
            lg, _ = e.prefill(0, prompt)
        else:
            for p in range(8):
                e.step([prompt[p]], [p], want_logits=False)
            e.reset(0)
            t0 = time.perf_counter()
            for p, t in enumerate(prompt):
                lg, _ = e.step([t], [p], want_logits=p == len(prompt) - 1)
            lg = lg[0]
        dt = time.perf_counter() - t0
        res[mode] = lg
        out[f"{mode}_tok_s"] = round(args.prompt / dt, 1)
        out[f"{mode}_s"] = round(dt, 3)
        e.close()
        del e
        torch.cuda.empty_cache()
    out["last_logits_bit_identical"] = bool(
        np.array_equal(res["prefill"].view(np.uint32), res["decode"].view(np.uint32)))
    d = res["decode"]
    out["tc_max_diff_of_range"] = float(np.abs(res["prefill_tc"] - d).max() / (d.max() - d.min()))
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
