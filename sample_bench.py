"""Device sampling (ec_op_sample_top_p: repetition penalty, UNK block,
softmax at temperature, top-p nucleus and the draw) through the C ABI, on
Llama-3 vocabulary rows (128256 logits, N(0, 3) values, a 512-token history
per row), temperature 0.7 and top-p 0.9 as the reference server uses
(worker.c:425-426).

Per batch size: device time per call (CUDA events on the launching stream,
the logits restored and L2 flushed between calls, not timed), and the bytes
of logits the call must read once (rows x vocab x 4) over that time.  Also
the device-to-host copy of the logits into pinned memory (513 KB per row),
which the reference's host-side sampling needs and device sampling removes.

  python sample_bench.py [--rows 1,8,64] [--iters 20]
"""
import argparse
import ctypes as C
import importlib.util
import json
import os
import sys

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
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", default="1,8,64")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--vocab", type=int, default=128256)
    a = ap.parse_args()
    import torch
    eng = _load("engine")
    L = eng.lib()
    n = a.vocab
    rng = np.random.default_rng(1)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    out = []
    for rows in [int(x) for x in a.rows.split(",")]:
        lg0 = torch.from_numpy((3.0 * rng.standard_normal((rows, n))).astype(np.float32)).cuda()
        lg = lg0.clone()
        hist = torch.from_numpy(rng.integers(0, n, (rows, 512)).astype(np.int32)).cuda()
        hl = torch.full((rows,), 512, dtype=torch.int32, device="cuda")
        r = torch.from_numpy(rng.uniform(0, 1, rows).astype(np.float32)).cuda()
        tok = torch.zeros(rows, dtype=torch.int32, device="cuda")
        s = torch.cuda.current_stream()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ts = []
        for it in range(a.iters + 3):
            lg.copy_(lg0)
            flush.zero_()
            ev0.record(s)
            eng.check(L.ec_op_sample_top_p(lg.data_ptr(), n, rows, hist.data_ptr(),
                                           hl.data_ptr(), 512, 0.7, 0.9, 1.2, 1, r.data_ptr(),
                                           tok.data_ptr(), C.c_void_p(s.cuda_stream)))
            ev1.record(s)
            torch.cuda.synchronize()
            if it >= 3:
                ts.append(ev0.elapsed_time(ev1))
        ms = float(np.median(ts))
        rec = dict(rows=rows, vocab=n, us_per_call=ms * 1e3, us_per_row=ms * 1e3 / rows,
                   logits_gbs=rows * n * 4 / (ms * 1e-3) / 1e9)
        # what device sampling removes: the logits' device-to-host copy
        h = torch.empty((rows, n), dtype=torch.float32, pin_memory=True)
        ts = []
        for it in range(a.iters + 3):
            ev0.record(s)
            h.copy_(lg0, non_blocking=True)
            ev1.record(s)
            torch.cuda.synchronize()
            if it >= 3:
                ts.append(ev0.elapsed_time(ev1))
        rec["d2h_us_per_call"] = float(np.median(ts)) * 1e3
        out.append(rec)
        print(json.dumps(rec), flush=True)
    return out


if __name__ == "__main__":
    main()
