"""Quantised GEMV sweep at batch 1, 8, 64, 512 through the
packed-layout entry points (ec_op_gemv_packed, ec_op_gemv_packed_batch).

For each (N, K) in {(4096,4096), (14336,4096), (4096,14336), (128256,4096)} and
weight kind INT8 (per-row fp32 scale) / FP8-E4M3 (per-tensor scale): time the
kernel with CUDA events on the launching stream, rotating over enough weight
copies that every launch reads its matrix from HBM (> 126 MB of L2), and report
GB/s of algorithmic bytes (N*K weights + scales + 4K x + 4N y) against the
measured HBM peak.  One JSON line per case.

  python gemv_sweep.py [--kinds int8,fp8] [--shapes 4096x4096,...]
        [--iters 50] [--warmup 5]
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


SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]


def run_case(torch, eng, kind, n, k, args, peak):
    L = eng.lib()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev)
    wk = {"int8": eng.EC_W_INT8, "fp8": eng.EC_W_FP8, "bf16": eng.EC_W_BF16}[kind]
    es = 2 if kind == "bf16" else 1
    wbytes = n * k * es
    copies = max(1, min(64, int(args.l2_bytes // wbytes) + 1))
    g = torch.Generator(device=dev)
    g.manual_seed(n + k)
    if kind == "int8":
        ws = [torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8)
              for _ in range(copies)]
        sc = torch.rand(n, generator=g, device=dev) * 1e-3 + 1e-4
    elif kind == "fp8":
        ws = [torch.randn((n, k), generator=g, device=dev).to(torch.float8_e4m3fn)
              .view(torch.uint8) for _ in range(copies)]
        sc = torch.full((1,), 0.01, device=dev)
    else:
        ws = [torch.randn((n, k), generator=g, device=dev).to(torch.bfloat16)
              for _ in range(copies)]
        sc = None
    nb = args.batch_now
    x = torch.randn((nb, k), generator=g, device=dev)
    y = torch.empty((nb, n), device=dev)
    sptr = sc.data_ptr() if sc is not None else None

    op = L.ec_op_gemv
    if args.layout == "tc":
        # tensor-core layout (INT8 only): ec_op_gemm_tc = digit planes +
        # tcgen05 GEMM + combine, synchronised at the end of every call
        pk = []
        for w_ in ws:
            dst = torch.zeros(L.ec_gemm_tc_bytes(n, k), dtype=torch.uint8, device=dev)
            eng.check(L.ec_gemm_tc_pack(w_.data_ptr(), dst.data_ptr(), n, k, stream.cuda_stream))
            pk.append(dst)
        ws = pk
    elif args.layout == "packed" and kind != "bf16":
        # the decode step's layout: repack each copy once, outside the timing
        op = L.ec_op_gemv_packed
        pk = []
        for w_ in ws:
            dst = torch.empty(L.ec_gemv_packed_bytes(n, k), dtype=torch.uint8, device=dev)
            eng.check(L.ec_gemv_pack(w_.data_ptr(), dst.data_ptr(), n, k, stream.cuda_stream))
            pk.append(dst)
        ws = pk

    def run(i):
        if args.layout == "tc":
            eng.check(L.ec_op_gemm_tc(ws[i % copies].data_ptr(), sptr, x.data_ptr(), y.data_ptr(),
                                      n, k, nb, stream.cuda_stream))
        elif nb == 1:
            eng.check(op(wk, ws[i % copies].data_ptr(), sptr, x.data_ptr(), y.data_ptr(),
                         n, k, stream.cuda_stream))
        else:
            eng.check(L.ec_op_gemv_packed_batch(wk, ws[i % copies].data_ptr(), sptr, x.data_ptr(),
                                                y.data_ptr(), n, k, nb, stream.cuda_stream))

    for i in range(args.warmup):
        run(i)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    for i in range(args.iters):
        run(i)
    ev[1].record(stream)
    torch.cuda.synchronize()
    us = ev[0].elapsed_time(ev[1]) * 1e3 / args.iters
    algo = wbytes + (4 * n if kind == "int8" else 4) + 4 * k * nb + 4 * n * nb
    gbs = algo / (us * 1e-6) / 1e9
    return {"kernel": "gemv", "layout": args.layout, "kind": kind, "N": n, "K": k, "batch": nb,
            "us": round(us, 2), "TFLOPs": round(2.0 * nb * n * k / (us * 1e-6) / 1e12, 2),
            "algo_bytes": algo, "GBps": round(gbs, 1), "frac_of_measured_peak": round(gbs / peak, 4),
            "l2": f"{copies} rotating weight copies"}


def main():
    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--kinds", default="int8,fp8")
    ap.add_argument("--shapes", default=",".join(f"{n}x{k}" for n, k in SHAPES))
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", default="1", help="activation vectors per call, e.g. 1,8,64,512")
    ap.add_argument("--layout", default="packed", choices=["packed", "rowmajor", "tc"],
                    help="packed: the decode step's kernel; rowmajor: ec_op_gemv; "
                         "tc: the tensor-core GEMM (INT8)")
    ap.add_argument("--l2-bytes", type=float, default=512e6, help="bytes of weight copies rotated")
    args = ap.parse_args()
    eng = _load("engine")
    peak = 6650.0
    pf = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pf):
        peak = float(json.load(open(pf))["hbm_gbs"])
    for kind in args.kinds.split(","):
        for shp in args.shapes.split(","):
            n, k = (int(v) for v in shp.split("x"))
            for nb in (int(v) for v in args.batch.split(",")):
                if args.layout == "tc" and kind != "int8":
                    continue
                if nb > 1 and (args.layout == "rowmajor" or kind == "bf16"):
                    continue
                args.batch_now = nb
                print(json.dumps(run_case(torch, eng, kind, n, k, args, peak)), flush=True)
                torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
