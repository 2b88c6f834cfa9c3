"""Isolated LSH sparse attention through the C ABI.

32 query heads, 8 KV heads, head_dim 128; K/V drawn N(0,1) and rounded to
BF16 (exactly representable in FP16 and BF16); per-key codes (unit 1) from
8 tables x 12-bit Gaussian projections of KV head 0; top-K 256 positions
(plus the reference's 128-position window as candidates); 64 planted keys per
query set to (that query's head of the group) + N(0, 0.1) at random earlier
positions, so recall = |attended & planted| / 64 is checkable.  Contexts 4k,
32k, 128k; 1 and 32 queries per call (queries share the cache).

Per configuration: device time per call (CUDA events on the launching
stream, L2 flushed between calls), queries/s, recall, and algorithmic bytes
per query over time: code reads (tables x 4 bytes per unit) + candidate K
reads (candidates x KV x hd x 2) + selected K and V (2 x top_k x KV x hd x 2).

  python lsh_attention_bench.py [--tokens 4096,32768,131072]
        [--queries 1,32] [--iters 10] [--cpu]   # --cpu: the restatement on one query
"""
import argparse
import ctypes as C
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


H, KV, HD, TABLES, BITS, TOP_K, WINDOW, RADIUS, MAX_CAND = 32, 8, 128, 8, 12, 256, 128, 4, 4096


def make_case(torch, T, Q, seed):
    """Device K/V [T][KV][HD] bf16 and queries [Q][H][HD]; planted positions."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    k = torch.randn((T, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn((T, KV, HD), generator=g, device="cuda").to(torch.bfloat16)
    base = torch.randn((Q, 1, HD), generator=g, device="cuda")
    q = (base + 0.1 * torch.randn((Q, H, HD), generator=g, device="cuda")).float()
    rng = np.random.default_rng(seed)
    pos = rng.choice(T - WINDOW, size=(Q, 64), replace=False)  # distinct over all queries
    grp = H // KV
    for i in range(Q):
        p = torch.from_numpy(pos[i]).cuda()
        heads = q[i, ::grp, :]  # [KV][HD]: each group's first query head
        k[p] = (heads[None] + 0.1 * torch.randn((64, KV, HD), generator=g, device="cuda")).to(
            torch.bfloat16)
    return k.contiguous(), v.contiguous(), q.contiguous(), pos


def main():
    import torch
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="4096,32768,131072")
    ap.add_argument("--queries", default="1,32")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--cpu", action="store_true", help="also time the restatement (one query)")
    ap.add_argument("--paged", action="store_true",
                    help="the cache as 16-token blocks under a shuffled page table")
    args = ap.parse_args()
    eng = _load("engine")
    L = eng.lib()
    peak = 6650.0
    pf = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pf):
        peak = float(json.load(open(pf))["hbm_gbs"])
    flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    for T in (int(x) for x in args.tokens.split(",")):
        for Q in (int(x) for x in args.queries.split(",")):
            k, v, q, planted = make_case(torch, T, Q, seed=T + Q)
            cfg = eng.LshAttnConfig(H, KV, HD, T, TABLES, BITS, 1, RADIUS, MAX_CAND, WINDOW, TOP_K, Q)
            h = C.c_void_p()
            eng.check(L.ec_lsh_attn_create(C.byref(cfg), 0, C.byref(h)))
            if args.paged:
                # blocks of 16 positions stored in a shuffled physical order
                nblk = T // 16
                pt = torch.randperm(nblk, device="cuda").to(torch.int32)
                kb = torch.empty_like(k).view(nblk, 16, KV, HD)
                vb = torch.empty_like(v).view(nblk, 16, KV, HD)
                kb[pt.long()] = k.view(nblk, 16, KV, HD)
                vb[pt.long()] = v.view(nblk, 16, KV, HD)
                torch.cuda.synchronize()
            t0 = time.perf_counter()
            if args.paged:
                eng.check(L.ec_lsh_attn_build_paged(h, kb.data_ptr(), vb.data_ptr(), pt.data_ptr(),
                                                    T, None))
            else:
                eng.check(L.ec_lsh_attn_build(h, k.data_ptr(), v.data_ptr(), T, None))
            build_s = time.perf_counter() - t0
            out = torch.empty((Q, H, HD), device="cuda")
            sel = torch.empty((Q, TOP_K), dtype=torch.int32, device="cuda")
            ns = torch.empty(Q, dtype=torch.int32, device="cuda")

            def call():
                eng.check(L.ec_lsh_attn_query(h, q.data_ptr(), Q, out.data_ptr(), sel.data_ptr(),
                                              ns.data_ptr(), None))
            for _ in range(3):
                call()
            torch.cuda.synchronize()
            times = []
            for _ in range(args.iters):
                flush.fill_(1)
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                call()
                b.record()
                torch.cuda.synchronize()
                times.append(a.elapsed_time(b))
            ms = float(np.median(times))
            stats = np.zeros(2 * Q, np.int32)
            eng.check(L.ec_lsh_attn_read(h, 2, stats.ctypes.data, stats.size))
            selh, nsh = sel.cpu().numpy(), ns.cpu().numpy()
            recall = float(np.mean([len(set(planted[i]) & set(selh[i, :nsh[i]].tolist())) / 64.0
                                    for i in range(Q)]))
            ncand = stats[1::2].astype(np.float64)
            algo = (TABLES * 4 * T + ncand * KV * HD * 2 + 2 * TOP_K * KV * HD * 2).sum()
            line = {"config": "lsh_attention", "cache": "paged" if args.paged else "linear",
                    "tokens": T, "queries": Q, "ms": round(ms, 4),
                    "queries_per_s": round(Q / (ms * 1e-3), 1), "recall": round(recall, 4),
                    "units_found_mean": float(stats[0::2].mean()),
                    "candidates_mean": float(ncand.mean()),
                    "GBps": round(algo / (ms * 1e-3) / 1e9, 1),
                    "frac_of_measured_peak": round(algo / (ms * 1e-3) / 1e9 / peak, 4),
                    "index_build_s": round(build_s, 3)}
            if args.cpu and Q == 1:
                sys.path.insert(0, os.path.join(ROOT, "oracle"))
                import oracle  # the restatement, timed as the CPU baseline
                P = oracle.port()
                kh, vh, qh = (x.cpu() for x in (k, v, q))
                ku = kh.view(torch.int16).numpy().view(np.uint16).reshape(-1)
                vu = vh.view(torch.int16).numpy().view(np.uint16).reshape(-1)
                lsh = P.port_lsh_create(TABLES, BITS, HD, 1, T + 1, RADIUS, 42)
                k0 = (ku.reshape(T, KV, HD)[:, 0, :].astype(np.uint32) << 16).view(np.float32)
                for t in range(T):
                    P.port_lsh_update(lsh, np.ascontiguousarray(k0[t]), t)
                ws, wo = np.zeros(T, np.int32), np.zeros(H * HD, np.float32)
                t0 = time.perf_counter()
                P.port_lsh_attend(lsh, ku, vu, T, np.ascontiguousarray(qh.numpy().reshape(-1)), H,
                                  KV, HD, WINDOW, MAX_CAND, TOP_K, ws, wo)
                line["cpu_query_ms"] = round((time.perf_counter() - t0) * 1e3, 3)
                line["cpu_cores"] = 1
                P.port_lsh_free(lsh)
            print(json.dumps(line), flush=True)
            L.ec_lsh_attn_destroy(h)
            del k, v, q
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
