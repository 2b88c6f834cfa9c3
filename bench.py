"""Decode throughput of the B200 hot path (BASELINE.json metric: decode tok/s).

Workload: Llama-3-8B-shaped random-init decoder, INT8
per-channel weights (power-of-two scales), paged INT8 KV cache (the
reference's default mode), a 2048-token random prompt already in the cache,
then greedy decode.  One step = one decode token of every sequence.

The JSON line's headline is batch 1 per GPU; `dp_b64` in the same line times
64 sequences per GPU (config 4's batch split data-parallel: global batch
64 x N) on the tensor-core path of the same engine.  `--attention` picks the
paged attention: `split` (default; the reference's block set and softmax
weights, additions regrouped over a cluster of CTAs) or `reference` (the
reference's sequential order, bit-identical logits).  Multi-GPU: one process
per GPU, independent sequences (weak scaling, no collective on the data
path); value = tokens of all ranks / max-over-ranks time.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

`--impl reference` times the reference engine's own CPU decode
(oracle/_ref, transformer_forward over BF16 weights equal to the INT8
weights) on the host cores at the same context, rank 0 only.
"""
import argparse
import ctypes as C
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import threading
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


METRIC = "decode tok/s (Llama-3-8B-shaped INT8, b=1 per GPU, 2k context)"
METRIC_B = "decode tok/s (Llama-3-8B-shaped INT8, b={} per GPU, 2k context)"
METRIC_70B = "decode tok/s (70B-shaped FP8 per-tensor, b={} per GPU, {} context, LSH top-{})"
METRIC_70B_TP = ("decode tok/s (70B-shaped FP8 per-tensor, b={}, tensor-parallel over {} GPUs, {} "
                 "context, LSH top-{})")
PROMPT = 2048
# --attention: the paged decode attention (engine_cuda.h attention_mode)
ATTN_MODES = {"reference": 0, "split": 1}
SEED = 1234


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class Clocks:
    """nvidia-smi sampling during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    return _load("dp").rank_env()


_JSON_FD = None  # the process's original stdout; everything else goes to stderr


def emit(line):
    """The bench's one JSON line, on the original stdout."""
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


class _StdoutToStderr:
    """Send file descriptor 1 to stderr while the reference's C code runs (it
    prints its own progress lines), so stdout carries only the JSON line."""

    def __enter__(self):
        sys.stdout.flush()
        self._saved = os.dup(1)
        os.dup2(2, 1)
        return self

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self._saved, 1)
        os.close(self._saved)
        return False


def cpu_baseline(cfg, model_src, n_prompt, steps, warmup, threads):
    """The reference's transformer_forward on the host (oracle/_ref), or the
    C restatement when the reference was not built here."""
    with _StdoutToStderr():
        return _cpu_baseline(cfg, model_src, n_prompt, steps, warmup, threads)


def _cpu_baseline(cfg, model_src, context, steps, warmup, threads):
    os.environ["OMP_NUM_THREADS"] = str(threads)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # CPU baseline leg only
    if oracle.ref_available():
        m, kind = oracle.RefModel(model_src, use_paged_kv=True, sparse_k=64), "reference"
        # positions 0..context-1 through the reference's own paged_kv_append
        # and lsh_update (synthetic K/V: no CPU prompt)
        m.fill_context(context, seed=7)
        tok, pos = 1, context
    else:
        m, kind = oracle.PortModel(model_src), "port"
        toks = _load("synth").prompt(cfg, 16, seed=7)
        for p in range(16):
            lg = m.forward(int(toks[p]), p)
        tok, pos = int(np.argmax(lg)), 16
    for _ in range(warmup):
        lg = m.forward(tok, pos)
        tok, pos = int(np.argmax(lg)), pos + 1
    t0 = time.perf_counter()
    for _ in range(steps):
        lg = m.forward(tok, pos)
        tok, pos = int(np.argmax(lg)), pos + 1
    dt = time.perf_counter() - t0
    return steps / dt, kind


def host_cores():
    """(threads used, physical cores) of this host."""
    logical = os.cpu_count() or 1
    try:
        import psutil
        physical = psutil.cpu_count(logical=False) or logical
    except Exception:
        physical = logical
    return logical, physical


def run_reference(args):
    ws, rank, local = dist_setup()
    if rank != 0:
        return
    S = _load("synth")
    cfg = S.LLAMA3_8B
    threads, physical = host_cores()
    try:
        import torch
        if not torch.cuda.is_available():
            raise RuntimeError("no device for weight generation")
        src = S.DeviceModel(cfg, seed=SEED, device=0)
        src_model = _HostWeights(cfg, src.bf16_weights())
        torch.cuda.empty_cache()
    except Exception as exc:  # generate on the host instead
        print(f"[bench] device generation unavailable ({exc}); host generation", file=sys.stderr)
        src_model = S.make_model(cfg, seed=SEED)
    val, kind = cpu_baseline(cfg, src_model, args.prompt, args.steps, args.warmup, threads)
    sample = (f"{args.steps} decode steps at context {args.prompt}.."
              f"{args.prompt + args.warmup + args.steps} (positions 0..{args.prompt - 1} of every "
              f"layer's paged cache filled with synthetic K/V through the reference's own "
              f"paged_kv_append and lsh_update, no CPU prompt)")
    line = {"metric": METRIC, "value": round(val, 4), "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 / val, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": config_block(args, ws, big=False, B=1),
            "cpu_baseline": {"value": round(val, 4), "unit": "tok/s", "cores": threads,
                             "physical_cores": physical, "kind": kind, "sample": sample},
            "e2e": {"value": round(val, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    line["config"]["weights"] = "bf16 (= int8 * pow2 scale)"
    emit(line)


def config_block(args, ws, big, B, tmb=0, tp=False):
    """The `config` object both arms print for the same workload."""
    return {"workload": f"{'70b' if big else 'llama3-8b'}-shape decode b={B}"
                        + (f" tensor-parallel over {ws} GPUs" if tp else " per GPU"),
            "global_batch": B if tp else ws * B, "context": args.prompt,
            "weights": "fp8 e4m3 per-tensor pow2 scale" if big else "int8 per-row pow2 scale",
            "kv": f"linear bf16, LSH top-{args.sparse_k}" if big else "paged int8",
            "attention": "reference order" if big else args.attention,
            "parallelism": f"tp{ws} (NCCL all-gathers, rank-order sums)" if tp
                           else f"dp{ws} (replicas)",
            "gemm": "tcgen05 int8 (digit planes)" if (not big and tmb) else "cuda-core gemv chain",
            "l2": "inputs larger than L2 ({} GB of weights streamed per step{})".format(
                "69.5" if big else "7.5", f" over {ws} GPUs" if tp else "")}


class _HostWeights:
    """Adapter: a config plus precomputed BF16 host weights for RefModel."""

    def __init__(self, cfg, bf):
        self.cfg, self._bf = cfg, bf

    def bf16_weights(self):
        return self._bf


def timed_steps(e, torch, stream, tok, pos, B, steps, warmup, local):
    """W untimed steps, then K steps bracketed by CUDA events on the engine's
    stream (inputs resident on the device, greedy tokens fed back on the
    device); returns ms per step, max over ranks."""
    dp = _load("dp")
    for _ in range(warmup):
        e.step_device(tok.data_ptr(), pos.data_ptr(), B, True)
    e.sync()
    dp.barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    ev0.record(stream)
    torch.cuda.nvtx.range_push("timed")  # lets a profiler select these launches
    for _ in range(steps):
        e.step_device(tok.data_ptr(), pos.data_ptr(), B, True)
    torch.cuda.nvtx.range_pop()
    ev1.record(stream)
    e.sync()
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1) / steps
    ms = dp.max_over_ranks(ms, f"cuda:{local}")
    dp.barrier()
    return ms


def e2e_steps(e, cur_tok, cur_pos, steps, local):
    """The same step through the C ABI with host buffers: tokens and positions
    copied in from pinned host memory, logits and greedy tokens copied out
    into pinned host memory, every step (the buffers a serving loop keeps)."""
    import torch
    dp = _load("dp")
    B, V = len(cur_tok), e.c.vocab_size
    pin = lambda shape, dt: torch.empty(shape, dtype=dt, pin_memory=True).numpy()
    tok_h, pos_h = pin(B, torch.int32), pin(B, torch.int32)
    out = (pin((B, V), torch.float32), pin(B, torch.int32))
    tok_h[:] = cur_tok
    pos_h[:] = cur_pos
    for _ in range(2):
        lg, am = e.step(tok_h, pos_h, out=out)
        tok_h[:] = am
        pos_h += 1
    t0 = time.perf_counter()
    for _ in range(steps):
        lg, am = e.step(tok_h, pos_h, out=out)
        tok_h[:] = am
        pos_h += 1
    ms = (time.perf_counter() - t0) * 1000.0 / steps
    return dp.max_over_ranks(ms, f"cuda:{local}"), [int(t) for t in tok_h], [int(p) for p in pos_h]


def run_cuda(args):
    import torch
    ws, rank, local = dist_setup()
    dp = _load("dp")
    torch.cuda.set_device(local)
    dp.init("nccl", torch.device("cuda", local))
    eng = _load("engine")
    S = _load("synth")
    B = args.batch
    big = args.model == "70b"
    dpb = 0 if (big or args.dp_batch <= B) else args.dp_batch  # the b=64-per-GPU record
    tmb = 0
    tp = None
    if big and args.tp and ws > 1:
        # config 5 tensor-parallel: every rank holds 1/N of the heads, FFN and
        # vocabulary rows and decodes the same sequences (ec_create_tp)
        import torch.distributed as dist
        box = [eng.tp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        tp = (rank, ws, box[0])
    if big:
        # FP8 E4M3 per-tensor weights (~70 GB), linear BF16
        # KV with the reference's LSH-routed top-K attention; one GPU, or split
        # tensor-parallel over the ranks with --tp
        cfg = S.LLAMA_70B
        e = eng.Engine(cfg, device=local, tp=tp, max_batch=B, weight_kind=eng.EC_W_FP8,
                       use_paged_kv=False, sparse_k=args.sparse_k)
        src = S.DeviceModel(cfg, seed=SEED, device=local, kind="fp8")
    else:
        cfg = S.LLAMA3_8B
        nb = max(B, dpb)
        tmb = args.tensor_min_batch if nb >= args.tensor_min_batch > 0 else 0
        e = eng.Engine(cfg, device=local, max_batch=nb, tensor_min_batch=tmb,
                       attention_mode=ATTN_MODES[args.attention])
        src = S.DeviceModel(cfg, seed=SEED, device=local)

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
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    # prompt: random tokens through the decode path (KV cache filled), every
    # sequence its own prompt, all sequences of the engine decoded together
    nseq = max(B, dpb)
    # tensor parallelism: every rank decodes the same sequences
    prank = 0 if tp else rank
    prompts = [S.prompt(cfg, args.prompt, seed=7 + prank * 1000 + b) for b in range(nseq)]
    for p in range(args.prompt):
        _, am = e.step([int(pr[p]) for pr in prompts], [p] * nseq, want_logits=False)
    dev = f"cuda:{local}"
    tok_all = torch.tensor([int(a) for a in am], dtype=torch.int32, device=dev)
    pos_all = torch.tensor([args.prompt] * nseq, dtype=torch.int32, device=dev)
    stream = torch.cuda.ExternalStream(e.stream())
    tok, pos = tok_all[:B].clone(), pos_all[:B].clone()
    with Clocks(local) as clk:
        ms = timed_steps(e, torch, stream, tok, pos, B, args.steps, args.warmup, local)
    # data parallel: every rank its own sequences; tensor parallel: the same B
    seq_ranks = 1 if tp else ws
    value = dp.job_throughput(B, seq_ranks, ms)
    e2e_ms, cur_tok, cur_pos = e2e_steps(e, [int(v) for v in tok.cpu()],
                                         [int(v) for v in pos.cpu()], args.steps, local)

    # live per-kernel timing (profiling mode: events around each launch)
    e.profile(True)
    for _ in range(3):
        lg, am = e.step(cur_tok, cur_pos, want_logits=False)
        cur_tok, cur_pos = [int(a) for a in am], [p + 1 for p in cur_pos]
    prof = e.profile_read()
    e.profile(False)
    launches_b = e.launches_per_step(B)

    dp_rec = None
    if dpb:
        # BASELINE config 4's batch split data-parallel: dpb sequences per GPU
        # (global batch dpb x N) on the tensor-core path, the same engine and
        # context; the first B sequences were advanced by the steps above, so
        # every sequence restarts from its own position
        tok_d, pos_d = tok_all.clone(), pos_all.clone()
        pos_d[:B] = torch.tensor(cur_pos, dtype=torch.int32, device=dev)
        tok_d[:B] = torch.tensor(cur_tok, dtype=torch.int32, device=dev)
        dsteps = max(3, min(args.steps, 20))
        with Clocks(local) as clk_d:
            ms_d = timed_steps(e, torch, stream, tok_d, pos_d, dpb, dsteps, args.warmup, local)
        e2e_d, _, _ = e2e_steps(e, [int(v) for v in tok_d.cpu()], [int(v) for v in pos_d.cpu()],
                                dsteps, local)
        dp_rec = {
            "metric": METRIC_B.format(dpb), "value": round(dp.job_throughput(dpb, ws, ms_d), 3),
            "unit": "tok/s", "n_gpus": ws, "steps": dsteps, "warmup": args.warmup,
            "ms_per_step": round(ms_d, 4), "higher_is_better": True, "scaling": "weak",
            "config": config_block(args, ws, big, dpb, tmb),
            "e2e": {"value": round(ws * dpb * 1000.0 / e2e_d, 3), "unit": "tok/s",
                    "h2d_bytes_per_step": 8 * dpb,
                    "d2h_bytes_per_step": 4 * dpb * (cfg.vocab_size + 1)},
            "gpu_launches": e.launches_per_step(dpb) * dsteps,
            "clocks": clk_d.summary()}

    # roofline of the dominant kernel: its algorithmic bytes per launch over its
    # event-timed average launch duration
    tot_ms = sum(v["ms"] for v in prof.values())
    weight_bytes = (sum(int(np.prod(s)) for s in S.mat_shapes(cfg).values()) * cfg.n_layers
                    + cfg.vocab_size * cfg.dim)
    if tp:
        weight_bytes //= ws  # this rank's shard
    if big:
        # linear BF16 K and V of the attended top-K tokens (candidate scoring
        # reads more K rows; not counted)
        kv_tok = cfg.n_layers * cfg.n_kv_heads * cfg.head_dim * 2 * 2
        att_tokens = min(args.prompt + args.warmup + args.steps, args.sparse_k)
    else:
        kv_tok = cfg.n_layers * cfg.n_kv_heads * (cfg.head_dim * 2 + 8)
        att_tokens = min(args.prompt + args.warmup + args.steps, 64 * 16)
    dom = max(prof, key=lambda k: prof[k]["ms"])
    d = dict(prof[dom])
    if dom == "attention" and not d["bytes"] and d["launches"]:
        # the attention launches record no bytes: K and V (with scales) of
        # the attended tokens of every sequence, one layer per launch
        d["bytes"] = d["launches"] * B * (kv_tok / cfg.n_layers) * att_tokens
    peak, peak_kind = peaks()
    achieved = (d["bytes"] / d["launches"]) / (d["ms"] / d["launches"] * 1e-3) / 1e9 \
        if d["launches"] and d["bytes"] else 0.0
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if os.path.exists(tpath) and not big:
        # ncu DRAM bytes per launch of the same kernel at the same batch (8B shape)
        tj = json.load(open(tpath)).get(f"{dom}@{B}")
        if tj:
            traffic = tj["traffic_bytes_per_launch"]
    step_bytes = weight_bytes + B * kv_tok * att_tokens

    if rank == 0:
        line = {
            "metric": (METRIC_70B_TP.format(B, ws, args.prompt, args.sparse_k) if tp else
                       METRIC_70B.format(B, args.prompt, args.sparse_k) if big else
                       METRIC if B == 1 else METRIC_B.format(B)), "value": round(value, 3),
            "unit": "tok/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": None,
            "dtype": "fp8" if big else "int8",
            "data": "synthetic",
            "config": config_block(args, ws, big, B, tmb if (tmb and B >= tmb) else 0, tp=bool(tp)),
            "e2e": {"value": round(seq_ranks * B * 1000.0 / e2e_ms, 3), "unit": "tok/s",
                    "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 4 * B * (cfg.vocab_size + 1)},
            "gpu_launches": launches_b * args.steps,
            "roofline": {"bound": "hbm", "kernel": dom,
                         "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "traffic_source": "ncu dram bytes per launch, profiles/",
                         "algorithmic_bytes_per_launch": round(d["bytes"] / d["launches"])
                         if d["launches"] else None,
                         "peak_source": peak_kind,
                         "step_frac": round(step_bytes / (ms * 1e-3) / 1e9 / peak, 4),
                         "step_bytes": step_bytes},
            "kernel_ms_per_step": {k: round(v["ms"] / 3, 4) for k, v in prof.items()},
            "kernel_share": {k: round(v["ms"] / tot_ms, 4) for k, v in prof.items() if tot_ms},
            "clocks": clk.summary(),
        }
        if dp_rec:
            line["dp_b%d" % dpb] = dp_rec
        threads, physical = host_cores()
        if big:
            line["cpu_baseline"] = {"value": None, "unit": "tok/s", "cores": threads,
                                    "kind": "reference",
                                    "sample": "unavailable: the reference's BF16 copy of the "
                                              "70B shape (~140 GB) exceeds host memory"}
        elif not args.no_cpu_baseline and ws == 1:  # rank 0, one GPU only
            del src
            torch.cuda.empty_cache()
            try:
                src2 = S.DeviceModel(cfg, seed=SEED, device=local)
                hw = _HostWeights(cfg, src2.bf16_weights())
                del src2
                torch.cuda.empty_cache()
                cps, kind = cpu_baseline(cfg, hw, args.prompt, 6, 1, threads)
                line["cpu_baseline"] = {
                    "value": round(cps, 4), "unit": "tok/s", "cores": threads,
                    "physical_cores": physical, "kind": kind,
                    "sample": f"6 decode steps of the 8B shape at context {args.prompt} (K/V of "
                              f"positions 0..{args.prompt - 1} synthetic through the "
                              f"reference's paged_kv_append)"}
            except Exception as exc:
                line["cpu_baseline"] = {"value": None, "unit": "tok/s", "cores": threads,
                                        "kind": "reference", "sample": f"failed: {exc}"}
        emit(line)
    e.close()
    dp.finish()


def main():
    # libraries and the reference engine print to stdout (NCCL's banner, the
    # reference's progress lines): send file descriptor 1 to stderr for the
    # whole run and keep the original for the JSON line
    global _JSON_FD
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prompt", type=int, default=PROMPT, help="tokens already in the cache")
    ap.add_argument("--batch", type=int, default=1,
                    help="sequences decoded together per GPU (b=64: the batched metric)")
    ap.add_argument("--model", default="8b", choices=["8b", "70b"],
                    help="8b: the headline INT8 config; 70b: FP8 config 5 on one GPU")
    ap.add_argument("--sparse-k", type=int, default=511, help="70b: LSH top-K (engine max 511)")
    ap.add_argument("--tp", action="store_true",
                    help="70b under torchrun: tensor-parallel over the ranks (else replicas)")
    ap.add_argument("--tensor-min-batch", type=int, default=16,
                    help="batches this large run their GEMMs on the tensor cores (0: never)")
    ap.add_argument("--dp-batch", type=int, default=64,
                    help="also time this many sequences per GPU (config 4's batch split "
                         "data-parallel; 0: skip)")
    ap.add_argument("--attention", default="split", choices=sorted(ATTN_MODES),
                    help="paged attention: reference order (bit-exact) or split (within "
                         "tolerance, same block set)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_cuda(args)


if __name__ == "__main__":
    main()
