"""The tensor-parallel split, on CPU with two gloo ranks: each rank takes the
column shard of a row-split matrix that ec_create_tp keeps (columns
[rank * K / 2, (rank + 1) * K / 2)) and the rows of a column-split one, runs
the restated GEMV on its shard, and the ranks exchange results with
all_gather -- the same data movement the engine does with NCCL.  The
rank-order sum of the partials is identical on both ranks and within float
rounding of the whole-matrix GEMV; the gathered row shards are the whole
output exactly."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _rank(rank, world, port_path, port_dir, out):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, port_dir)
    import oracle
    dist.init_process_group("gloo", rank=rank, world_size=world)
    P = oracle.port()
    rng = np.random.default_rng(5)
    m, k = 64, 256
    w = rng.standard_normal((m, k), dtype=np.float32) * np.float32(0.02)
    x = rng.standard_normal(k, dtype=np.float32)
    q = np.clip(np.rint(w / (np.abs(w).max(axis=1, keepdims=True) / 127)), -127, 127).astype(np.int8)
    s = (np.abs(w).max(axis=1) / np.float32(127)).astype(np.float32)
    full = np.zeros(m, np.float32)
    P.port_gemv_q8(full, np.ascontiguousarray(q), s, x, m, k)
    # row-split (o, down): columns of this rank, partial outputs summed in rank order
    kl = k // world
    part = np.zeros(m, np.float32)
    P.port_gemv_q8(part, np.ascontiguousarray(q[:, rank * kl:(rank + 1) * kl]), s,
                   np.ascontiguousarray(x[rank * kl:(rank + 1) * kl]), m, kl)
    parts = [torch.zeros(m) for _ in range(world)]
    dist.all_gather(parts, torch.from_numpy(part))
    total = parts[0].numpy().copy()
    for r in range(1, world):
        total = (total + parts[r].numpy()).astype(np.float32)
    # column-split (QKV, gate/up, LM head): rows of this rank, gathered in order
    ml = m // world
    rows = np.zeros(ml, np.float32)
    P.port_gemv_q8(rows, np.ascontiguousarray(q[rank * ml:(rank + 1) * ml]),
                   np.ascontiguousarray(s[rank * ml:(rank + 1) * ml]), x, ml, k)
    got = [torch.zeros(ml) for _ in range(world)]
    dist.all_gather(got, torch.from_numpy(rows))
    gathered = np.concatenate([g.numpy() for g in got])
    np.save(os.path.join(out, f"r{rank}.npy"), np.stack([total, full, gathered]))
    dist.destroy_process_group()


def test_tp_split_and_sum_two_gloo_ranks(tmp_path, oracle):
    import torch.multiprocessing as tmp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(29600 + os.getpid() % 1000)
    tmp.spawn(_rank, args=(2, oracle.PORT_SO, os.path.dirname(oracle.__file__), str(tmp_path)),
              nprocs=2, join=True)
    a = np.load(tmp_path / "r0.npy")
    b = np.load(tmp_path / "r1.npy")
    assert np.array_equal(a[0].view(np.uint32), b[0].view(np.uint32))  # same sum on every rank
    assert np.abs(a[0] - a[1]).max() <= 1e-5 * np.abs(a[1]).max()      # the whole GEMV
    assert np.array_equal(a[2].view(np.uint32), a[1].view(np.uint32))   # row shards: exact
