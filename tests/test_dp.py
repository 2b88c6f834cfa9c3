"""Data-parallel plumbing of the decode bench (42-berlin-engine_b200/dp.py) on
CPU: two gloo ranks on 127.0.0.1, the sharding of sequences, the
max-over-ranks timing and the whole-job throughput."""
import os
import socket

import pytest

from conftest import load_pkg_module


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world),
                      RANK=str(rank), LOCAL_RANK=str(rank))
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    dp = load_pkg_module("dp")
    assert dp.init("gloo") == world
    start, count = dp.shard(13, world, rank)
    dp.barrier()
    t = dp.max_over_ranks(1.0 + 1.5 * rank)
    thr = dp.job_throughput(count, world, t)
    dp.finish()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{start} {count} {t} {thr}")


def test_two_gloo_ranks(tmp_path):
    mp = pytest.importorskip("torch.multiprocessing")
    world, port = 2, _free_port()
    mp.spawn(_rank_main, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    rows = [open(tmp_path / f"rank{r}.txt").read().split() for r in range(world)]
    (s0, c0, t0, _), (s1, c1, t1, thr1) = rows
    assert (int(s0), int(c0), int(s1), int(c1)) == (0, 7, 7, 6)  # 13 sequences over 2 ranks
    assert float(t0) == float(t1) == 2.5                        # the slower rank's time
    assert float(thr1) == pytest.approx(2 * 6 * 1000.0 / 2.5)


def test_shard_covers_every_sequence_once():
    dp = load_pkg_module("dp")
    for total in (0, 1, 7, 64, 512, 513):
        for world in (1, 2, 3, 8):
            got = [dp.shard(total, world, r) for r in range(world)]
            assert sum(c for _, c in got) == total
            pos = 0
            for start, count in got:
                assert start == pos
                pos += count
            assert max(c for _, c in got) - min(c for _, c in got) <= 1
    with pytest.raises(ValueError):
        dp.shard(4, 2, 2)
