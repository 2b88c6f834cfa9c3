"""Data parallelism for the decode path: one process per GPU, each with a full
replica of the weights and its own independent sequences.  The path shards
by sequence (survey: independent decode sequences split across GPUs), so the
data path has no collective; the only cross-rank traffic is a barrier before
and after the timed region and the maximum of the per-rank times.

Launch: python -m torch.distributed.run --nnodes=1 --nproc-per-node N
        --master-addr 127.0.0.1 --master-port P <script>
"""
import os


def rank_env():
    """(world_size, rank, local_rank) from the launcher's environment."""
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard(global_batch, world, rank):
    """The sequences [start, start + count) rank `rank` decodes: contiguous,
    as even as possible, the first ranks taking one more when uneven."""
    if global_batch < 0 or world <= 0 or not 0 <= rank < world:
        raise ValueError("bad shard request")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def init(backend, device=None):
    """Join the process group when launched with more than one rank."""
    import torch.distributed as dist
    world, _, _ = rank_env()
    if world > 1 and not dist.is_initialized():
        if device is not None:
            dist.init_process_group(backend, device_id=device)
        else:
            dist.init_process_group(backend)
    return world


def barrier():
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()


def max_over_ranks(value, device="cpu"):
    """The largest of every rank's `value` (a time): the job's time."""
    import torch
    import torch.distributed as dist
    if not (dist.is_initialized() and dist.get_world_size() > 1):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_throughput(tokens_per_rank, world, ms_max):
    """Whole-job tokens per second: every rank's tokens over the slowest rank's
    time per step."""
    return world * tokens_per_rank * 1000.0 / ms_max


def finish():
    import torch.distributed as dist
    if dist.is_initialized():
        dist.destroy_process_group()
