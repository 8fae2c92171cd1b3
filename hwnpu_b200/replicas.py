"""Multi-GPU by replicas (no collective on the decode path).

Sequences are independent, so a job of several GPUs runs one engine replica a GPU with the
weights replicated, and splits the sequences between them round robin (the partition of the
64-sequence ragged-batch workload). The only cross-rank traffic is the
timing: the job's time is the slowest replica's, and its throughput is the tokens of all replicas
over that time. Works over any torch.distributed backend (gloo on CPU for the tests, NCCL on the
GPUs).
"""


def shard(n_items, rank, world):
    """The items of `rank`: i with i % world == rank (round robin, sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    return list(range(rank, n_items, world))


def job_time(seconds, dist=None, device=None):
    """The slowest rank's time (max over ranks); the local time without a process group."""
    if dist is None:
        return float(seconds)
    import torch

    t = torch.tensor([float(seconds)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def job_total(count, dist=None, device=None):
    """The sum over ranks of a per-rank count (tokens processed)."""
    if dist is None:
        return int(count)
    import torch

    t = torch.tensor([int(count)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(t.item())
