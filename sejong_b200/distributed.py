"""Data-parallel plumbing: one process per GPU, NCCL over NVLink (gloo on CPU for tests).

The reference trains on one GPU (crates/sejong-gpu/src/hip.rs:114-138); data parallelism is an
addition.  Each rank trains on its own batch drawn with its own seed; the cross-entropy seed of
every rank is loss_scale / (rows_per_rank * world) (the reference seeds loss_scale / rows,
crates/sejong-gpu/src/graph.rs:539-549), so a SUM all-reduce of the per-rank gradients is the
gradient of the mean loss over the global batch, and a SUM of the per-rank loss sums is that
mean loss.  The FP64 gradient norm and the clip are then taken on the reduced gradient, which
matches the single-process norm of crates/sejong-train/src/lib.rs:199-238.
"""
import datetime
import os

import torch
import torch.distributed as dist


def rank_seed(base, rank):
    """Seed of rank `rank`'s data stream (rank 0 keeps the single-process seed)."""
    return int(base) + int(rank)


def ce_seed(rows_per_rank, world, loss_scale=1.0):
    """Per-row cross-entropy seed so that the SUM over ranks is the global-batch mean."""
    return float(loss_scale) / (int(rows_per_rank) * int(world))


def exchange(grad_flat, loss_sum, group=None, norm_partials=None):
    """In-place SUM all-reduce of the flat gradient buffer and of the loss sum.

    With expert parallelism `grad_flat` is the replicated range only and `norm_partials` (FP64)
    carries the sums of squares of each rank's own experts' gradients, so that after the
    exchange every rank sees the global gradient norm."""
    if group is None and not dist.is_initialized():
        return
    if dist.get_world_size(group) == 1:
        return
    dist.all_reduce(grad_flat, group=group)
    dist.all_reduce(loss_sum, group=group)
    if norm_partials is not None:
        dist.all_reduce(norm_partials, group=group)


def init_from_env(backend="nccl", timeout_s=300):
    """Initialise the default process group from torchrun's environment.

    Returns (rank, world, local_rank, group); group is None for a single process.  A short
    timeout makes ranks that wait for a failed peer end with an error instead of hanging.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world == 1:
        return rank, 1, local, None
    kwargs = dict(timeout=datetime.timedelta(seconds=timeout_s))
    if backend == "nccl":
        torch.cuda.set_device(local)
        kwargs["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, **kwargs)
    return rank, world, local, dist.group.WORLD
