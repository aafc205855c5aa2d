"""Data-parallel training of the decoder across GPUs.

One process per GPU (torchrun), each with its own decoder engine and its own
share of the clips. The path has no data-path collective: after every rank's
backward, the flat gradient buffer (one tensor for all parameters) is averaged
with a single all-reduce (NCCL over NVLink on GPUs, gloo on CPU), then every
rank applies the same Adam update. With equal shards and a mean loss per shard,
the averaged gradient equals the gradient of the mean loss over the global batch.
"""

from __future__ import annotations


def shard(n_global: int, rank: int, world: int) -> slice:
    """Contiguous, equal share of a global batch of ``n_global`` clips for ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"brosoundml: shard: bad rank {rank} of {world}")
    if n_global % world != 0:
        raise ValueError(f"brosoundml: shard: global batch {n_global} does not split into {world} equal shares")
    n = n_global // world
    return slice(rank * n, (rank + 1) * n)


def average_gradients(grads, group=None) -> None:
    """In-place mean of the flat gradient buffer over the ranks of ``group``
    (no-op without an initialised process group or with one rank)."""
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    if dist.get_backend(group) == "gloo":   # gloo has no AVG reduction
        dist.all_reduce(grads, op=dist.ReduceOp.SUM, group=group)
        grads /= dist.get_world_size(group)
    else:
        dist.all_reduce(grads, op=dist.ReduceOp.AVG, group=group)
