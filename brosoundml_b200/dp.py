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


class NcclComm:
    """A communicator of the library's own NCCL path (``bsml_nccl_*``), for callers
    without torch.distributed: rank 0 makes :meth:`unique_id` and passes the 128
    bytes to the other ranks by any channel; every rank then builds its
    communicator and all-reduces its flat gradient once per step."""

    @staticmethod
    def unique_id() -> bytes:
        import ctypes

        from . import _lib

        buf = ctypes.create_string_buffer(128)
        _lib.check(_lib.lib().bsml_nccl_unique_id(ctypes.cast(buf, ctypes.c_void_p)))
        return buf.raw

    def __init__(self, nranks: int, uid: bytes, rank: int, device: int, timeout_ms: int = 120000):
        import ctypes

        from . import _lib

        if len(uid) != 128:
            raise ValueError("brosoundml: NcclComm: the unique id has 128 bytes")
        buf = ctypes.create_string_buffer(uid, 128)
        c = ctypes.c_void_p()
        self._c = None
        _lib.check(_lib.lib().bsml_nccl_comm_init_timeout(nranks, ctypes.cast(buf, ctypes.c_void_p), rank, device,
                                                          timeout_ms, ctypes.byref(c)))
        self._c = c

    def sync(self) -> None:
        """Waits for the current stream's work, bounded by the communicator's
        timeout; raises (and aborts the communicator) when a peer has left or
        NCCL reports an error."""
        import ctypes

        import torch

        from . import _lib

        _lib.check(_lib.lib().bsml_nccl_sync(self._c, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))

    def allreduce(self, grads, average: bool = True) -> None:
        """In place over a float32 CUDA tensor, on the current stream."""
        import ctypes

        import torch

        from . import _lib

        if not (grads.is_cuda and grads.dtype == torch.float32 and grads.is_contiguous()):
            raise TypeError("brosoundml: NcclComm.allreduce needs a contiguous float32 CUDA tensor")
        _lib.check(_lib.lib().bsml_allreduce_grads(self._c, ctypes.c_void_p(grads.data_ptr()), grads.numel(),
                                                   1 if average else 0,
                                                   ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))

    def close(self) -> None:
        from . import _lib

        if getattr(self, "_c", None) is not None and _lib._lib is not None:
            _lib.lib().bsml_nccl_comm_destroy(self._c)
            self._c = None

    __del__ = close
