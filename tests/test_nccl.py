"""The library's own NCCL path for callers without torch.distributed
(bsml_nccl_* / bsml_allreduce_grads, loaded at run time): a unique id on the
CPU, a one-rank communicator on one GPU, and (where two GPUs exist) a two-process
all-reduce that sums and averages."""

import os
import tempfile

import pytest

from tests.conftest import cuda_available


def test_unique_id_without_gpu():
    from brosoundml_b200.dp import NcclComm
    a, b = NcclComm.unique_id(), NcclComm.unique_id()
    assert len(a) == 128 and a != b


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")
def test_single_rank_allreduce():
    import torch

    from brosoundml_b200.dp import NcclComm
    comm = NcclComm(1, NcclComm.unique_id(), 0, 0)
    g = torch.arange(1000, dtype=torch.float32, device="cuda")
    ref = g.clone()
    comm.allreduce(g, average=True)
    comm.allreduce(g, average=False)
    torch.cuda.synchronize()
    assert torch.equal(g, ref)
    comm.close()


def _rank(rank, path, q):
    import time

    import torch

    from brosoundml_b200.dp import NcclComm
    torch.cuda.set_device(rank)
    if rank == 0:
        uid = NcclComm.unique_id()
        with open(path + ".tmp", "wb") as f:
            f.write(uid)
        os.replace(path + ".tmp", path)
    else:
        for _ in range(600):
            if os.path.exists(path):
                break
            time.sleep(0.05)
        uid = open(path, "rb").read()
    comm = NcclComm(2, uid, rank, rank)
    g = torch.full((4096,), float(rank + 1), device="cuda")
    comm.allreduce(g, average=False)
    h = torch.full((4096,), float(rank + 1), device="cuda")
    comm.allreduce(h, average=True)
    torch.cuda.synchronize()
    q.put((rank, float(g[0]), float(g.max() - g.min()), float(h[0])))
    comm.close()


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")
def test_two_rank_allreduce():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    path = os.path.join(tempfile.mkdtemp(), "uid")
    ps = [ctx.Process(target=_rank, args=(r, path, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = sorted(q.get(timeout=180) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    for rank, s, spread, avg in out:
        assert s == 3.0 and spread == 0.0 and avg == 1.5, (rank, s, avg)
