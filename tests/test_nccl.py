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


def _run_ranks(target, n, *args, timeout=180):
    """Child processes (spawned), one per rank; always terminated and joined."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=target, args=(r, *args, q)) for r in range(n)]
    try:
        for p in ps:
            p.start()
        return sorted(q.get(timeout=timeout) for _ in range(n))
    finally:
        for p in ps:
            p.join(timeout=30)
            if p.is_alive():
                p.terminate()
                p.join(timeout=30)


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")
def test_two_rank_allreduce():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = os.path.join(tempfile.mkdtemp(), "uid")
    out = _run_ranks(_rank, 2, path)
    for rank, s, spread, avg in out:
        assert s == 3.0 and spread == 0.0 and avg == 1.5, (rank, s, avg)


def _rank_leaves(rank, path, q):
    """Rank 1 takes part in one step and leaves between steps (its collectives
    finished, its communicator destroyed); rank 0's next step must end in an
    error within the communicator's timeout, not hang."""
    import time

    os.environ["NCCL_NVLS_ENABLE"] = "0"   # plain peer transport: no multicast objects
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
    comm = NcclComm(2, uid, rank, rank, timeout_ms=5000)
    g = torch.full((4096,), float(rank + 1), device="cuda")
    comm.allreduce(g, average=False)
    comm.sync()
    ok1 = float(g[0]) == 3.0
    if rank == 1:
        comm.close()
        q.put((rank, ok1, None, 0.0))
        return
    time.sleep(1.0)   # rank 1 has gone
    t0 = time.time()
    err = None
    try:
        comm.allreduce(g, average=False)
        comm.sync()
    except RuntimeError as e:
        err = str(e)
    dt = time.time() - t0
    # the context still computes after the abort
    x = torch.arange(10, device="cuda", dtype=torch.float32)
    ok2 = float((x * 2).sum()) == 90.0
    comm.close()
    q.put((rank, ok1 and ok2, err, dt))


@pytest.mark.gpu
@pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")
def test_peer_leaves_between_steps():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = os.path.join(tempfile.mkdtemp(), "uid")
    out = _run_ranks(_rank_leaves, 2, path)
    (r0, ok0, err, dt), (r1, ok1, _, _) = out
    assert ok0 and ok1
    assert err is not None and "aborted" in err, err
    assert dt < 30.0, dt
