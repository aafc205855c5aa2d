"""Data-parallel host logic on CPU: two gloo ranks each run the float64 oracle on
their shard of a global batch, average the flat gradient with
brosoundml_b200.dp.average_gradients, and must reproduce the single-process
gradient of the mean L1 loss over the whole batch."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from brosoundml_b200 import config, dp, synth
from oracle import oracle as _orc
from oracle.oracle import Oracle

B_GLOBAL, T, FRAMES = 4, 4, 33   # the miniature config takes har from the caller (1 channel)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(cfg):
    inp = synth.make_inputs(cfg, B_GLOBAL, T, 1)
    inp["har"] = np.random.default_rng(3).normal(0, 1, (B_GLOBAL, cfg["har_ch"], FRAMES)).astype(np.float32)
    S = cfg["hop"] * (FRAMES - 1)
    tgt = np.random.default_rng(4).uniform(-0.1, 0.1, (B_GLOBAL, S)).astype(np.float32)
    return inp, tgt


def _shard_grads(cfg, params, inp, tgt, sl):
    orc = Oracle(cfg)
    x = {k: v[sl] for k, v in inp.items()}
    out = orc.run(params, x["asr"], x["F0"], x["N"], x["style"], har=x["har"], dtype=np.float64)
    _, da = synth.l1_grad(out["audio"], tgt[sl].astype(np.float64))
    return orc.run(params, x["asr"], x["F0"], x["N"], x["style"], har=x["har"], daudio=da,
                   dtype=np.float64)["grads"]


def _rank(rank, world, port, q):
    # the two ranks share the host's cores: a few oracle threads each, no oversubscription
    _orc.set_threads(max(1, (os.cpu_count() or 2) // (2 * world)))
    torch.set_num_threads(1)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    code = 1
    try:
        cfg = config.miniature()
        orc = Oracle(cfg)
        params = synth.init_params(orc.table, orc.n_params, 0).astype(np.float64)
        inp, tgt = _batch(cfg)
        g = torch.from_numpy(_shard_grads(cfg, params, inp, tgt, dp.shard(B_GLOBAL, rank, world)))
        dp.average_gradients(g)
        if rank == 0:
            q.put(g.numpy())
        code = 0
    finally:
        # leave without interpreter teardown: tearing down gloo next to the oracle's
        # OpenMP runtime crashes this torch build after the work is done
        q.close()
        q.join_thread()
        os._exit(code)


def test_shard_rules():
    assert dp.shard(8, 1, 4) == slice(2, 4)
    with pytest.raises(ValueError):
        dp.shard(6, 0, 4)
    with pytest.raises(ValueError):
        dp.shard(8, 4, 4)


def test_two_rank_gradient_average_matches_full_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    g_dp = q.get(timeout=300)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cfg = config.miniature()
    orc = Oracle(cfg)
    params = synth.init_params(orc.table, orc.n_params, 0).astype(np.float64)
    inp, tgt = _batch(cfg)
    g_full = _shard_grads(cfg, params, inp, tgt, slice(0, B_GLOBAL))
    np.testing.assert_allclose(g_dp, g_full, rtol=1e-10, atol=1e-14)


def _rank_leaves(rank, world, port, q):
    from datetime import timedelta
    import time

    torch.set_num_threads(1)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)   # leaves between steps: never joins the gradient all-reduce
    t0 = time.time()
    try:
        dp.average_gradients(torch.ones(16, dtype=torch.float64))
        q.put(("ok", time.time() - t0, ""))
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        q.put(("error", time.time() - t0, f"{type(e).__name__}: {str(e)[:200]}"))
    q.close()
    q.join_thread()
    os._exit(0)


def test_rank_that_leaves_gives_an_error_not_a_hang():
    """A rank that exits between steps: the surviving rank's gradient all-reduce ends
    with an error (peer gone or process-group timeout), never a hang."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank_leaves, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    outcome, dt, msg = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
    assert outcome == "error", msg
    assert dt < 60, dt
