"""Failure detection on the GPU without a fault: every tensor-core kernel's waits
are bounded; a wait that runs out leaves a code in the device error word
(bsml_device_error) and the kernel returns, so the context stays usable. The
self-test kernel waits on a barrier that nothing completes."""

import time

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


def test_bounded_wait_gives_up_reports_and_leaves_the_context_usable():
    import torch

    from brosoundml_b200 import _lib
    from brosoundml_b200.decoder import Block

    L = _lib.lib()
    torch.cuda.init()
    assert L.bsml_device_error() == 0           # reads and clears the word
    t0 = time.time()
    _lib.check(L.bsml_selftest_bounded_wait(None))
    code = L.bsml_device_error()               # synchronises
    dt = time.time() - t0
    assert code == 1, code                      # TC_ERR_WAIT_FULL
    assert 1.5 < dt < 30, dt
    assert L.bsml_device_error() == 0           # cleared by the read
    # the context still runs tensor-core work correctly afterwards
    spec = dict(kind=2, style_dim=16, cin=64, cout=64, kernel=3, dil=[1, 3, 5])
    a = Block(spec, 0, math="tf32x3")
    b = Block(spec, 0, math="fp32")
    rng = np.random.default_rng(0)
    p = torch.tensor(rng.uniform(-0.1, 0.1, a.n_params).astype(np.float32), device="cuda")
    x = torch.randn(2, 64, 300, device="cuda")
    s = torch.randn(2, 16, device="cuda")
    ya = a.forward(p, x, s)
    yb = b.forward(p, x, s)
    torch.cuda.synchronize()
    assert float((ya - yb).norm() / yb.norm()) < 1e-5
    assert L.bsml_device_error() == 0
