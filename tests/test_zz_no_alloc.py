"""GPU test of bsml_conv1d_backward_weight_noalloc, the weight-gradient entry point
for callers that may not allocate device memory (a real-time audio thread, an
application whose device memory is owned by its own arena). It must give what the
allocating entry point gives, call after call, though every call reuses one static
scratch array. This file is named to be collected last."""

import ctypes

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

if cuda_available():
    import torch

    from brosoundml_b200 import _lib

# (B, Ci, L, Co, k, stride, pad, dil): a generator conv (k7, dilation 3) and a
# strided noise conv; the two calls in a row use different shapes and data
CASES = [(2, 128, 2000, 128, 7, 1, 9, 3), (1, 22, 1201, 256, 12, 6, 3, 1)]


def _P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


def _call(name, dy, x, case, dW, db):
    B, Ci, L, Co, k, s, p, d = case
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    fn = getattr(_lib.lib(), name)
    _lib.check(fn(_P(dy), _P(x), B, Ci, L, Co, k, s, p, d, _P(dW), _P(db), st))


def test_noalloc_weight_gradient_matches_allocating_entry_point():
    for i, case in enumerate(CASES):   # two calls in a row
        B, Ci, L, Co, k, s, p, d = case
        Lo = (L + 2 * p - d * (k - 1) - 1) // s + 1
        g = torch.Generator(device="cuda").manual_seed(1234 + i)
        dy = torch.randn((B, Co, Lo), device="cuda", generator=g)
        x = torch.randn((B, Ci, L), device="cuda", generator=g)
        ref_w, ref_b = torch.empty((Co, Ci, k), device="cuda"), torch.empty(Co, device="cuda")
        got_w, got_b = torch.full((Co, Ci, k), float("nan"), device="cuda"), torch.full((Co,), float("nan"), device="cuda")
        _call("bsml_conv1d_backward_weight", dy, x, case, ref_w, ref_b)
        _call("bsml_conv1d_backward_weight_noalloc", dy, x, case, got_w, got_b)
        torch.cuda.synchronize()
        # same tolerance as the other conv atoms (rel-L2 1e-5)
        assert _rel(got_w, ref_w) < 1e-5
        assert _rel(got_b, ref_b) < 1e-5


def test_noalloc_rejects_problems_beyond_its_scratch():
    B, Ci, L, Co, k = 16, 128, 24001, 128, 7   # ~98 M floats of scratch
    dy = torch.zeros(1, device="cuda")
    with pytest.raises(_lib.BsmlError, match="static maximum"):
        _call("bsml_conv1d_backward_weight_noalloc", dy, dy, (B, Ci, L, Co, k, 1, 3, 1), dy, None)
