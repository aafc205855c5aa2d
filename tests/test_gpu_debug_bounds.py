"""The bounds-checking debug build (make -C brosoundml_b200 DEBUG=1 ->
libbsml_b200_debug.so, selected with BSML_LIB): a whole-decoder training step and
both block kinds run with every channels-last row access of the elementwise,
normalisation and spectral kernels checked, and none leaves its view. Run in a
child process because a process loads one build of the library."""

import os
import subprocess
import sys

import pytest

from tests.conftest import ROOT, cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

DEBUG_LIB = os.path.join(ROOT, "brosoundml_b200", "libbsml_b200_debug.so")

CHILD = r"""
import ctypes, sys
import numpy as np, torch
sys.path.insert(0, ROOT)
from brosoundml_b200 import _lib, config, synth
from brosoundml_b200.decoder import Block, Decoder
assert _lib.LIB_PATH.endswith("libbsml_b200_debug.so")
rec = (ctypes.c_int * 5)()
def check(what):
    _lib.check(_lib.lib().bsml_debug_bounds(ctypes.cast(rec, ctypes.c_void_p)))
    assert list(rec) == [0] * 5, (what, list(rec))
    assert _lib.lib().bsml_device_error() == 0, what
for which, B, T, math in (("miniature", 2, 4, "fp32"), ("kokoro_82m", 2, 8, "tf32x3")):
    cfg = getattr(config, which)()
    d = Decoder(cfg, 0, math=math)
    p = torch.tensor(synth.init_params(d.table, d.n_params, 0), device="cuda")
    x = {k: torch.tensor(v, device="cuda") for k, v in synth.make_inputs(cfg, B, T, 1).items()}
    har = None
    if which == "miniature":
        har = torch.rand((B, 1, 33), device="cuda") - 0.5
    a = d.forward(p, x["asr"], x["F0"], x["N"], x["style"], har=har)
    d.backward(torch.randn_like(a) * 1e-3)
    check(which)
for spec, L in ((dict(kind=2, style_dim=128, cin=128, cout=128, kernel=7, dil=[1, 3, 5]), 300),
                (dict(kind=1, style_dim=128, cin=130, cout=64, upsample=1), 40)):
    blk = Block(spec, 0, math="tf32x3")
    p = torch.randn(blk.n_params, device="cuda") * 0.05
    xx = torch.randn((2, spec["cin"], L), device="cuda")
    y = blk.forward(p, xx, torch.randn((2, 128), device="cuda"))
    blk.backward(torch.randn_like(y))
    check(spec["kind"])
print("DEBUG_BOUNDS_OK")
"""


def test_debug_build_reports_no_out_of_range_access():
    if not os.path.exists(DEBUG_LIB):
        pytest.skip("the debug build is made by __graft_entry__.build()")
    env = dict(os.environ, BSML_LIB=DEBUG_LIB)
    r = subprocess.run([sys.executable, "-c", f"ROOT = {ROOT!r}\n" + CHILD], capture_output=True, text=True,
                       timeout=600, env=env)
    assert r.returncode == 0 and "DEBUG_BOUNDS_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])
