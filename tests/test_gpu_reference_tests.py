"""The reference's own C++ tests, run against this build's reference-signature
layer on the GPU.

tests/test_kokoro_decoder_backward.cpp and tests/test_decoder_lora.cpp of the
reference are compiled unchanged apart from the device constant (Device::CPU ->
Device::CUDA) against include/ (brotensor/tensor.h, brosoundml/*.h,
kokoro_decoder_backward.h) and libbsml_ref.so by the recipe in oracle/Makefile
(outputs in oracle/_ref/, built by __graft_entry__.build() where the reference
checkout is present; the binaries travel with the build). They check, with the
reference's own tolerances:
  * per-element central finite differences of the AdaIN affine and the spectral head,
  * directional finite differences of both residual blocks, the backbone and the
    generator assemblies, and of DecoderLora's adapter and gate gradients,
  * DecoderLora's neutral identity (cond = 0 reproduces DecoderBackbone::forward
    + Generator::forward within 1e-4) and its checkpoint round trip (1e-7),
  * the conditioning gate's zero initialisation, g(0) = 0 and its FD gradients.
A run prints "<name>: OK" and exits 0, or lists each failure and exits 1."""

import os
import subprocess

import pytest

from tests.conftest import ROOT, cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

REF_BIN = os.path.join(ROOT, "oracle", "_ref")


@pytest.mark.parametrize("name", ["test_decoder_lora", "test_kokoro_decoder_backward"])
def test_reference_cpp_test_passes(name, tmp_path):
    exe = os.path.join(REF_BIN, name)
    if not os.path.exists(exe):
        pytest.skip(f"{exe} is not built (build() makes it where the reference checkout is present)")
    # the reference's checkpoint test writes its file into the working directory
    r = subprocess.run([exe], capture_output=True, text=True, timeout=900, cwd=str(tmp_path))
    print(r.stdout[-4000:])
    assert r.returncode == 0 and f"{name}: OK" in r.stdout, (r.stdout[-4000:], r.stderr[-2000:])


def test_gpu_checkpoint_loads_in_the_reference(tmp_path):
    """An ELRA1 file written by the GPU DecoderLora (bsml_lora_save) restores, through
    the reference's own DecoderLora::load (oracle/_ref/libref_compose.so, the
    reference's src/decoder_lora.cpp compiled here), to exactly the GPU's values."""
    import ctypes

    import numpy as np
    import torch

    from brosoundml_b200 import config
    from brosoundml_b200.decoder import Decoder
    from brosoundml_b200.lora import DecoderLora
    from oracle.oracle import Oracle
    from tests.test_ref_compose_cpu import LIB, _cfg, _lib, _p, _table

    if not os.path.exists(LIB):
        pytest.skip("libref_compose.so is built where the reference checkout is present")
    cfg = config.miniature()
    o = Oracle(cfg)
    d = Decoder(cfg, 0)
    lora = DecoderLora(d, rank=4, scale=1.75, seed=3)
    with torch.no_grad():
        lora.params().uniform_(-0.3, 0.3)
    torch.cuda.synchronize()
    path = str(tmp_path / "gpu.elra")
    lora.save(path)
    want = lora.params().cpu().numpy()
    L = _lib()
    names, offs, nums = _table(o)
    c = _cfg(cfg)
    params = np.zeros(o.n_params, np.float32)
    oA, oB = np.array(lora.off_A, np.int64), np.array(lora.off_B, np.int64)
    back = np.zeros(lora.n_params, np.float32)
    sc = ctypes.c_float(0)
    rc = L.refc_lora_load(ctypes.byref(c), len(o.table), names, _p(offs), _p(nums), _p(params), 4, path.encode(),
                          lora.off_W1, lora.off_W2, _p(oA), _p(oB), _p(back), ctypes.byref(sc))
    assert rc == 0, L.refc_last_error()
    assert np.array_equal(back, want) and abs(sc.value - 1.75) < 1e-7
