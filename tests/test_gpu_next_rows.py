"""The rows after the training path, held to the oracle.

* Inference: bsml_decoder_decode is Kokoro::Impl::decode_back_half
  (src/kokoro.cpp:352-407) batched: backbone with style = ref_s[:, :style_dim], the
  harmonic source from F0, generator, iSTFT. Compared with the float64 oracle's
  forward on the same har bytes (the bsml_harmonic_source atom runs the engine's own
  kernels on the same F0; the har itself is checked against the reference's
  arithmetic in test_gpu_parity.py::test_harmonic_source).
* KokoroDecodePrep files (include/brosoundml/kokoro.h:132-147: ref_s, asr, F0_pred,
  N_pred, har) written to disk, loaded, stacked into a batch and run through a
  training step (forward, L1-shaped upstream gradient, backward), against the float64
  oracle on the same arrays."""

import ctypes

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from brosoundml_b200 import config, synth  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402
from tests.helpers import rel_l2  # noqa: E402


def _har_gpu(cfg, o, params_dev, F0):
    import torch

    from brosoundml_b200 import _lib
    lw = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.weight")["offset"]
    lb = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.bias")["offset"]
    B, F = F0.shape
    f0 = torch.tensor(np.ascontiguousarray(F0), device="cuda")
    har = torch.empty((B, cfg["har_ch"], config.har_frames(cfg, F // 2)), device="cuda")
    c = _lib.make_config(cfg)
    _lib.check(_lib.lib().bsml_harmonic_source(ctypes.byref(c), ctypes.c_void_p(f0.data_ptr()), B, F,
                                               ctypes.c_void_p(params_dev.data_ptr() + 4 * lw),
                                               ctypes.c_void_p(params_dev.data_ptr() + 4 * lb),
                                               ctypes.c_void_p(har.data_ptr()),
                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    return har.cpu().numpy()


def test_decode_back_half_vs_oracle():
    import torch

    from brosoundml_b200.decoder import Decoder
    cfg, B, T = config.kokoro_82m(), 2, 32
    S = cfg["style_dim"]
    o = Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, B, T, 7)
    ref_s = np.concatenate([x["style"], np.random.default_rng(8).normal(0, 1, (B, S)).astype(np.float32)], axis=1)
    dec = Decoder(cfg, 0, math="tf32x3")
    pd = torch.tensor(params, device="cuda")
    dv = {k: torch.tensor(v, device="cuda") for k, v in x.items()}
    audio = dec.decode(pd, torch.tensor(ref_s, device="cuda"), dv["asr"], dv["F0"], dv["N"])
    torch.cuda.synchronize()
    har = _har_gpu(cfg, o, pd, x["F0"])
    r64 = o.run(params, x["asr"], x["F0"], x["N"], np.ascontiguousarray(ref_s[:, :S]), har=har, dtype=np.float64)
    e = rel_l2(audio.cpu().numpy(), r64["audio"])
    print(f"decode_back_half vs float64 oracle: audio rel-L2 {e:.2e}")
    assert e < 1e-4


def test_decode_prep_files_drive_a_training_step(tmp_path):
    import torch

    from brosoundml_b200 import weights
    from brosoundml_b200.decoder import Decoder
    cfg, B, T = config.kokoro_82m(), 2, 32
    S = cfg["style_dim"]
    o = Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    paths = []
    for b in range(B):
        x = synth.make_inputs(cfg, 1, T, 20 + b)
        ref_s = np.concatenate([x["style"], np.zeros((1, S), np.float32)], axis=1)
        har = o.harmonic_source(params, x["F0"])
        p = str(tmp_path / f"clip{b}.safetensors")
        weights.save_decode_prep(p, ref_s[0], x["asr"][0], x["F0"][0], x["N"][0], har[0])
        paths.append(p)
    batch = weights.stack_decode_preps([weights.load_decode_prep(p) for p in paths])
    asr, F0, N, har = batch["asr"], batch["F0"], batch["N"], batch["har"]
    style = np.ascontiguousarray(batch["ref_s"][:, :S])
    assert asr.shape == (B, cfg["asr_dim"], T) and har.shape[0] == B
    dec = Decoder(cfg, 0, math="tf32x3")
    t = lambda a: torch.tensor(np.ascontiguousarray(a, np.float32), device="cuda")  # noqa: E731
    audio = dec.forward(t(params), t(asr), t(F0), t(N), t(style), har=t(har))
    target = synth.make_target(cfg, B, T, 3)[:, :audio.shape[1]]
    # an L1-shaped upstream gradient, taken from the oracle's audio so both sides get the same bytes
    r = o.run(params, asr, F0, N, style, har=har)
    da = (np.sign(r["audio"] - target) / target.size).astype(np.float32)
    g = dec.backward(t(da))
    torch.cuda.synchronize()
    r64 = o.run(params, asr, F0, N, style, har=har, daudio=da, dtype=np.float64)
    ea = rel_l2(audio.cpu().numpy(), r64["audio"])
    eg = rel_l2(g["grads"].cpu().numpy(), r64["grads"])
    ed = rel_l2(g["d_asr"].cpu().numpy(), r64["d_asr"])
    print(f"decode-prep step vs float64 oracle: audio {ea:.2e}, grads {eg:.2e}, d_asr {ed:.2e}")
    assert ea < 1e-4 and eg < 1e-4 and ed < 1e-3
