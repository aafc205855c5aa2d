"""Whole-decoder parity at the benchmarked configuration
(B = 16 clips x T = 200 asr frames, 5 s of audio each), with bench.py's seeded
weights and inputs, in the TF32x3, TF32x3W (TF32x3 with BF16x3 weight gradients),
TF32x3F (TF32x3 forward, BF16x3 input and weight gradients: the bench's headline mode)
and BF16x3 modes.

The GPU runs the whole batch the way bench.py does: its own harmonic source (no
har passed), the full-size workspace plan, several persistent tiles per CTA and
the split counts of a 16-clip batch. The upstream gradient is non-zero only on
clips 0 and 15, so the weight gradients of the batch equal those of a 2-clip
batch, which the float64 oracle computes from the same bytes. The oracle is
given the engine's har for those two clips (the bsml_harmonic_source atom runs
the same kernels on the same F0: bitwise the same har). The har itself is held
to the reference's arithmetic in test_gpu_parity.py::test_harmonic_source at
this clip length; the decoder comparison needs identical har bytes because its
angle channels are atan2 of exactly-zero bins in unvoiced frames (rounding
noise in any implementation).

Bars (rel-L2 against the float64 answer; per tensor, the denominator floored at
1e-3 of the global gradient norm, since biases that feed an instance norm have
an exactly-zero true gradient):
  TF32x3, TF32x3W, TF32x3F: audio, whole gradient vector, d_style <= 1e-4 (the 3xTF32 bar);
          d_asr and every gradient tensor <= 1e-3
  BF16x3: all of the above <= 2e-2
d_asr and the backbone's tensors sit at the end of the whole backward chain, where
fp32 rounding has accumulated most: on these two clips the fp32 CPU restatement
(oracle/kokoro_oracle.cpp in float) is itself 3.4e-3 from the float64 answer on
d_asr, 1.5e-3 on the whole gradient and up to 3.7e-3 on single backbone tensors,
so 1e-3 there is tighter than fp32 arithmetic alone guarantees.
"""

import ctypes

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from brosoundml_b200 import config, synth  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402
from tests.helpers import per_tensor_rel, rel_l2  # noqa: E402

B, T = 16, 200
CLIPS = [0, 15]
# (audio / grads / d_style, d_asr and per tensor)
BARS = {"tf32x3": (1e-4, 1e-3), "tf32x3w": (1e-4, 1e-3), "tf32x3f": (1e-4, 1e-3), "bf16x3": (2e-2, 2e-2)}


@pytest.fixture(scope="module")
def case():
    import torch

    from brosoundml_b200 import _lib

    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, B, T, 1)
    S = config.audio_len(cfg, T)
    da = np.zeros((B, S), np.float32)
    rng = np.random.default_rng(7)
    for b in CLIPS:
        da[b] = rng.normal(0, 1e-3, S).astype(np.float32)
    # the engine's har for the two clips
    lw = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.weight")["offset"]
    lb = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.bias")["offset"]
    pd = torch.tensor(params, device="cuda")
    f0 = torch.tensor(np.ascontiguousarray(x["F0"][CLIPS]), device="cuda")
    har = torch.empty((len(CLIPS), cfg["har_ch"], config.har_frames(cfg, T)), device="cuda")
    c = _lib.make_config(cfg)
    _lib.check(_lib.lib().bsml_harmonic_source(ctypes.byref(c), ctypes.c_void_p(f0.data_ptr()), len(CLIPS), 2 * T,
                                               ctypes.c_void_p(pd.data_ptr() + 4 * lw),
                                               ctypes.c_void_p(pd.data_ptr() + 4 * lb),
                                               ctypes.c_void_p(har.data_ptr()),
                                               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    har_h = har.cpu().numpy()
    xs = {k: np.ascontiguousarray(v[CLIPS]) for k, v in x.items()}
    r64 = o.run(params, xs["asr"], xs["F0"], xs["N"], xs["style"], har=har_h, daudio=da[CLIPS], dtype=np.float64)
    return dict(cfg=cfg, o=o, params=params, x=x, da=da, r64=r64)


@pytest.mark.parametrize("math", ["tf32x3", "tf32x3w", "tf32x3f", "bf16x3"])
def test_config2_whole_decoder(case, math):
    import torch

    from brosoundml_b200 import _lib
    from brosoundml_b200.decoder import Decoder

    cfg, o, r64 = case["cfg"], case["o"], case["r64"]
    d = Decoder(cfg, 0, math=math)
    t = {k: torch.tensor(v, device="cuda") for k, v in case["x"].items()}
    audio = d.forward(torch.tensor(case["params"], device="cuda"), t["asr"], t["F0"], t["N"], t["style"])
    g = d.backward(torch.tensor(case["da"], device="cuda"))
    torch.cuda.synchronize()
    assert _lib.lib().bsml_device_error() == 0
    a = audio.cpu().numpy()
    grads = g["grads"].cpu().numpy()
    d_asr, d_style = g["d_asr"].cpu().numpy(), g["d_style"].cpu().numpy()
    whole, per = BARS[math]
    errs = dict(audio=rel_l2(a[CLIPS], r64["audio"]), grads=rel_l2(grads, r64["grads"]),
                d_asr=rel_l2(d_asr[CLIPS], r64["d_asr"]), d_style=rel_l2(d_style[CLIPS], r64["d_style"]))
    pt = per_tensor_rel(o.table, grads, r64["grads"])
    worst = sorted(pt.items(), key=lambda kv: -kv[1])[:4]
    print(f"config 2 {math}: {errs}; worst tensors {worst}")
    for k, v in errs.items():
        assert v < (per if k == "d_asr" else whole), (k, v)
    assert worst[0][1] < per, worst
    # clips without an upstream gradient get exactly none
    others = [b for b in range(B) if b not in CLIPS]
    assert not d_asr[others].any() and not d_style[others].any()
    assert np.isfinite(a).all()
    del d
