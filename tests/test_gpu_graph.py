"""CUDA-graph capture and replay of library calls (bsml_graph_*): a forward, L1
loss and backward recorded once and replayed must give the eager results, also
after new data is written into the captured input buffers."""

import numpy as np
import pytest

from brosoundml_b200 import config, synth
from tests.conftest import cuda_available
from tests.helpers import rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


@pytest.mark.parametrize("which,math", [("miniature", "fp32"), ("kokoro", "tf32x3")])
def test_graph_replay_matches_eager(which, math):
    import torch

    from brosoundml_b200.decoder import Decoder, Graph, l1_loss

    if which == "miniature":
        cfg, B, T = config.miniature(), 2, 4
    else:
        cfg, B, T = config.kokoro_82m(), 1, 32
    dec = Decoder(cfg, 0, math=math)
    rng = np.random.default_rng(0)
    params = torch.tensor(synth.init_params(dec.table, dec.n_params, 0), device="cuda")
    frames = (2 * T * cfg["upsample_scale"]) // cfg["hop"] + 1

    def inputs(seed):
        x = synth.make_inputs(cfg, B, T, seed)
        r = np.random.default_rng(seed)
        har = r.uniform(-0.4, 0.4, (B, cfg["har_ch"], frames)).astype(np.float32)
        tgt = r.uniform(-0.1, 0.1, (B, dec.audio_len(T, frames))).astype(np.float32)
        return {k: torch.tensor(v, device="cuda") for k, v in dict(x, har=har, tgt=tgt).items()}

    buf = inputs(1)
    audio = torch.empty((B, dec.audio_len(T, frames)), device="cuda")
    loss, da = torch.empty(1, device="cuda"), torch.empty_like(audio)
    grads = torch.empty(dec.n_params, device="cuda")
    d_asr = torch.empty_like(buf["asr"])
    d_style = torch.empty_like(buf["style"])
    s = torch.cuda.Stream()

    def step():
        dec.forward(params, buf["asr"], buf["F0"], buf["N"], buf["style"], har=buf["har"], audio=audio)
        l1_loss(audio, buf["tgt"], loss, da)
        dec.backward(da, grads=grads, d_asr=d_asr, d_style=d_style)

    def snapshot():
        torch.cuda.synchronize()
        return [t.clone() for t in (audio, loss, grads, d_asr, d_style)]

    with torch.cuda.stream(s):
        step()                      # eager: plans the workspace
    ref1 = snapshot()
    g = Graph(s)
    with g:
        step()
    assert g.kernels > 50
    for t in (audio, grads):
        t.zero_()
    torch.cuda.synchronize()
    g.replay(s)
    got1 = snapshot()
    tol = 1e-6 if math == "fp32" else 1e-5   # double-atomic sums may add in another order
    for a, b in zip(got1, ref1):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < tol
    # new data in the same buffers: the replay follows it
    new = inputs(2)
    for k in buf:
        buf[k].copy_(new[k])
    g.replay(s)
    got2 = snapshot()
    with torch.cuda.stream(s):
        step()
    ref2 = snapshot()
    assert rel_l2(got2[0].cpu().numpy(), got1[0].cpu().numpy()) > 1e-3   # the data did change
    for a, b in zip(got2, ref2):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < tol


def test_graph_needs_a_stream():
    from brosoundml_b200 import _lib
    assert _lib.lib().bsml_graph_begin(None) != 0
    assert "legacy default stream" in _lib.lib().bsml_last_error().decode()


def test_decode_back_half_inference():
    """bsml_decoder_decode = Kokoro::Impl::decode_back_half batched: ref_s rows of
    2*style_dim (the decoder reads the first half), the harmonic source from F0;
    equal to the forward given style = ref_s[:, :style_dim] and replayable as a
    CUDA graph. (Against the oracle it is compared with har given: the phase
    channels of har are angles, whose +-pi branch cut turns rounding-level
    differences of the two harmonic sources into jumps, test_gpu_parity.py.)"""
    import torch

    from brosoundml_b200.decoder import Decoder, Graph

    cfg, B, T = config.kokoro_82m(), 2, 32
    S = cfg["style_dim"]
    dec = Decoder(cfg, 0, math="tf32x3")
    params = torch.tensor(synth.init_params(dec.table, dec.n_params, 0), device="cuda")
    x = synth.make_inputs(cfg, B, T, 1)
    ref_s = np.concatenate([x["style"], np.random.default_rng(5).normal(0, 1, (B, S)).astype(np.float32)], axis=1)
    dv = {k: torch.tensor(v, device="cuda") for k, v in x.items()}
    rs = torch.tensor(ref_s, device="cuda")
    a_dec = dec.decode(params, rs, dv["asr"], dv["F0"], dv["N"]).clone()
    a_fwd = dec.forward(params, dv["asr"], dv["F0"], dv["N"], rs[:, :S].contiguous()).clone()
    torch.cuda.synchronize()
    assert rel_l2(a_dec.cpu().numpy(), a_fwd.cpu().numpy()) < 1e-6
    # inference as a replayed graph on a side stream
    s = torch.cuda.Stream()
    out = torch.empty_like(a_dec)
    with torch.cuda.stream(s):
        dec.decode(params, rs, dv["asr"], dv["F0"], dv["N"], audio=out)
    g = Graph(s)
    with g:
        dec.decode(params, rs, dv["asr"], dv["F0"], dv["N"], audio=out)
    out.zero_()
    torch.cuda.synchronize()
    g.replay(s)
    torch.cuda.synchronize()
    assert rel_l2(out.cpu().numpy(), a_dec.cpu().numpy()) < 1e-5
