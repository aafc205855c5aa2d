"""The decoder's assemblies as separate calls (bsml_backbone_* / bsml_generator_*,
the reference's decoder_backbone_forward_train / _backward and
generator_forward_train / generator_backward, src/kokoro_decoder_backward.h:213-293)
and the spectral-head atoms (spectral_head_forward_train / _backward, :145-161).

The backbone part followed by the generator part is the whole decoder: the same
audio bit for bit, and the two backwards chained through dgen_in give the whole
decoder's gradients. The spectral head is checked against torch float64 autograd
(leaky_relu, conv1d, exp / sin, torch.istft with center=True and a periodic Hann
window: the ops the reference composes, kokoro_decoder_backward.cpp:378-458)."""

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

from brosoundml_b200 import config, synth  # noqa: E402
from oracle.oracle import Oracle  # noqa: E402
from tests.helpers import random_params, rel_l2  # noqa: E402


def _dev(a):
    import torch
    return torch.tensor(np.ascontiguousarray(a, np.float32), device="cuda")


@pytest.mark.parametrize("which,math,B,T", [("miniature", "fp32", 2, 4), ("kokoro_82m", "tf32x3", 2, 8)])
def test_parts_chain_to_the_whole_decoder(which, math, B, T):
    import torch

    from brosoundml_b200.decoder import Decoder
    cfg = getattr(config, which)()
    o = Oracle(cfg)
    params = (random_params(o.table, o.n_params, 3) if which == "miniature"
              else synth.init_params(o.table, o.n_params, 0)).astype(np.float32)
    x = synth.make_inputs(cfg, B, T, 1)
    frames = config.har_frames(cfg, T) if which == "kokoro_82m" else 33
    har = np.random.default_rng(5).uniform(-0.4, 0.4, (B, cfg["har_ch"], frames)).astype(np.float32)
    t = {k: _dev(v) for k, v in x.items()}
    pd, hd = _dev(params), _dev(har)
    full = Decoder(cfg, 0, math=math)
    audio = full.forward(pd, t["asr"], t["F0"], t["N"], t["style"], har=hd)
    da = _dev(np.random.default_rng(9).normal(0, 1e-3, tuple(audio.shape)))
    g = full.backward(da, want_aff=True)

    parts = Decoder(cfg, 0, math=math)
    gen_in = parts.forward_backbone(pd, t["asr"], t["F0"], t["N"], t["style"])
    assert gen_in.shape[2] == parts.backbone_out_len(T) == 2 * T
    audio2 = parts.forward_generator(pd, gen_in, hd, t["style"])
    torch.cuda.synchronize()
    assert torch.equal(audio, audio2)
    gg = parts.backward_generator(da, want_aff=True)
    # the backbone's caches were replaced by the generator forward: run it again
    gen_in2 = parts.forward_backbone(pd, t["asr"], t["F0"], t["N"], t["style"])
    assert torch.equal(gen_in, gen_in2)
    gb = parts.backward_backbone(gg["dgen_in"], want_aff=True)
    torch.cuda.synchronize()
    total = (gg["grads"] + gb["grads"]).cpu().numpy()
    assert rel_l2(total, g["grads"].cpu().numpy()) < 1e-6
    assert rel_l2((gg["d_aff"] + gb["d_aff"]).cpu().numpy(), g["d_aff"].cpu().numpy()) < 1e-6
    assert rel_l2(gb["d_asr"].cpu().numpy(), g["d_asr"].cpu().numpy()) < 1e-6
    assert rel_l2((gg["d_style"] + gb["d_style"]).cpu().numpy(), g["d_style"].cpu().numpy()) < 1e-6


def test_parts_reference_mode_affines():
    """Caller-supplied affines: each part reads only its own AdaINs and returns
    the gradients of its own (the others' stay zero)."""
    import torch

    from brosoundml_b200.decoder import Decoder
    cfg = config.miniature()
    o = Oracle(cfg)
    params = random_params(o.table, o.n_params, 4).astype(np.float32)
    B, T = 2, 4
    x = synth.make_inputs(cfg, B, T, 2)
    har = np.random.default_rng(6).uniform(-0.4, 0.4, (B, 1, 33)).astype(np.float32)
    aff = np.random.default_rng(8).uniform(-0.4, 0.4, B * o.aff_per_clip).astype(np.float32)
    t = {k: _dev(v) for k, v in x.items()}
    pd, hd, ad = _dev(params), _dev(har), _dev(aff)
    d = Decoder(cfg, 0)
    gen_in = d.forward_backbone(pd, t["asr"], t["F0"], t["N"], aff_in=ad)
    audio = d.forward_generator(pd, gen_in, hd, aff_in=ad)
    da = _dev(np.random.default_rng(1).normal(0, 1e-3, tuple(audio.shape)))
    gg = d.backward_generator(da, want_aff=True)
    r = o.run(params, x["asr"], x["F0"], x["N"], x["style"], har=har, aff_in=aff, daudio=da.cpu().numpy(),
              want_aff=True, dtype=np.float64)
    assert rel_l2(audio.cpu().numpy(), r["audio"]) < 1e-4
    n_bb = 2 * (1 + cfg["n_decode"])                 # backbone AdaINs come first
    bb_len = B * 2 * sum(o.aff_C[:n_bb])
    dg = gg["d_aff"].cpu().numpy()
    assert not dg[:bb_len].any()
    d.forward_backbone(pd, t["asr"], t["F0"], t["N"], aff_in=ad)
    gb = d.backward_backbone(gg["dgen_in"], want_aff=True)
    db = gb["d_aff"].cpu().numpy()
    assert not db[bb_len:].any()
    torch.cuda.synchronize()
    assert rel_l2(dg + db, r["d_aff"]) < 1e-4
    assert float(gb["d_style"].abs().max()) == 0.0


@pytest.mark.parametrize("B,C,L,n_fft,hop,k", [(2, 4, 8, 16, 4, 7), (1, 128, 241, 20, 5, 7), (3, 2, 17, 8, 4, 7)])
def test_spectral_head_atoms(B, C, L, n_fft, hop, k):
    import ctypes

    import torch

    from brosoundml_b200 import _lib
    rng = np.random.default_rng(B * 1000 + C)
    Cp = n_fft + 2
    x = rng.normal(0, 0.4, (B, C, L))
    W = rng.normal(0, 0.3 / np.sqrt(C * k), (Cp, C, k))
    b = rng.normal(0, 0.1, Cp)
    S = hop * (L - 1)
    da = rng.normal(0, 1, (B, S))
    # torch float64 reference of the head
    xt = torch.tensor(x, requires_grad=True)
    post = torch.nn.functional.conv1d(torch.nn.functional.leaky_relu(xt, 0.01), torch.tensor(W), torch.tensor(b),
                                      padding=(k - 1) // 2)
    nf = n_fft // 2 + 1
    spec = torch.polar(torch.exp(post[:, :nf]), torch.sin(post[:, nf:]))
    win = torch.hann_window(n_fft, periodic=True, dtype=torch.float64)
    audio = torch.istft(spec, n_fft, hop, n_fft, win, center=True, normalized=False, onesided=True, length=S)
    audio.backward(torch.tensor(da))
    L_ = _lib.lib()
    xd, Wd, bd, dad = _dev(x), _dev(W), _dev(b), _dev(da)
    postd = torch.empty((B, Cp, L), device="cuda")
    aud = torch.empty((B, S), device="cuda")
    dxd = torch.empty((B, C, L), device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    _lib.check(L_.bsml_spectral_head_forward(P(xd), B, C, L, P(Wd), P(bd), n_fft, hop, k, P(postd), P(aud), st))
    _lib.check(L_.bsml_spectral_head_backward(P(xd), P(postd), P(dad), B, C, L, P(Wd), n_fft, hop, k, P(dxd), st))
    torch.cuda.synchronize()
    assert rel_l2(postd.cpu().numpy(), post.detach().numpy()) < 1e-5
    assert rel_l2(aud.cpu().numpy(), audio.detach().numpy()) < 1e-5
    assert rel_l2(dxd.cpu().numpy(), xt.grad.numpy()) < 1e-5


def test_transpose_atom():
    import ctypes

    import torch

    from brosoundml_b200 import _lib
    a = torch.arange(2 * 5 * 7, dtype=torch.float32, device="cuda").reshape(2, 5, 7)
    out = torch.empty((2, 7, 5), device="cuda")
    _lib.check(_lib.lib().bsml_transpose(ctypes.c_void_p(a.data_ptr()), 2, 5, 7, ctypes.c_void_p(out.data_ptr()),
                                         ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    assert torch.equal(out, a.transpose(1, 2).contiguous())
