"""CPU tests of the oracle itself.

1. The hand-written C++ oracle equals an independent PyTorch autograd model of
   the same decoder (forward audio, every parameter gradient, d_asr, d_style and
   the per-AdaIN (dGamma, dBeta) the reference trains on), in float64.
2. The reference's finite-difference methodology
   (tests/test_kokoro_decoder_backward.cpp:79-117): per-element central FD for
   the AdaIN affine and the iSTFT head, directional <g, v> checks for the
   instance-norm stacks — here in float64, so the tolerances are tight.
"""

import numpy as np
import pytest
import torch

from brosoundml_b200 import config, synth
from oracle.oracle import Oracle
from oracle.torch_decoder import TorchDecoder, harmonic_source_torch
from tests.helpers import per_tensor_rel, random_params, rel_l2


def _torch_run(cfg, o, p, x, har, da):
    td = TorchDecoder(cfg, o.table, p)
    asr = torch.tensor(x["asr"], dtype=torch.float64, requires_grad=True)
    sty = torch.tensor(x["style"], dtype=torch.float64, requires_grad=True)
    audio = td.forward(asr, torch.tensor(x["F0"], dtype=torch.float64), torch.tensor(x["N"], dtype=torch.float64),
                       sty, torch.tensor(har))
    for t in td.aff_list:
        t.retain_grad()
    audio.backward(torch.tensor(da))
    daff = np.concatenate([a.grad.numpy().reshape(-1) for a in td.reorder_affines()])
    return audio.detach().numpy(), td.grads_flat(o.n_params), asr.grad.numpy(), sty.grad.numpy(), daff


@pytest.mark.parametrize("which", ["miniature", "kokoro"])
def test_oracle_matches_torch_autograd(which):
    torch.set_num_threads(4)
    if which == "miniature":
        cfg, B, T, frames = config.miniature(), 2, 4, 33
    else:
        cfg, B, T = config.kokoro_82m(), 2, 4
        frames = config.har_frames(cfg, T)
    o = Oracle(cfg)
    p = random_params(o.table, o.n_params, 3) if which == "miniature" else \
        synth.init_params(o.table, o.n_params, 0).astype(np.float64)
    x = synth.make_inputs(cfg, B, T, 1)
    har = np.random.default_rng(5).uniform(-0.4, 0.4, (B, cfg["har_ch"], frames))
    S = cfg["hop"] * (frames - 1)
    da = np.random.default_rng(7).normal(0, 1, (B, S))
    r = o.run(p, x["asr"], x["F0"], x["N"], x["style"], har=har, daudio=da, dtype=np.float64)
    audio, g, dasr, dsty, daff = _torch_run(cfg, o, p, x, har, da)
    tol = 1e-12 if which == "miniature" else 1e-6
    assert rel_l2(r["audio"], audio) < tol
    assert rel_l2(r["grads"], g) < tol
    assert rel_l2(r["d_asr"], dasr) < tol
    assert rel_l2(r["d_style"], dsty) < tol
    assert rel_l2(r["d_aff"], daff) < tol
    worst = max(per_tensor_rel(o.table, r["grads"], g).values())
    assert worst < 100 * tol


def test_harmonic_source_matches_closed_form():
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    p = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, 2, 8, 1)
    h1 = o.harmonic_source(p, x["F0"])
    lw = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.weight")
    lb = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.bias")
    h2 = harmonic_source_torch(x["F0"], p[lw["offset"]:lw["offset"] + 9], p[lb["offset"]:lb["offset"] + 1], cfg)
    nf = cfg["n_fft"] // 2 + 1
    assert h1.shape == (2, 22, config.har_frames(cfg, 8))
    c1 = h1[:, :nf] * np.exp(1j * h1[:, nf:])
    c2 = h2[:, :nf] * np.exp(1j * h2[:, nf:])
    # fp32 running phase sum (reference) vs float64 closed form
    assert np.linalg.norm(c1 - c2) / np.linalg.norm(c2) < 1e-4


# ── finite differences (reference methodology, float64) ─────────────────────

def _fd_dir(loss, P, grad, rng, h=1e-5):
    v = rng.uniform(-1, 1, P.shape)
    saved = P.copy()
    P[...] = saved + h * v
    lp = loss()
    P[...] = saved - h * v
    lm = loss()
    P[...] = saved
    return float((grad * v).sum()), (lp - lm) / (2 * h)


def test_fd_adain_affine_per_element():
    o = Oracle(config.miniature())
    rng = np.random.default_rng(0xADA1)
    B, C, L = 1, 8, 16
    x = rng.uniform(-0.8, 0.8, (B, C, L))
    gb = np.concatenate([rng.uniform(-0.5, 0.5, (B, C)), rng.uniform(-0.4, 0.4, (B, C))], 1)
    tgt = rng.uniform(-0.5, 0.5, (B, C, L))
    y = o.adain_fwd(x, gb)
    dx, dgb = o.adain_bwd(x, gb, y - tgt)

    def loss():
        return 0.5 * float(((o.adain_fwd(x, gb) - tgt) ** 2).sum())

    h = 1e-6
    for P, G in ((x, dx), (gb, dgb)):
        flat, gflat = P.reshape(-1), G.reshape(-1)
        for i in range(flat.size):
            s = flat[i]
            flat[i] = s + h
            lp = loss()
            flat[i] = s - h
            lm = loss()
            flat[i] = s
            fd = (lp - lm) / (2 * h)
            assert abs(fd - gflat[i]) <= 1e-7 + 1e-6 * abs(fd)


def test_fd_istft_head_per_element():
    o = Oracle(config.miniature())
    rng = np.random.default_rng(0x57ED)
    B, n_fft, hop, L = 2, 16, 4, 8
    nf = n_fft // 2 + 1
    re, im = rng.normal(0, 1, (B, nf, L)), rng.normal(0, 1, (B, nf, L))
    tgt = rng.normal(0, 1, (B, hop * (L - 1)))
    a = o.istft_fwd(re, im, n_fft, hop)
    dre, dim = o.istft_bwd(a - tgt, n_fft, hop, L)

    def loss():
        return 0.5 * float(((o.istft_fwd(re, im, n_fft, hop) - tgt) ** 2).sum())

    h = 1e-6
    for P, G in ((re, dre), (im, dim)):
        flat, gflat = P.reshape(-1), G.reshape(-1)
        for i in range(flat.size):
            s = flat[i]
            flat[i] = s + h
            lp = loss()
            flat[i] = s - h
            lm = loss()
            flat[i] = s
            assert abs((lp - lm) / (2 * h) - gflat[i]) <= 1e-7 + 1e-6 * abs(gflat[i])


def test_fd_decoder_directional():
    """Directional derivative of the whole miniature decoder (MSE loss) along a
    random direction, for every parameter tensor group and the inputs — the
    reference's e2e check (tests/test_kokoro_decoder_backward.cpp:553-560),
    widened to all grads."""
    cfg = config.miniature()
    o = Oracle(cfg)
    B, T, frames = 2, 4, 33
    p = random_params(o.table, o.n_params, 11)
    x = {k: v.astype(np.float64) for k, v in synth.make_inputs(cfg, B, T, 1).items()}
    x["F0"] = np.random.default_rng(2).normal(0, 1, x["F0"].shape)
    har = np.random.default_rng(5).uniform(-0.4, 0.4, (B, 1, frames))
    tgt = np.random.default_rng(6).uniform(-0.3, 0.3, (B, 4 * (frames - 1)))

    def loss():
        a = o.run(p, x["asr"], x["F0"], x["N"], x["style"], har=har, dtype=np.float64)["audio"]
        return 0.5 * float(((a - tgt) ** 2).sum())

    a = o.run(p, x["asr"], x["F0"], x["N"], x["style"], har=har, dtype=np.float64)["audio"]
    r = o.run(p, x["asr"], x["F0"], x["N"], x["style"], har=har, daudio=a - tgt, dtype=np.float64)
    rng = np.random.default_rng(99)
    groups = {}
    for e in o.table:
        if not e["trainable"]:
            continue
        key = e["name"].split(".")[0] if not e["name"].startswith("generator") else ".".join(e["name"].split(".")[:3])
        groups.setdefault(key, []).append(e)
    for key, ents in groups.items():
        idx = np.concatenate([np.arange(e["offset"], e["offset"] + e["numel"]) for e in ents])
        view = p[idx]
        g = r["grads"][idx]
        v = rng.uniform(-1, 1, idx.size)
        h = 1e-6
        p[idx] = view + h * v
        lp = loss()
        p[idx] = view - h * v
        lm = loss()
        p[idx] = view
        an, fd = float((g * v).sum()), (lp - lm) / (2 * h)
        assert abs(an - fd) <= 1e-6 + 1e-5 * abs(fd), (key, an, fd)
    for name, grad in (("asr", r["d_asr"]), ("style", r["d_style"])):
        an, fd = _fd_dir(loss, x[name], grad, rng, h=1e-6)
        assert abs(an - fd) <= 1e-6 + 1e-5 * abs(fd), (name, an, fd)


def test_fd_reference_mode_affines():
    """Reference mode: (gamma, beta) supplied directly; the oracle's per-AdaIN
    grads are the derivative of the loss w.r.t. those vectors
    (kokoro_decoder_backward.h:223-231, 281-293)."""
    cfg = config.miniature()
    o = Oracle(cfg)
    B, T, frames = 1, 4, 33
    p = random_params(o.table, o.n_params, 21)
    x = {k: v.astype(np.float64) for k, v in synth.make_inputs(cfg, B, T, 1).items()}
    har = np.random.default_rng(5).uniform(-0.4, 0.4, (B, 1, frames))
    aff = np.random.default_rng(8).uniform(-0.4, 0.4, B * o.aff_per_clip)
    tgt = np.random.default_rng(6).uniform(-0.3, 0.3, (B, 4 * (frames - 1)))

    def loss():
        a = o.run(p, x["asr"], x["F0"], x["N"], x["style"], har=har, aff_in=aff, dtype=np.float64)["audio"]
        return 0.5 * float(((a - tgt) ** 2).sum())

    a = o.run(p, x["asr"], x["F0"], x["N"], x["style"], har=har, aff_in=aff, dtype=np.float64)["audio"]
    r = o.run(p, x["asr"], x["F0"], x["N"], x["style"], har=har, aff_in=aff, daudio=a - tgt, dtype=np.float64)
    an, fd = _fd_dir(loss, aff, r["d_aff"], np.random.default_rng(1), h=1e-6)
    assert abs(an - fd) <= 1e-6 + 1e-5 * abs(fd)


def test_harmonic_source_needs_matching_channels():
    """The built-in harmonic source makes n_fft + 2 channels: a config with another
    har_ch must be given har explicitly (the miniature config has har_ch = 1)."""
    cfg = config.miniature()
    o = Oracle(cfg)
    x = synth.make_inputs(cfg, 1, 4, 1)
    p = np.zeros(o.n_params, np.float32)
    with pytest.raises(ValueError):
        o.run(p, x["asr"], x["F0"], x["N"], x["style"])
