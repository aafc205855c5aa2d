"""GPU parity: every C-ABI entry point against the CPU oracle on the same seeded inputs.

Tolerances (rel-L2 per tensor, gradient tensors floored at 1e-3 of the global
gradient norm because biases feeding an instance norm have a zero true gradient):
  fp32 CUDA-core path  ......... 1e-5 (atoms), 1e-4 (whole decoder)
  tf32x3 tensor-core path ...... 1e-4 (the bar the north star sets)
  bf16x3 tensor-core path ...... 2e-2 (BASELINE's BF16 bar)
  bf16 (one product) ........... audio 2e-2, gradients 1.5e-1: an opt-in fast mode
                                 that is not one of BASELINE's modes (its gradients
                                 miss the 2e-2 BF16 bar)
"""

import ctypes

import numpy as np
import pytest

from tests.conftest import cuda_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA GPU")]

if cuda_available():
    import torch

    from brosoundml_b200 import _lib
    from brosoundml_b200.decoder import Decoder, adam_step, l1_loss

from brosoundml_b200 import config, synth
from oracle.oracle import Oracle
from tests.helpers import per_tensor_rel, random_params, rel_l2

TOL = {"fp32": 1e-4, "tf32x3": 1e-4, "tf32x3w": 1e-4, "tf32x3f": 1e-4, "bf16": 2e-2}
# BF16 operands (8-bit mantissa) through this random-init decoder: the audio stays
# within ~1e-2 but gradients drift by ~7e-2 (instance norms over short rows amplify
# operand rounding), so one-product BF16 is an opt-in fast mode with a looser, stated
# bar; BASELINE's BF16 mode is BF16x3, held to 2e-2.
BF16_GRAD_BAR = 1.5e-1


def dev(a):
    return torch.tensor(np.ascontiguousarray(a, np.float32), device="cuda")


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@pytest.fixture(scope="module")
def orc():
    return Oracle(config.miniature())


# ── atoms ────────────────────────────────────────────────────────────────────

CONV_CASES = [  # (B, Ci, L, Co, k, stride, pad, dil)
    (2, 16, 40, 24, 3, 1, 1, 1),
    (2, 128, 300, 128, 7, 1, 9, 3),
    (1, 128, 257, 128, 11, 1, 25, 5),
    (2, 1, 64, 1, 3, 2, 1, 1),        # F0_conv / N_conv
    (2, 22, 241, 256, 12, 6, 3, 1),   # noise_convs[0]
    (2, 128, 97, 22, 7, 1, 3, 1),     # conv_post
    (3, 514, 9, 70, 1, 1, 0, 1),      # 1x1 projection with odd channel counts
]


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv1d_atoms(orc, case):
    B, Ci, L, Co, k, s, p, d = case
    rng = np.random.default_rng(hash(case) % 2**32)
    x = rng.normal(0, 1, (B, Ci, L)).astype(np.float32)
    W = rng.normal(0, 0.1, (Co, Ci, k)).astype(np.float32)
    b = rng.normal(0, 0.1, Co).astype(np.float32)
    Lo = (L + 2 * p - d * (k - 1) - 1) // s + 1
    dy = rng.normal(0, 1, (B, Co, Lo)).astype(np.float32)
    lib = _lib.lib()
    y = torch.empty((B, Co, Lo), device="cuda")
    xd, Wd, bd, dyd = dev(x), dev(W), dev(b), dev(dy)
    _lib.check(lib.bsml_conv1d_forward(P(xd), B, Ci, L, P(Wd), P(bd), Co, k, s, p, d, P(y), stream()))
    assert rel_l2(host(y), orc.conv_fwd(x, W, b, s, p, d)) < 1e-5
    dW = torch.empty((Co, Ci, k), device="cuda")
    db = torch.empty(Co, device="cuda")
    _lib.check(lib.bsml_conv1d_backward_weight(P(dyd), P(xd), B, Ci, L, Co, k, s, p, d, P(dW), P(db), stream()))
    rW, rb = orc.conv_wgrad(dy, x, k, s, p, d)
    assert rel_l2(host(dW), rW) < 1e-5
    assert rel_l2(host(db), rb) < 1e-5
    if s == 1:
        dx = torch.empty((B, Ci, L), device="cuda")
        _lib.check(lib.bsml_conv1d_backward_input(P(dyd), B, Ci, L, P(Wd), Co, k, s, p, d, P(dx), stream()))
        assert rel_l2(host(dx), orc.conv_dgrad(dy, W, L, s, p, d)) < 1e-5


TC_CONV_CASES = [  # (B, Ci, L, Co, k, pad, dil): stride-1 shapes the tensor-core kernel takes
    (2, 128, 300, 128, 7, 9, 3),       # generator stage 1, dilated
    (1, 256, 517, 256, 11, 25, 5),     # generator stage 0, two M tiles, ragged N tile
    (2, 514, 37, 1024, 3, 1, 1),       # backbone encode conv1: K tail (514 = 16*32 + 2)
    (3, 1090, 20, 512, 3, 1, 1),       # decode.3 conv1: K tail, 4 M tiles
    (2, 64, 129, 96, 1, 0, 1),         # 1x1, partial M tile
    (8, 128, 24000, 128, 7, 9, 3),     # several 256-position tiles per persistent CTA
    (16, 96, 3000, 128, 3, 1, 1),      # odd promotion-group count per tile, two tiles on some CTAs
    (1, 1024, 64, 1024, 3, 1, 1),      # config-0 backbone: 8 output tiles, K split over idle SMs
]
# tf32x3 with promoted accumulation is fp32-grade; bf16 is one bf16 product; tf32x3w
# runs the forward and input gradients as tf32x3 and the weight gradients as bf16x3;
# tf32x3f the forward as tf32x3 and both gradients as bf16x3
TC_TOL = {"tf32x3": 1e-5, "bf16x3": 1e-4, "bf16": 1e-2}
FWD_TOL = dict(TC_TOL, tf32x3w=TC_TOL["tf32x3"], tf32x3f=TC_TOL["tf32x3"])
DG_TOL = dict(TC_TOL, tf32x3w=TC_TOL["tf32x3"], tf32x3f=TC_TOL["bf16x3"])
WG_TOL = dict(TC_TOL, tf32x3w=TC_TOL["bf16x3"], tf32x3f=TC_TOL["bf16x3"])


@pytest.fixture
def atom_math():
    def set_(m):
        _lib.check(_lib.lib().bsml_set_atom_math({"fp32": 0, "tf32x3": 1, "bf16": 2, "bf16x3": 3, "tf32x3w": 4,
                                                  "tf32x3f": 5}[m]))
    yield set_
    set_("fp32")


@pytest.mark.parametrize("math", ["tf32x3", "bf16x3", "bf16", "tf32x3f"])
@pytest.mark.parametrize("case", TC_CONV_CASES)
def test_tc_conv_atoms(orc, atom_math, math, case):
    """tcgen05 implicit-GEMM forward and input-gradient convs against the oracle."""
    B, Ci, L, Co, k, p, d = case
    rng = np.random.default_rng(abs(hash(case)) % 2**32)
    x = rng.normal(0, 1, (B, Ci, L)).astype(np.float32)
    W = rng.normal(0, 0.1, (Co, Ci, k)).astype(np.float32)
    b = rng.normal(0, 0.1, Co).astype(np.float32)
    Lo = L + 2 * p - d * (k - 1)
    dy = rng.normal(0, 1, (B, Co, Lo)).astype(np.float32)
    lib = _lib.lib()
    atom_math(math)
    xd, Wd, bd, dyd = dev(x), dev(W), dev(b), dev(dy)
    y = torch.empty((B, Co, Lo), device="cuda")
    _lib.check(lib.bsml_conv1d_forward(P(xd), B, Ci, L, P(Wd), P(bd), Co, k, 1, p, d, P(y), stream()))
    assert rel_l2(host(y), orc.conv_fwd(x, W, b, 1, p, d)) < FWD_TOL[math]
    dx = torch.empty((B, Ci, L), device="cuda")
    _lib.check(lib.bsml_conv1d_backward_input(P(dyd), B, Ci, L, P(Wd), Co, k, 1, p, d, P(dx), stream()))
    assert rel_l2(host(dx), orc.conv_dgrad(dy, W, L, 1, p, d)) < DG_TOL[math]
    assert lib.bsml_device_error() == 0


@pytest.mark.parametrize("math", ["tf32x3", "bf16x3", "bf16", "tf32x3w", "tf32x3f"])
@pytest.mark.parametrize("case", TC_CONV_CASES + [(3, 128, 1000, 128, 11, 25, 5)])
def test_tc_wgrad_atoms(orc, atom_math, math, case):
    """tcgen05 weight gradient (MN-major operands, split-K) against the oracle."""
    B, Ci, L, Co, k, p, d = case
    rng = np.random.default_rng(abs(hash(case)) % 2**32 + 1)
    x = rng.normal(0, 1, (B, Ci, L)).astype(np.float32)
    Lo = L + 2 * p - d * (k - 1)
    dy = rng.normal(0, 1, (B, Co, Lo)).astype(np.float32)
    atom_math(math)
    xd, dyd = dev(x), dev(dy)
    dW = torch.empty((Co, Ci, k), device="cuda")
    db = torch.empty(Co, device="cuda")
    _lib.check(_lib.lib().bsml_conv1d_backward_weight(P(dyd), P(xd), B, Ci, L, Co, k, 1, p, d, P(dW), P(db),
                                                      stream()))
    rW, rb = orc.conv_wgrad(dy, x, k, 1, p, d)
    assert rel_l2(host(dW), rW) < WG_TOL[math]
    assert rel_l2(host(db), rb) < 1e-5
    assert _lib.lib().bsml_device_error() == 0


@pytest.mark.parametrize("math", ["tf32x3", "bf16x3", "bf16", "tf32x3w", "tf32x3f"])
@pytest.mark.parametrize("case", [(2, 512, 40, 256, 20, 10, 5), (2, 256, 100, 128, 12, 6, 3),
                                  (16, 256, 400, 128, 12, 6, 3)])
def test_tc_convT_atoms(orc, atom_math, math, case):
    """ConvTranspose1d on the tcgen05 kernels: forward by stride phases (strided output
    rows); input and weight gradients as stride-1 problems over the row-packed dy."""
    B, Ci, L, Co, k, s, p = case
    rng = np.random.default_rng(5 + k)
    x = rng.normal(0, 1, (B, Ci, L)).astype(np.float32)
    W = rng.normal(0, 0.05, (Ci, Co, k)).astype(np.float32)
    b = rng.normal(0, 0.1, Co).astype(np.float32)
    Lu = (L - 1) * s - 2 * p + k
    dy = rng.normal(0, 1, (B, Co, Lu)).astype(np.float32)
    lib = _lib.lib()
    atom_math(math)
    xd, Wd, bd, dyd = dev(x), dev(W), dev(b), dev(dy)
    y = torch.empty((B, Co, Lu), device="cuda")
    _lib.check(lib.bsml_conv_transpose1d_forward(P(xd), B, Ci, L, P(Wd), P(bd), Co, k, s, p, P(y), stream()))
    assert rel_l2(host(y), orc.convT_fwd(x, W, b, s, p)) < FWD_TOL[math]
    dx = torch.empty((B, Ci, L), device="cuda")
    _lib.check(lib.bsml_conv_transpose1d_backward_input(P(dyd), B, Ci, L, P(Wd), Co, k, s, p, P(dx), stream()))
    assert rel_l2(host(dx), orc.convT_dgrad(dy, W, L, s, p)) < DG_TOL[math]
    dW = torch.empty((Ci, Co, k), device="cuda")
    db = torch.empty(Co, device="cuda")
    _lib.check(lib.bsml_conv_transpose1d_backward_weight(P(dyd), P(xd), B, Ci, L, Co, k, s, p, P(dW), P(db),
                                                          stream()))
    rW, rb = orc.convT_wgrad(dy, x, k, s, p)
    assert rel_l2(host(dW), rW) < WG_TOL[math]
    assert rel_l2(host(db), rb) < 1e-5
    assert lib.bsml_device_error() == 0


CONVT_CASES = [  # (B, Ci, L, Co, k, stride, pad)
    (2, 64, 12, 32, 20, 10, 5),    # ups[0] shape family
    (2, 32, 30, 16, 12, 6, 3),     # ups[1]
    (3, 8, 8, 4, 4, 2, 1),         # reference miniature
]


@pytest.mark.parametrize("case", CONVT_CASES)
def test_conv_transpose1d_atoms(orc, case):
    B, Ci, L, Co, k, s, p = case
    rng = np.random.default_rng(7 + k)
    x = rng.normal(0, 1, (B, Ci, L)).astype(np.float32)
    W = rng.normal(0, 0.1, (Ci, Co, k)).astype(np.float32)
    b = rng.normal(0, 0.1, Co).astype(np.float32)
    Lu = (L - 1) * s - 2 * p + k
    dy = rng.normal(0, 1, (B, Co, Lu)).astype(np.float32)
    lib = _lib.lib()
    xd, Wd, bd, dyd = dev(x), dev(W), dev(b), dev(dy)
    y = torch.empty((B, Co, Lu), device="cuda")
    _lib.check(lib.bsml_conv_transpose1d_forward(P(xd), B, Ci, L, P(Wd), P(bd), Co, k, s, p, P(y), stream()))
    assert rel_l2(host(y), orc.convT_fwd(x, W, b, s, p)) < 1e-5
    dx = torch.empty((B, Ci, L), device="cuda")
    _lib.check(lib.bsml_conv_transpose1d_backward_input(P(dyd), B, Ci, L, P(Wd), Co, k, s, p, P(dx), stream()))
    assert rel_l2(host(dx), orc.convT_dgrad(dy, W, L, s, p)) < 1e-5
    dW = torch.empty((Ci, Co, k), device="cuda")
    db = torch.empty(Co, device="cuda")
    _lib.check(lib.bsml_conv_transpose1d_backward_weight(P(dyd), P(xd), B, Ci, L, Co, k, s, p, P(dW), P(db),
                                                          stream()))
    rW, rb = orc.convT_wgrad(dy, x, k, s, p)
    assert rel_l2(host(dW), rW) < 1e-5
    assert rel_l2(host(db), rb) < 1e-5


@pytest.mark.parametrize("shape", [(1, 8, 16), (3, 130, 1001)])
def test_adain_snake_atoms(orc, shape):
    B, C, L = shape
    rng = np.random.default_rng(11)
    x = rng.normal(0.3, 1.5, (B, C, L)).astype(np.float32)
    gb = rng.uniform(-0.5, 0.5, (B, 2 * C)).astype(np.float32)
    dy = rng.normal(0, 1, (B, C, L)).astype(np.float32)
    alpha = rng.uniform(0.5, 1.5, C).astype(np.float32)
    lib = _lib.lib()
    xd, gbd, dyd, ad = dev(x), dev(gb), dev(dy), dev(alpha)
    y = torch.empty_like(xd)
    _lib.check(lib.bsml_adain_affine_forward(P(xd), P(gbd), B, C, L, 1e-5, P(y), stream()))
    assert rel_l2(host(y), orc.adain_fwd(x, gb)) < 1e-5
    dx = torch.empty_like(xd)
    dgb = torch.empty_like(gbd)
    _lib.check(lib.bsml_adain_affine_backward(P(xd), P(gbd), P(dyd), B, C, L, 1e-5, P(dx), P(dgb), stream()))
    rdx, rdgb = orc.adain_bwd(x, gb, dy)
    assert rel_l2(host(dx), rdx) < 1e-5
    assert rel_l2(host(dgb), rdgb) < 1e-5
    _lib.check(lib.bsml_snake_forward(P(xd), P(ad), B, C, L, P(y), stream()))
    assert rel_l2(host(y), orc.snake_fwd(x, alpha)) < 1e-5
    da = torch.empty(C, device="cuda")
    _lib.check(lib.bsml_snake_backward(P(xd), P(ad), P(dyd), B, C, L, P(dx), P(da), stream()))
    rdx, rda = orc.snake_bwd(x, alpha, dy)
    assert rel_l2(host(dx), rdx) < 1e-5
    assert rel_l2(host(da), rda) < 1e-5


@pytest.mark.parametrize("n_fft,hop,L", [(20, 5, 241), (8, 4, 17), (16, 4, 9)])
def test_istft_atoms(orc, n_fft, hop, L):
    B = 2
    nf = n_fft // 2 + 1
    rng = np.random.default_rng(n_fft)
    re, im = rng.normal(0, 1, (B, nf, L)).astype(np.float32), rng.normal(0, 1, (B, nf, L)).astype(np.float32)
    da = rng.normal(0, 1, (B, hop * (L - 1))).astype(np.float32)
    lib = _lib.lib()
    # keep every device tensor referenced while the library reads it
    red, imd, dad = dev(re), dev(im), dev(da)
    a = torch.empty((B, hop * (L - 1)), device="cuda")
    _lib.check(lib.bsml_istft_forward(P(red), P(imd), B, n_fft, hop, L, P(a), stream()))
    assert rel_l2(host(a), orc.istft_fwd(re, im, n_fft, hop)) < 1e-5
    dre = torch.empty((B, nf, L), device="cuda")
    dim = torch.empty((B, nf, L), device="cuda")
    _lib.check(lib.bsml_istft_backward(P(dad), B, n_fft, hop, L, P(dre), P(dim), stream()))
    rre, rim = orc.istft_bwd(da, n_fft, hop, L)
    assert rel_l2(host(dre), rre) < 1e-5
    assert rel_l2(host(dim), rim) < 1e-5


def _har_gpu(cfg, o, p, F0, mode):
    lw = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.weight")["offset"]
    lb = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.bias")["offset"]
    B, F = F0.shape
    pd, f0d = dev(p), dev(F0)
    har = torch.empty((B, cfg["har_ch"], config.har_frames(cfg, F // 2)), device="cuda")
    c = _lib.make_config(cfg)
    _lib.check(_lib.lib().bsml_harmonic_source_mode(ctypes.byref(c), P(f0d), B, F,
                                                    ctypes.c_void_p(pd.data_ptr() + 4 * lw),
                                                    ctypes.c_void_p(pd.data_ptr() + 4 * lb), P(har),
                                                    {"fp32": 0, "exact": 1}[mode], stream()))
    return host(har)


def _spectrum(h, nf):
    return h[:, :nf] * np.exp(1j * h[:, nf:].astype(np.float64))


# The reference's phase is an fp32 running sum (kokoro_modules.cpp:1601-1616); the
# default GPU mode reproduces its every rounding, so only the sines, the mixture and
# the STFT sums differ (a few fp32 ulps). Compared on the complex spectrum |X| e^{i angle X}:
# the angle channels alone are atan2 of bins that are exactly zero in unvoiced
# stretches (a constant source under a periodic Hann window), i.e. rounding noise in
# any implementation. T=200 is config 2's clip length, T=1600 config 4's longest.
HAR_BAR = 1e-5


@pytest.mark.parametrize("T", [16, 200, 1600])
def test_harmonic_source(T):
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    p = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, 2, T, 1)
    ref = o.harmonic_source(p, x["F0"])
    h = _har_gpu(cfg, o, p, x["F0"], "fp32")
    nf = cfg["n_fft"] // 2 + 1
    c1, c2 = _spectrum(h, nf), _spectrum(ref, nf)
    assert np.linalg.norm(c1 - c2) / np.linalg.norm(c2) < HAR_BAR
    assert rel_l2(h[:, :nf], ref[:, :nf]) < HAR_BAR


def test_harmonic_source_exact_phase_mode():
    """The double-precision phase mode is an accurate sine source, close to the
    reference's on short clips (its fp32 phase has drifted little by then)."""
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    p = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, 2, 16, 1)
    ref = o.harmonic_source(p, x["F0"])
    h = _har_gpu(cfg, o, p, x["F0"], "exact")
    nf = cfg["n_fft"] // 2 + 1
    c1, c2 = _spectrum(h, nf), _spectrum(ref, nf)
    assert np.linalg.norm(c1 - c2) / np.linalg.norm(c2) < 1e-4


def test_l1_and_adam():
    rng = np.random.default_rng(3)
    a = rng.normal(0, 1, 1000).astype(np.float32)
    t = rng.normal(0, 1, 1000).astype(np.float32)
    loss, da = l1_loss(dev(a), dev(t))
    assert abs(float(host(loss)[0]) - np.abs(a - t).mean()) < 1e-6
    assert np.array_equal(host(da), (np.sign(a - t) / a.size).astype(np.float32))
    p, g = rng.normal(0, 1, 500).astype(np.float32), rng.normal(0, 1, 500).astype(np.float32)
    pd, gd, m, v = dev(p), dev(g), torch.zeros(500, device="cuda"), torch.zeros(500, device="cuda")
    pr, mr, vr = p.astype(np.float64), np.zeros(500), np.zeros(500)
    for step in (1, 2, 3):
        adam_step(pd, gd, m, v, 1e-2, step)
        mr = 0.9 * mr + 0.1 * g
        vr = 0.999 * vr + 0.001 * g.astype(np.float64) ** 2
        pr -= 1e-2 * (mr / (1 - 0.9 ** step)) / (np.sqrt(vr / (1 - 0.999 ** step)) + 1e-8)
    assert rel_l2(host(pd), pr) < 1e-6


# ── whole decoder ────────────────────────────────────────────────────────────
#
# The exact answer is the float64 oracle. With random N(0, 0.02) weights and
# instance norms over short rows these decoders are ill-conditioned in fp32: the
# fp32 oracle itself sits up to ~1e-3 (per tensor, 1e-2 at T=3) from the float64
# one. So each GPU tensor must be as close to the float64 answer as the fp32 CPU
# restatement is (within FACTOR x its error, or under the absolute bar), and the
# whole gradient vector must meet the rel-L2 bar at realistic lengths.

FACTOR = 4.0


def _run_both(cfg, B, T, params, har=None, aff_in=None, math="fp32", seed=1, f64=True):
    o = Oracle(cfg)
    x = synth.make_inputs(cfg, B, T, seed)
    r = o.run(params, x["asr"], x["F0"], x["N"], x["style"], har=har, aff_in=aff_in, want_aff=True)
    da = np.random.default_rng(99).normal(0, 1e-3, r["audio"].shape).astype(np.float32)
    r = o.run(params, x["asr"], x["F0"], x["N"], x["style"], har=har, aff_in=aff_in, daudio=da, want_aff=True)
    r64 = None
    if f64:
        r64 = o.run(params, x["asr"], x["F0"], x["N"], x["style"], har=har, aff_in=aff_in, daudio=da, want_aff=True,
                    dtype=np.float64)
    d = Decoder(cfg, math=math)
    aff_out = torch.empty(B * d.aff_per_clip, device="cuda")
    t = {k: dev(v) for k, v in x.items()}
    pd = dev(params)
    hd = None if har is None else dev(har)
    ad = None if aff_in is None else dev(aff_in)
    dad = dev(da)
    audio = d.forward(pd, t["asr"], t["F0"], t["N"], t["style"], har=hd, aff_in=ad, aff_out=aff_out)
    g = d.backward(dad, want_aff=True)
    out = dict(audio=host(audio), aff=host(aff_out), grads=host(g["grads"]), d_asr=host(g["d_asr"]),
               d_style=host(g["d_style"]), d_aff=host(g["d_aff"]))
    return o, r, r64, out


def _check_vs_exact(o, r32, r64, got, bar):
    """Every gradient tensor within max(bar, FACTOR x fp32-oracle error) of the float64 answer."""
    e_gpu = per_tensor_rel(o.table, got["grads"], r64["grads"])
    e_32 = per_tensor_rel(o.table, r32["grads"], r64["grads"])
    bad = {k: (e_gpu[k], e_32[k]) for k in e_gpu if e_gpu[k] > max(bar, FACTOR * e_32[k])}
    assert not bad, sorted(bad.items(), key=lambda kv: -kv[1][0])[:6]
    for key in ("audio", "d_asr", "d_style", "d_aff"):
        eg, e3 = rel_l2(got[key], r64[key]), rel_l2(r32[key], r64[key])
        assert eg <= max(bar, FACTOR * e3), (key, eg, e3)


@pytest.mark.parametrize("math", ["fp32"])
def test_decoder_miniature_full(math):
    cfg = config.miniature()
    o = Oracle(cfg)
    params = random_params(o.table, o.n_params, 3).astype(np.float32)
    har = np.random.default_rng(5).uniform(-0.4, 0.4, (2, 1, 33)).astype(np.float32)
    o, r, r64, g = _run_both(cfg, 2, 4, params, har=har, math=math)
    assert rel_l2(g["aff"], r["aff"]) < 1e-6
    _check_vs_exact(o, r, r64, g, TOL[math])
    assert rel_l2(g["grads"], r64["grads"]) < TOL[math]


def test_decoder_miniature_reference_mode():
    """Reference semantics: (gamma, beta) supplied by the caller; per-AdaIN grads
    are what DecoderLora::backward consumes (decoder_lora.cpp:273-292)."""
    cfg = config.miniature()
    o = Oracle(cfg)
    params = random_params(o.table, o.n_params, 4).astype(np.float32)
    har = np.random.default_rng(6).uniform(-0.4, 0.4, (2, 1, 33)).astype(np.float32)
    aff = np.random.default_rng(8).uniform(-0.4, 0.4, 2 * o.aff_per_clip).astype(np.float32)
    o, r, r64, g = _run_both(cfg, 2, 4, params, har=har, aff_in=aff)
    assert rel_l2(g["audio"], r64["audio"]) < 1e-4
    assert rel_l2(g["d_aff"], r64["d_aff"]) < 1e-4
    assert np.all(g["d_style"] == 0)


# At a handful of frames per clip the decoder is not smooth at fp32 resolution:
# a leaky-ReLU pre-activation within rounding distance of 0 takes slope 1 in one
# implementation and 0.1/0.2 in another, and with 6-12 samples per instance-norm
# row one such flip moves a channel's gradient by ~1 %. (Two identical clips give
# bitwise-identical per-clip gradients on the GPU, so this is not an indexing
# effect; the fp32 oracle shows the same size of deviation on other clips.)
SHORT_T_BAR = 5e-2


@pytest.mark.parametrize("math", ["fp32", "tf32x3"])
@pytest.mark.parametrize("B,T", [(2, 6), (1, 3)])
def test_decoder_kokoro_short(math, B, T):
    """Kokoro-82M dimensions at very short T; the harmonic source on both sides
    is replaced by one shared har (its phase arithmetic differs by rounding and
    is tested on its own)."""
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, B, T, 1)
    har = o.harmonic_source(params, x["F0"])
    o, r, r64, g = _run_both(cfg, B, T, params, har=har, math=math)
    _check_vs_exact(o, r, r64, g, max(TOL[math], SHORT_T_BAR))
    assert rel_l2(g["audio"], r64["audio"]) < TOL[math]
    assert _lib.lib().bsml_device_error() == 0


def test_duplicate_clips_identical():
    """Two identical clips in one batch give bitwise-identical per-clip results."""
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    p = synth.init_params(o.table, o.n_params, 0)
    x1 = synth.make_inputs(cfg, 1, 6, 1)
    x = {k: np.concatenate([v, v], 0) for k, v in x1.items()}
    har = o.harmonic_source(p, x["F0"])
    d = Decoder(cfg)
    t = {k: dev(v) for k, v in x.items()}
    pd, hd = dev(p), dev(har)
    audio = d.forward(pd, t["asr"], t["F0"], t["N"], t["style"], har=hd)
    da1 = np.random.default_rng(99).normal(0, 1e-3, (1, audio.shape[1])).astype(np.float32)
    dad = dev(np.concatenate([da1, da1], 0))
    g = d.backward(dad, want_aff=True)
    a = host(audio)
    assert np.array_equal(a[0], a[1])
    daff = host(g["d_aff"])
    off = 0
    for C in o.aff_C:
        assert np.array_equal(daff[off:off + 2 * C], daff[off + 2 * C:off + 4 * C])
        off += 4 * C
    dasr = host(g["d_asr"])
    assert np.array_equal(dasr[0], dasr[1])


@pytest.mark.parametrize("math", ["bf16", "bf16x3"])
def test_decoder_kokoro_bf16(math):
    """BF16 modes at config-0 shapes. One bf16 product: audio within 2e-2, gradients
    within the stated 1.5e-1 bar. BF16x3 (hi + lo bf16 operands, three products):
    audio and gradients within BASELINE's BF16 bar of 2e-2."""
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, 1, 32, 1)
    har = o.harmonic_source(params, x["F0"])
    o, r, r64, g = _run_both(cfg, 1, 32, params, har=har, math=math)
    ea, eg = rel_l2(g["audio"], r64["audio"]), rel_l2(g["grads"], r64["grads"])
    print(f"{math}: audio {ea:.2e} grads {eg:.2e}")
    assert ea < TOL["bf16"]
    assert eg < (BF16_GRAD_BAR if math == "bf16" else TOL["bf16"])
    assert _lib.lib().bsml_device_error() == 0


@pytest.mark.parametrize("math", ["fp32", "tf32x3", "tf32x3w", "tf32x3f"])
def test_decoder_kokoro_t32(math):
    """BASELINE config 0 shapes (B=1, T=32): whole-gradient rel-L2 bar against the
    exact (float64) answer, and per tensor within the fp32 noise floor."""
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, 1, 32, 1)
    har = o.harmonic_source(params, x["F0"])
    o, r, r64, g = _run_both(cfg, 1, 32, params, har=har, math=math)
    _check_vs_exact(o, r, r64, g, max(TOL[math], 2e-3))
    assert rel_l2(g["grads"], r64["grads"]) < TOL[math]
    assert rel_l2(g["audio"], r64["audio"]) < TOL[math]
    assert _lib.lib().bsml_device_error() == 0


def test_decoder_kokoro_t100_tf32x3():
    """Longer clips (T=100, 2.5 s): tf32x3 within 1e-5 of the exact answer on the
    whole gradient vector (fp32-grade; the fp32 oracle itself is at ~2e-3 here)."""
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    params = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, 1, 100, 1)
    har = o.harmonic_source(params, x["F0"])
    o, r, r64, g = _run_both(cfg, 1, 100, params, har=har, math="tf32x3")
    assert rel_l2(g["grads"], r64["grads"]) < 1e-5
    assert rel_l2(g["audio"], r64["audio"]) < 1e-5
    assert rel_l2(g["d_asr"], r64["d_asr"]) < 1e-4


def test_decoder_kokoro_harmonic_source_inside():
    """No har supplied: the engine runs the harmonic source itself. Its output
    equals running the decoder on the bsml_harmonic_source atom's har (which is
    checked against the oracle above on the complex spectrum: the phase channels
    are atan2 of bins that are exactly zero in unvoiced stretches, i.e. rounding
    noise in any implementation, the reference's included)."""
    cfg = config.kokoro_82m()
    o = Oracle(cfg)
    B, T = 2, 8
    params = synth.init_params(o.table, o.n_params, 0)
    x = synth.make_inputs(cfg, B, T, 1)
    t = {k: dev(v) for k, v in x.items()}
    pd = dev(params)
    lw = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.weight")["offset"]
    lb = next(e for e in o.table if e["name"] == "generator.m_source.l_linear.bias")["offset"]
    frames = config.har_frames(cfg, T)
    har = torch.empty((B, cfg["har_ch"], frames), device="cuda")
    c = _lib.make_config(cfg)
    _lib.check(_lib.lib().bsml_harmonic_source(ctypes.byref(c), P(t["F0"]), B, 2 * T,
                                               ctypes.c_void_p(pd.data_ptr() + 4 * lw),
                                               ctypes.c_void_p(pd.data_ptr() + 4 * lb), P(har), stream()))
    d1, d2 = Decoder(cfg), Decoder(cfg)
    a1 = host(d1.forward(pd, t["asr"], t["F0"], t["N"], t["style"]))
    a2 = host(d2.forward(pd, t["asr"], t["F0"], t["N"], t["style"], har=har))
    assert np.array_equal(a1, a2)
