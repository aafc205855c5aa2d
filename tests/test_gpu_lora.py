"""DecoderLora on the GPU (bsml_lora_*) against the float64 oracle, plus the
reference's own LoRA properties: neutral identity at gate zero
(tests/test_kokoro_decoder_backward.cpp:516-530), Adam with one shared step,
gradient accumulation until zero_grad, and the ELRA1 checkpoint round trip
(:562-577) with its error paths (src/decoder_lora.cpp:334-382); and the conv-weight
LoRA (bsml_convlora_*, BASELINE config 3) against the float64 oracle of the folded
decoder, its zero-B identity, accumulation and Adam."""

import numpy as np
import pytest

from brosoundml_b200 import config, synth
from oracle import lora_oracle as lo
from oracle.oracle import Oracle
from tests.conftest import cuda_available
from tests.helpers import random_params, rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

RANK, SCALE = 8, 2.0


def _torch():
    import torch
    return torch


def _case(which, seed=0):
    rng = np.random.default_rng(seed)
    if which == "miniature":
        cfg, B, T, frames = config.miniature(), 2, 4, 33
        o = Oracle(cfg)
        p = random_params(o.table, o.n_params, 11).astype(np.float32)
        har = rng.uniform(-0.4, 0.4, (B, cfg["har_ch"], frames)).astype(np.float32)
    else:
        cfg, B, T = config.kokoro_82m(), 2, 32
        o = Oracle(cfg)
        p = synth.init_params(o.table, o.n_params, 0)
        # har from the caller: the GPU harmonic source forms each frame's phase exactly
        # where the reference accumulates it in fp32, so the two differ by design
        har = rng.uniform(-1, 1, (B, cfg["har_ch"], config.har_frames(cfg, T))).astype(np.float32)
    x = synth.make_inputs(cfg, B, T, 1)
    S = cfg["style_dim"]
    ref_s = np.concatenate([x["style"], rng.normal(0, 1, (B, S)).astype(np.float32)], axis=1)   # (B, 2S)
    cond = rng.normal(0, 1, (B, lo.IN_DIM)).astype(np.float32)
    return cfg, o, p, x, har, ref_s, cond


def _dev(a):
    torch = _torch()
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _make(cfg, math, seed=5, rank=RANK):
    from brosoundml_b200.decoder import Decoder
    from brosoundml_b200.lora import DecoderLora
    dec = Decoder(cfg, 0, math=math)
    return dec, DecoderLora(dec, rank=rank, scale=SCALE, seed=seed)


@pytest.mark.parametrize("which,math", [("miniature", "fp32"), ("miniature", "tf32x3"), ("kokoro", "tf32x3"),
                                        ("kokoro", "bf16x3"), ("kokoro", "tf32x3f")])
def test_lora_forward_backward_vs_oracle(which, math):
    torch = _torch()
    cfg, o, p, x, har, ref_s, cond = _case(which)
    dec, lora = _make(cfg, math)
    lay = lo.LoraLayout(o.aff_C, RANK, cfg["style_dim"])
    assert lora.n_params == lay.n_params and lora.off_A == lay.off_A and lora.off_B == lay.off_B
    lp = np.random.default_rng(3).uniform(-0.3, 0.3, lay.n_params).astype(np.float32)
    lora.params().copy_(_dev(lp))
    pd = _dev(p)
    audio = lora.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(ref_s), _dev(cond), har=_dev(har))
    da = np.random.default_rng(4).normal(0, 1, tuple(audio.shape)).astype(np.float32)
    lora.zero_grad()
    lora.backward(_dev(da))
    torch.cuda.synchronize()
    S = cfg["style_dim"]
    r = lo.run(o, lay, p.astype(np.float64), lp.astype(np.float64), x["asr"], x["F0"], x["N"], ref_s[:, :S], cond,
               SCALE, har=har, daudio=da.astype(np.float64))
    tol = 2e-2 if math == "bf16x3" else 1e-4   # the BF16 and 3xTF32 bars against float64
    assert rel_l2(audio.cpu().numpy(), r["audio"]) < tol
    g = lora.grads().cpu().numpy()
    assert rel_l2(g, r["grads"]) < tol
    for key, s in (("W1", slice(lay.off_W1, lay.off_W2)), ("W2", slice(lay.off_W2, lay.off_A[0]))):
        assert rel_l2(g[s], r["grads"][s]) < 10 * tol, key


def test_lora_neutral_identity():
    """A fresh DecoderLora has gate W2 = 0, so g(v) = 0 for any condition and the
    audio equals the base decoder's (fc(style) affines)."""
    torch = _torch()
    cfg, o, p, x, har, ref_s, cond = _case("kokoro", 1)
    dec, lora = _make(cfg, "tf32x3")
    assert float(lora.params()[lora.off_W2:lora.off_A[0]].abs().max()) == 0.0
    pd = _dev(p)
    a_lora = lora.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(ref_s), _dev(cond),
                          har=_dev(har)).clone()
    a_base = dec.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(x["style"]), har=_dev(har))
    torch.cuda.synchronize()
    assert rel_l2(a_lora.cpu().numpy(), a_base.cpu().numpy()) < 1e-5


def test_lora_adam_and_grad_accumulation():
    torch = _torch()
    cfg, o, p, x, har, ref_s, cond = _case("miniature", 2)
    dec, lora = _make(cfg, "fp32")
    lora.params()[lora.off_W2:lora.off_A[0]].uniform_(-0.3, 0.3)   # open the gate
    pd = _dev(p)
    args = (pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(ref_s), _dev(cond))
    audio = lora.forward(*args, har=_dev(har))
    da = torch.randn_like(audio)
    lora.zero_grad()
    lora.backward(da)
    g1 = lora.grads().clone()
    lora.forward(*args, har=_dev(har))
    lora.backward(da)
    torch.cuda.synchronize()
    assert torch.allclose(lora.grads(), 2 * g1, rtol=1e-6, atol=1e-12)   # accumulates until zero_grad
    lora.zero_grad()
    torch.cuda.synchronize()
    assert float(lora.grads().abs().max()) == 0.0
    lora.backward(da)
    p0, g = lora.params().clone().double(), lora.grads().clone().double()
    lr, b1, b2, eps = 1e-3, 0.9, 0.999, 1e-8
    lora.adam_step(lr, b1, b2, eps)
    torch.cuda.synchronize()
    assert lora.step == 1
    m = (1 - b1) * g
    v = (1 - b2) * g * g
    expect = p0 - lr * (m / (1 - b1)) / (torch.sqrt(v / (1 - b2)) + eps)
    assert torch.allclose(lora.params().double(), expect, rtol=1e-5, atol=1e-7)


def test_lora_checkpoint_roundtrip(tmp_path):
    torch = _torch()
    from brosoundml_b200._lib import BsmlError
    cfg = config.miniature()
    dec, lora = _make(cfg, "fp32", seed=9)
    lora.params()[lora.off_W2:lora.off_A[0]].uniform_(-0.3, 0.3)
    saved = lora.params().cpu().numpy().copy()
    path = str(tmp_path / "lora.elra")
    lora.save(path)
    # the file, read independently, holds exactly the parameters in the ELRA1 order
    rank, sd, scale, hidden, W1, W2, ads = lo.read_elra1(path)
    lay = lo.LoraLayout(lora.adapter_C, lora.rank, lora.style_dim)
    assert (rank, sd, hidden) == (lora.rank, lora.style_dim, lo.HIDDEN) and scale == np.float32(SCALE)
    assert np.array_equal(W1, lay.W1(saved)) and np.array_equal(W2, lay.W2(saved))
    assert len(ads) == lora.n_adapters
    for a, (C, A, B) in enumerate(ads):
        assert C == lora.adapter_C[a] and np.array_equal(A, lay.A(saved, a)) and np.array_equal(B, lay.B(saved, a))
    # load restores the values bit for bit
    lora.params().zero_()
    lora.load(path)
    torch.cuda.synchronize()
    assert np.array_equal(lora.params().cpu().numpy(), saved)
    # error paths: bad magic, architecture mismatch
    bad = tmp_path / "bad.elra"
    bad.write_bytes(b"NOTLORA!" + open(path, "rb").read()[8:])
    with pytest.raises(BsmlError, match="bad magic"):
        lora.load(str(bad))
    _, other = _make(cfg, "fp32", rank=4)
    with pytest.raises(BsmlError, match="architecture mismatch"):
        other.load(path)


# ── conv-weight LoRA ─────────────────────────────────────
def _make_conv(cfg, math, seed=5, rank=RANK):
    from brosoundml_b200.decoder import Decoder
    from brosoundml_b200.lora import ConvLora
    dec = Decoder(cfg, 0, math=math)
    return dec, ConvLora(dec, rank=rank, scale=SCALE, seed=seed)


@pytest.mark.parametrize("which,math", [("miniature", "fp32"), ("kokoro", "tf32x3"), ("kokoro", "tf32x3f")])
def test_conv_lora_forward_backward_vs_oracle(which, math):
    torch = _torch()
    cfg, o, p, x, har, ref_s, cond = _case(which)
    dec, cl = _make_conv(cfg, math)
    lay = lo.ConvLoraLayout(o.table, RANK)
    assert cl.n_params == lay.n_params and len(cl.weights) == len(lay.ws)
    for w, e in zip(cl.weights, lay.ws):
        assert (w["w"], w["rows"], w["cols"], w["offA"], w["offB"]) == (e["w"], e["rows"], e["cols"], e["offA"],
                                                                        e["offB"])
    lp = np.random.default_rng(3).normal(0, 0.02, lay.n_params).astype(np.float32)
    cl.params().copy_(_dev(lp))
    pd = _dev(p)
    audio = cl.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(x["style"]), har=_dev(har))
    da = np.random.default_rng(4).normal(0, 1, tuple(audio.shape)).astype(np.float32)
    cl.zero_grad()
    cl.backward(_dev(da))
    torch.cuda.synchronize()
    r = lo.conv_lora_run(o, lay, p.astype(np.float64), lp.astype(np.float64), x["asr"], x["F0"], x["N"],
                         x["style"], SCALE, har=har, daudio=da.astype(np.float64))
    tol = 1e-4   # fp32 / TF32x3 / TF32x3F against the float64 oracle
    assert rel_l2(audio.cpu().numpy(), r["audio"]) < tol
    g = cl.grads().cpu().numpy()
    assert rel_l2(g, r["grads"]) < tol
    for i in (0, len(lay.ws) // 2, len(lay.ws) - 1):
        w = lay.ws[i]
        sA, sB = slice(w["offA"], w["offB"]), slice(w["offB"], w["offB"] + w["rows"] * RANK)
        assert rel_l2(g[sA], r["grads"][sA]) < 10 * tol and rel_l2(g[sB], r["grads"][sB]) < 10 * tol, i


def test_conv_lora_starts_as_the_base_decoder():
    """B = 0 at creation: the adapted decoder equals the base decoder; A ~ N(0, 0.01)."""
    torch = _torch()
    cfg, o, p, x, har, ref_s, cond = _case("kokoro", 1)
    dec, cl = _make_conv(cfg, "tf32x3")
    P = cl.params()
    for w in cl.weights[:4]:
        assert float(P[w["offB"]:w["offB"] + w["rows"] * RANK].abs().max()) == 0.0
    A = torch.cat([P[w["offA"]:w["offB"]] for w in cl.weights])
    assert abs(float(A.std()) - 0.01) < 1e-3 and abs(float(A.mean())) < 1e-3
    pd = _dev(p)
    a_cl = cl.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(x["style"]), har=_dev(har)).clone()
    a_base = dec.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(x["style"]), har=_dev(har))
    torch.cuda.synchronize()
    assert rel_l2(a_cl.cpu().numpy(), a_base.cpu().numpy()) < 1e-6   # atomics may reorder sums


def test_conv_lora_adam_and_grad_accumulation():
    torch = _torch()
    cfg, o, p, x, har, ref_s, cond = _case("miniature", 2)
    dec, cl = _make_conv(cfg, "fp32")
    cl.params().normal_(0, 0.02)
    pd = _dev(p)
    args = (pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(x["style"]))
    audio = cl.forward(*args, har=_dev(har))
    da = torch.randn_like(audio)
    cl.zero_grad()
    cl.backward(da)
    g1 = cl.grads().clone()
    cl.forward(*args, har=_dev(har))
    cl.backward(da)
    torch.cuda.synchronize()
    assert torch.allclose(cl.grads(), 2 * g1, rtol=1e-5, atol=1e-10)
    cl.zero_grad()
    cl.backward(da)
    p0, g = cl.params().clone().double(), cl.grads().clone().double()
    lr, b1, b2, eps = 1e-3, 0.9, 0.999, 1e-8
    cl.adam_step(lr, b1, b2, eps)
    torch.cuda.synchronize()
    expect = p0 - lr * ((1 - b1) * g / (1 - b1)) / (torch.sqrt((1 - b2) * g * g / (1 - b2)) + eps)
    assert torch.allclose(cl.params().double(), expect, rtol=1e-5, atol=1e-7)


def _train_steps(obj, fwd, n, lr=1e-3):
    torch = _torch()
    for _ in range(n):
        audio = fwd()
        obj.zero_grad()
        obj.backward(torch.sin(audio * 3.0))   # a fixed, data-dependent upstream gradient
        obj.adam_step(lr)


def test_lora_full_state_resume(tmp_path):
    """save(full_state) then load(full_state) into a fresh object: the next steps
    match continuing the original (parameters, moments, shared step); the plain
    readers still read the file."""
    torch = _torch()
    cfg, o, p, x, har, ref_s, cond = _case("miniature", 3)
    dec, a = _make(cfg, "fp32", seed=4)
    a.params()[a.off_W2:a.off_A[0]].uniform_(-0.3, 0.3)
    pd = _dev(p)
    fwd_a = lambda: a.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(ref_s), _dev(cond),
                              har=_dev(har))
    _train_steps(a, fwd_a, 2)
    path = str(tmp_path / "state.elra")
    a.save(path, full_state=True)
    _, b = _make(cfg, "fp32", seed=77)
    b.load(path, full_state=True)
    torch.cuda.synchronize()
    assert b.step == a.step == 2
    assert torch.equal(a.params(), b.params())
    fwd_b = lambda: b.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(ref_s), _dev(cond),
                              har=_dev(har))
    _train_steps(a, fwd_a, 2)
    _train_steps(b, fwd_b, 2)
    torch.cuda.synchronize()
    assert b.step == 4
    assert float((a.params() - b.params()).abs().max()) <= 1e-6 * float(a.params().abs().max())
    # the plain ELRA1 readers stop before the optimiser state
    _, c = _make(cfg, "fp32", seed=5)
    c.load(path)
    rank, sd, scale, hidden, W1, W2, ads = lo.read_elra1(path)
    assert len(ads) == c.n_adapters
    # a plain ELRA1 file has no state to resume from
    a.save(str(tmp_path / "plain.elra"))
    from brosoundml_b200._lib import BsmlError
    with pytest.raises(BsmlError, match="no optimiser state"):
        c.load(str(tmp_path / "plain.elra"), full_state=True)


def test_conv_lora_state_resume(tmp_path):
    torch = _torch()
    cfg, o, p, x, har, ref_s, cond = _case("miniature", 4)
    dec, a = _make_conv(cfg, "fp32", seed=2)
    pd = _dev(p)
    fwd_a = lambda: a.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(x["style"]), har=_dev(har))
    _train_steps(a, fwd_a, 2)
    path = str(tmp_path / "conv.eclr")
    a.save(path)
    _, b = _make_conv(cfg, "fp32", seed=9)
    b.load(path)
    fwd_b = lambda: b.forward(pd, _dev(x["asr"]), _dev(x["F0"]), _dev(x["N"]), _dev(x["style"]), har=_dev(har))
    _train_steps(a, fwd_a, 2)
    _train_steps(b, fwd_b, 2)
    torch.cuda.synchronize()
    assert float((a.params() - b.params()).abs().max()) <= 1e-6 * float(a.params().abs().max())
    from brosoundml_b200._lib import BsmlError
    _, c = _make_conv(cfg, "fp32", rank=4)
    with pytest.raises(BsmlError, match="architecture mismatch"):
        c.load(path)
