"""One decoder block on the GPU (bsml_block_*): the reference's block atoms
detail::adain_resblk_1d_* and detail::adain_resblock1_* (src/kokoro_decoder_backward.h:82-144)
against the float64 block oracle, in every math mode, in both affine modes; and
BASELINE config 1 (one AdaINResBlock1, [8, 128, 24000], k=7) at full size against a
plain PyTorch fp32 autograd restatement run on the same GPU (cuDNN, TF32 off)."""

import numpy as np
import pytest

from oracle.oracle import BlockOracle
from tests.conftest import cuda_available
from tests.helpers import per_tensor_rel, random_params, rel_l2

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]

TOL = {"fp32": 1e-4, "tf32x3": 1e-4, "tf32x3w": 1e-4, "tf32x3f": 1e-4, "bf16": 2e-2, "bf16x3": 2e-2}
# BF16 gradients: the same stated bar as the whole decoder's BF16 mode (operand
# rounding amplified by the instance norms); outputs keep the 2e-2 bar
BF16_GRAD_BAR = 1.5e-1
CASES = [
    # (name, spec, B, L)
    ("resblock1_C128_k7", dict(kind=2, style_dim=128, cin=128, cout=128, kernel=7, dil=[1, 3, 5]), 2, 700),
    ("resblock1_C256_k11", dict(kind=2, style_dim=128, cin=256, cout=256, kernel=11, dil=[1, 3, 5]), 1, 300),
    ("resblock1_C20_k3", dict(kind=2, style_dim=16, cin=20, cout=20, kernel=3, dil=[1, 3, 5]), 3, 97),
    ("resblk1d_decode_1090_1024", dict(kind=1, style_dim=128, cin=1090, cout=1024, upsample=0), 2, 40),
    ("resblk1d_up_1090_512", dict(kind=1, style_dim=128, cin=1090, cout=512, upsample=1), 2, 40),
    ("resblk1d_encode_514_1024", dict(kind=1, style_dim=128, cin=514, cout=1024, upsample=0), 1, 33),
    ("resblk1d_plain_64", dict(kind=1, style_dim=32, cin=64, cout=64, upsample=0), 2, 51),
]


def _torch():
    import torch
    return torch


def _dev(a):
    torch = _torch()
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def _inputs(o, B, L, seed):
    rng = np.random.default_rng(seed)
    sp = o.spec_dict
    p = random_params(o.table, o.n_params, seed, -0.1, 0.1).astype(np.float32)
    x = rng.normal(0, 1, (B, sp["cin"], L)).astype(np.float32)
    style = rng.normal(0, 1, (B, sp["style_dim"])).astype(np.float32)
    dy = rng.normal(0, 1, (B, sp["cout"], o.out_len(L))).astype(np.float32)
    return p, x, style, dy


@pytest.mark.parametrize("math", ["fp32", "tf32x3", "bf16", "bf16x3", "tf32x3w", "tf32x3f"])
@pytest.mark.parametrize("name,spec,B,L", CASES, ids=[c[0] for c in CASES])
def test_block_vs_oracle(name, spec, B, L, math):
    torch = _torch()
    from brosoundml_b200.decoder import Block
    o = BlockOracle(spec)
    p, x, style, dy = _inputs(o, B, L, 1)
    blk = Block(spec, 0, math=math)
    assert blk.n_params == o.n_params
    y = blk.forward(_dev(p), _dev(x), _dev(style))
    g = blk.backward(_dev(dy))
    torch.cuda.synchronize()
    r = o.run(p.astype(np.float64), x, style, dy=dy, dtype=np.float64)
    tol = TOL[math]
    assert rel_l2(y.cpu().numpy(), r["y"]) < tol
    gt = tol if math != "bf16" else BF16_GRAD_BAR
    assert rel_l2(g["dx"].cpu().numpy(), r["dx"]) < gt
    assert rel_l2(g["d_style"].cpu().numpy(), r["d_style"]) < gt
    if math == "bf16":
        assert rel_l2(g["grads"].cpu().numpy(), r["grads"]) < BF16_GRAD_BAR
    else:
        worst = per_tensor_rel(o.table, g["grads"].cpu().numpy(), r["grads"])
        bad = {k: v for k, v in worst.items() if v > tol}
        assert not bad, bad


@pytest.mark.parametrize("name,spec,B,L", [CASES[0], CASES[4]], ids=[CASES[0][0], CASES[4][0]])
def test_block_reference_mode(name, spec, B, L):
    """Caller-supplied (gamma, beta) (the LoRA path): y, dx and d_aff against the oracle."""
    torch = _torch()
    from brosoundml_b200.decoder import Block
    o = BlockOracle(spec)
    p, x, style, dy = _inputs(o, B, L, 2)
    aff = np.random.default_rng(3).uniform(-0.5, 0.5, B * o.aff_per_clip).astype(np.float32)
    blk = Block(spec, 0, math="tf32x3")
    y = blk.forward(_dev(p), _dev(x), aff_in=_dev(aff))
    g = blk.backward(_dev(dy), want_aff=True)
    torch.cuda.synchronize()
    r = o.run(p.astype(np.float64), x, style, aff_in=aff, dy=dy, dtype=np.float64)
    assert rel_l2(y.cpu().numpy(), r["y"]) < 1e-4
    assert rel_l2(g["dx"].cpu().numpy(), r["dx"]) < 1e-4
    assert rel_l2(g["d_aff"].cpu().numpy(), r["d_aff"]) < 1e-4
    assert float(g["d_style"].abs().max()) == 0.0


def test_block_handles_reject_the_other_api():
    torch = _torch()
    from brosoundml_b200 import _lib, config
    from brosoundml_b200.decoder import Block, Decoder, _ptr
    L = _lib.lib()
    z = torch.zeros(1 << 16, device="cuda")
    blk = Block(CASES[2][1], 0)
    assert L.bsml_decoder_forward(blk._h, 1, 2, _ptr(z), _ptr(z), _ptr(z), _ptr(z), _ptr(z), None, 0, None,
                                  _ptr(z), None, None) != 0
    assert "single block" in L.bsml_last_error().decode()
    dec = Decoder(config.miniature(), 0)
    assert L.bsml_block_forward(dec._h, 1, 8, _ptr(z), _ptr(z), _ptr(z), None, _ptr(z), None, None) != 0
    assert "whole decoder" in L.bsml_last_error().decode()
    assert L.bsml_block_backward(blk._h, _ptr(z), None, None, None, None, None) != 0
    assert "no matching forward" in L.bsml_last_error().decode()


def test_config1_resblock1_full_size_vs_torch_fp32():
    """BASELINE config 1 at full size: x [8, 128, 24000], style [8, 128], k = 7,
    dilations [1, 3, 5], weights N(0, 0.02), alpha = 1, upstream grad N(0, 1); the
    TF32x3 block against torch fp32 autograd (cuDNN with TF32 disabled) on the GPU."""
    torch = _torch()
    from brosoundml_b200.decoder import Block
    from oracle.torch_decoder import TorchDecoder
    spec = dict(kind=2, style_dim=128, cin=128, cout=128, kernel=7, dil=[1, 3, 5])
    B, L = 8, 24000
    o = BlockOracle(spec)
    rng = np.random.default_rng(11)
    p = np.zeros(o.n_params, np.float32)
    for e in o.table:
        s = slice(e["offset"], e["offset"] + e["numel"])
        p[s] = 1.0 if ".alpha" in "." + e["name"] else rng.normal(0, 0.02, e["numel"])
    g = torch.Generator(device="cuda").manual_seed(12)
    x = torch.randn(B, 128, L, device="cuda", generator=g)
    style = torch.randn(B, 128, device="cuda", generator=g)
    dy = torch.randn(B, 128, L, device="cuda", generator=g)
    blk = Block(spec, 0, math="tf32x3")
    y = blk.forward(_dev(p), x, style)
    out = blk.backward(dy)
    torch.cuda.synchronize()
    prev = torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        td = TorchDecoder({}, [dict(e, name="blk." + e["name"]) for e in o.table], p, dtype=torch.float32,
                          device="cuda")
        td.aff_list = []
        xt = x.clone().requires_grad_(True)
        st = style.clone().requires_grad_(True)
        yt = td.rb1(xt, "blk", st, 7, [1, 3, 5], None)
        yt.backward(dy)
        torch.cuda.synchronize()
    finally:
        torch.backends.cudnn.allow_tf32, torch.backends.cuda.matmul.allow_tf32 = prev
    tol = 1e-4
    assert rel_l2(y.cpu().numpy(), yt.detach().cpu().numpy()) < tol
    assert rel_l2(out["dx"].cpu().numpy(), xt.grad.cpu().numpy()) < tol
    assert rel_l2(out["d_style"].cpu().numpy(), st.grad.cpu().numpy()) < tol
    g, gt = out["grads"].cpu().numpy(), td.grads_flat(o.n_params)
    # convs1.i feeds only adain2.i's instance norm, which removes any per-channel
    # constant: the true bias gradient is exactly zero and both sides hold rounding
    # noise, checked against the global gradient norm instead
    zero = [e for e in o.table if e["name"].startswith("convs1.") and e["name"].endswith(".bias")]
    tot = float(np.linalg.norm(gt))
    for e in zero:
        sl = slice(e["offset"], e["offset"] + e["numel"])
        assert float(np.linalg.norm(g[sl])) < 1e-6 * tot and float(np.linalg.norm(gt[sl])) < 1e-6 * tot, e["name"]
    worst = per_tensor_rel([e for e in o.table if e not in zero], g, gt)
    bad = {k: v for k, v in worst.items() if v > tol}
    assert not bad, bad
