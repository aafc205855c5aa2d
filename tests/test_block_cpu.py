"""CPU tests of the block-level oracle (one AdainResBlk1d or one AdaINResBlock1 on its
own: the reference's block atoms, src/kokoro_decoder_backward.h:82-144, and BASELINE
config 1): the C++ oracle against an independent PyTorch autograd restatement in
float64 (outputs, every parameter gradient, dX, d_style, and the per-AdaIN
(dGamma, dBeta) of the reference mode), plus a directional finite-difference check
in the reference's manner (tests/test_kokoro_decoder_backward.cpp:219-330)."""

import numpy as np
import pytest
import torch

from oracle.oracle import BlockOracle
from oracle.torch_decoder import TorchDecoder
from tests.helpers import per_tensor_rel, random_params, rel_l2

SPECS = {
    "resblock1_k3": dict(kind=2, style_dim=8, cin=6, cout=6, kernel=3, dil=[1, 3, 5]),
    "resblock1_k7": dict(kind=2, style_dim=5, cin=4, cout=4, kernel=7, dil=[1, 3, 5]),
    "resblk1d_up_sc": dict(kind=1, style_dim=8, cin=6, cout=4, upsample=1),
    "resblk1d_plain": dict(kind=1, style_dim=8, cin=5, cout=5, upsample=0),
}


def _inputs(o, B, L, seed):
    rng = np.random.default_rng(seed)
    sp = o.spec_dict
    p = random_params(o.table, o.n_params, seed)
    x = rng.normal(0, 1, (B, sp["cin"], L))
    style = rng.normal(0, 1, (B, sp["style_dim"]))
    dy = rng.normal(0, 1, (B, sp["cout"], o.out_len(L)))
    return p, x, style, dy


def _torch_block(o, p, x, style, dy, aff_list=None):
    table = [dict(e, name="blk." + e["name"]) for e in o.table]
    td = TorchDecoder({}, table, p)
    td.aff_list = []
    sp = o.spec_dict
    xt = torch.tensor(x, requires_grad=True)
    st = torch.tensor(style, requires_grad=True)
    aff = None if aff_list is None else [torch.tensor(a, requires_grad=True) for a in aff_list]
    aff_keep = None if aff is None else list(aff)
    if sp["kind"] == 1:
        y = td.blk(xt, "blk", st, sp["cin"], sp["cout"], bool(sp["upsample"]), aff)
    else:
        y = td.rb1(xt, "blk", st, sp["kernel"], sp["dil"], aff)
    y.backward(torch.tensor(dy))
    daff = None if aff_keep is None else np.concatenate([a.grad.numpy().reshape(-1) for a in aff_keep])
    ds = np.zeros_like(style) if st.grad is None else st.grad.numpy()
    return y.detach().numpy(), td.grads_flat(o.n_params), xt.grad.numpy(), ds, daff


@pytest.mark.parametrize("name", sorted(SPECS))
def test_block_oracle_matches_torch_autograd(name):
    o = BlockOracle(SPECS[name])
    B, L = 2, 23
    p, x, style, dy = _inputs(o, B, L, 3)
    r = o.run(p, x, style, dy=dy, dtype=np.float64)
    y, g, dx, ds, _ = _torch_block(o, p, x, style, dy)
    assert r["y"].shape == y.shape
    assert rel_l2(r["y"], y) < 1e-12
    assert rel_l2(r["dx"], dx) < 1e-11
    assert rel_l2(r["d_style"], ds) < 1e-11
    worst = max(per_tensor_rel(o.table, r["grads"], g).values())
    assert worst < 1e-10, worst


@pytest.mark.parametrize("name", ["resblock1_k3", "resblk1d_up_sc"])
def test_block_reference_mode_daff(name):
    """Caller-supplied (gamma, beta) per AdaIN (the LoRA path): d_aff equals autograd's."""
    o = BlockOracle(SPECS[name])
    B, L = 2, 17
    p, x, style, dy = _inputs(o, B, L, 4)
    rng = np.random.default_rng(5)
    aff = rng.uniform(-0.5, 0.5, B * o.aff_per_clip)
    r = o.run(p, x, style, aff_in=aff, dy=dy, dtype=np.float64)
    # unpack [a][B][2C] into the per-AdaIN (B, 2C) list in adapter order
    lst, off = [], 0
    for C in o.aff_C:
        lst.append(aff[off:off + B * 2 * C].reshape(B, 2 * C))
        off += B * 2 * C
    y, _, dx, _, daff = _torch_block(o, p, x, style, dy, aff_list=lst)
    assert rel_l2(r["y"], y) < 1e-12
    assert rel_l2(r["dx"], dx) < 1e-11
    assert rel_l2(r["d_aff"], daff) < 1e-11
    assert np.all(r["d_style"] == 0)


def test_block_directional_fd():
    o = BlockOracle(SPECS["resblock1_k3"])
    B, L = 1, 19
    p, x, style, dy = _inputs(o, B, L, 6)
    r = o.run(p, x, style, dy=dy, dtype=np.float64)

    def loss(pp, xx, ss):
        return float((o.run(pp, xx, ss, dtype=np.float64)["y"] * dy).sum())

    rng = np.random.default_rng(7)
    h = 1e-6
    vp, vx, vs = rng.uniform(-1, 1, p.shape), rng.uniform(-1, 1, x.shape), rng.uniform(-1, 1, style.shape)
    for an, fd in ((float((r["grads"] * vp).sum()), (loss(p + h * vp, x, style) - loss(p - h * vp, x, style)) / (2 * h)),
                   (float((r["dx"] * vx).sum()), (loss(p, x + h * vx, style) - loss(p, x - h * vx, style)) / (2 * h)),
                   (float((r["d_style"] * vs).sum()),
                    (loss(p, x, style + h * vs) - loss(p, x, style - h * vs)) / (2 * h))):
        assert abs(an - fd) <= 1e-6 * max(1.0, abs(fd)), (an, fd)


@pytest.mark.parametrize("name", sorted(SPECS))
def test_block_layout_matches_library(name):
    """The library's block parameter table (no device needed) equals the oracle's."""
    from brosoundml_b200 import _lib
    n, table, aff_C, apc = _lib.block_layout(SPECS[name])
    o = BlockOracle(SPECS[name])
    assert (n, aff_C, apc) == (o.n_params, o.aff_C, o.aff_per_clip)
    assert [(e["name"], e["offset"], e["shape"]) for e in table] == [(e["name"], e["offset"], e["shape"])
                                                                      for e in o.table]


def test_block_spec_validation():
    from brosoundml_b200 import _lib
    with pytest.raises(_lib.BsmlError, match="cin == cout"):
        _lib.block_layout(dict(kind=2, style_dim=4, cin=4, cout=6, kernel=3, dil=[1, 1, 1]))
    with pytest.raises(_lib.BsmlError, match="unknown block kind"):
        _lib.block_layout(dict(kind=7, style_dim=4, cin=4, cout=4))
