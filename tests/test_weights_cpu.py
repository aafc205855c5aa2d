"""safetensors IO on the CPU (library reader, no device): parameters by layout
table with weight-norm fusion (scripts/convert-kokoro.py:71-110), dtype
conversion, the reference's missing-key / size errors
(src/kokoro_modules.cpp:99-125), and KokoroDecodePrep files
(include/brosoundml/kokoro.h:132-147)."""

import numpy as np
import pytest

from brosoundml_b200 import _lib, config, weights


class _Table:
    def __init__(self, cfg):
        self.n_params, self.table, _, _ = _lib.layout(cfg)


def _fuse(g, v):
    n = np.sqrt((v.astype(np.float64) ** 2).reshape(v.shape[0], -1).sum(1))
    return (g.reshape(-1, *([1] * (v.ndim - 1))) * v / np.maximum(n, 1e-12).reshape(-1, *([1] * (v.ndim - 1))))


def test_load_params_plain_and_weight_norm(tmp_path):
    m = _Table(config.miniature())
    rng = np.random.default_rng(0)
    expect = np.zeros(m.n_params, np.float32)
    tensors = {}
    for i, e in enumerate(m.table):
        w = rng.normal(0, 0.1, e["shape"]).astype(np.float32)
        key = "decoder.module." + e["name"]
        if e["name"].endswith(".weight") and len(e["shape"]) == 3 and i % 2 == 0:
            g = rng.uniform(0.5, 1.5, (e["shape"][0], 1, 1)).astype(np.float32)
            tensors[key + "_g"], tensors[key + "_v"] = g, w
            w = _fuse(g, w).astype(np.float32)
        elif i % 5 == 1:
            tensors[key] = w.astype(np.float16)        # converted to fp32 on read
            w = w.astype(np.float16).astype(np.float32)
        else:
            tensors[key] = w
        expect[e["offset"]:e["offset"] + e["numel"]] = w.reshape(-1)
    tensors["decoder.module.unused"] = np.ones(3, np.float32)   # extra keys are ignored
    path = str(tmp_path / "model.safetensors")
    weights.save_safetensors(path, tensors, {"format": "pt"})
    got = weights.load_params(m, path)
    assert np.allclose(got, expect, rtol=2e-6, atol=1e-7)
    with weights.SafeTensorsFile(path) as f:
        names = f.tensors()
        assert names["decoder.module.unused"] == ("F32", (3,))
        assert f.metadata("format") == "pt"


def test_load_params_errors(tmp_path):
    m = _Table(config.miniature())
    e0 = m.table[0]
    path = str(tmp_path / "bad.safetensors")
    weights.save_safetensors(path, {"decoder.module." + e0["name"]: np.zeros(e0["numel"] + 1, np.float32)})
    with pytest.raises(_lib.BsmlError, match="elements; expected"):
        weights.load_params(m, path)
    weights.save_safetensors(path, {"decoder.module." + e0["name"]: np.zeros(e0["numel"], np.float32)})
    with pytest.raises(_lib.BsmlError, match="missing safetensors key 'decoder.module." + m.table[1]["name"]):
        weights.load_params(m, path)
    (tmp_path / "trunc.safetensors").write_bytes(b"\x10\x00\x00\x00\x00\x00\x00\x00{")
    with pytest.raises(_lib.BsmlError, match="header"):
        weights.SafeTensorsFile(str(tmp_path / "trunc.safetensors"))


def test_decode_prep_roundtrip_and_stack(tmp_path):
    rng = np.random.default_rng(1)
    T, S, H, har_ch, frames = 6, 4, 5, 3, 20
    paths = []
    clips = []
    for c in range(3):
        d = dict(ref_s=rng.normal(size=(1, 2 * S)), asr=rng.normal(size=(1, H, T)), F0_pred=rng.uniform(80, 300, 2 * T),
                 N_pred=rng.normal(size=(1, 2 * T)), har=rng.normal(size=(1, har_ch, frames)))
        p = str(tmp_path / f"clip{c}.safetensors")
        weights.save_decode_prep(p, **d)
        paths.append(p)
        clips.append(d)
    preps = [weights.load_decode_prep(p) for p in paths]
    assert preps[0]["total"] == T and preps[0]["frames"] == frames
    assert np.array_equal(preps[1]["asr"], clips[1]["asr"][0].astype(np.float32))
    batch = weights.stack_decode_preps(preps)
    assert batch["asr"].shape == (3, H, T) and batch["F0"].shape == (3, 2 * T) and batch["har"].shape == (3, har_ch, frames)
    assert np.array_equal(batch["ref_s"][2], clips[2]["ref_s"][0].astype(np.float32))
    # clips of different length do not stack
    weights.save_decode_prep(str(tmp_path / "long.safetensors"), np.zeros(2 * S), np.zeros((H, T + 1)),
                             np.zeros(2 * T + 2), np.zeros(2 * T + 2))
    with pytest.raises(ValueError, match="differ in length"):
        weights.stack_decode_preps(preps + [weights.load_decode_prep(str(tmp_path / "long.safetensors"))])
    weights.save_safetensors(str(tmp_path / "other.safetensors"), {"x": np.zeros(2, np.float32)}, {"format": "x"})
    with pytest.raises(ValueError, match="not a KokoroDecodePrep"):
        weights.load_decode_prep(str(tmp_path / "other.safetensors"))


@pytest.mark.gpu
def test_loaded_checkpoint_drives_the_decoder(tmp_path):
    """A checkpoint written with the upstream keys (weight-norm pairs on the convs)
    loads into the parameter vector the engine runs on: same audio as the vector it
    was written from."""
    from tests.conftest import cuda_available
    if not cuda_available():
        pytest.skip("needs a CUDA device")
    import torch

    from brosoundml_b200 import synth
    from brosoundml_b200.decoder import Decoder
    cfg = config.miniature()
    dec = Decoder(cfg, 0, math="tf32x3")
    p = synth.init_params(dec.table, dec.n_params, 0)
    tensors = {}
    rng = np.random.default_rng(2)
    for e in dec.table:
        w = p[e["offset"]:e["offset"] + e["numel"]].reshape(e["shape"]).astype(np.float64)
        key = "decoder.module." + e["name"]
        if e["name"].endswith(".weight") and len(e["shape"]) == 3:
            g = np.sqrt((w ** 2).reshape(w.shape[0], -1).sum(1)).reshape(-1, 1, 1)
            v = w * rng.uniform(0.5, 2.0, (w.shape[0], 1, 1))    # any positive per-row rescaling of w
            tensors[key + "_g"], tensors[key + "_v"] = g.astype(np.float32), v.astype(np.float32)
        else:
            tensors[key] = w.astype(np.float32)
    path = str(tmp_path / "model.safetensors")
    weights.save_safetensors(path, tensors)
    q = weights.load_params(dec, path)
    assert np.allclose(q, p, rtol=1e-5, atol=1e-7)
    B, T, frames = 2, 4, 33
    x = synth.make_inputs(cfg, B, T, 1)
    har = np.random.default_rng(3).uniform(-0.4, 0.4, (B, cfg["har_ch"], frames)).astype(np.float32)
    dv = {k: torch.tensor(v, device="cuda") for k, v in dict(x, har=har).items()}
    a = dec.forward(torch.tensor(p, device="cuda"), dv["asr"], dv["F0"], dv["N"], dv["style"], har=dv["har"]).clone()
    b = dec.forward(torch.tensor(q, device="cuda"), dv["asr"], dv["F0"], dv["N"], dv["style"], har=dv["har"]).clone()
    torch.cuda.synchronize()
    assert float((a - b).norm() / a.norm()) < 1e-5
