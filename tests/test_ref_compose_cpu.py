"""The oracle's composition checked against the reference's own code.

oracle/_ref/libref_compose.so holds the reference's src/kokoro_decoder_backward.cpp
and src/decoder_lora.cpp compiled unchanged from the reference checkout (recipe:
oracle/Makefile, target ref-compose) against CPU stand-ins for the absent op
library brotensor (oracle/ref_cpu/). Its only repository-written parts are those
op stand-ins and a driver that fills the reference's weight structs from the flat
parameter vector. So these tests pin the oracle's composition — the order and
wiring of every op, the concatenations and slices, the reflect pad, the noise
branch, the mean over resblocks, the spectral head's host adjoint, the adapter and
gate chain of DecoderLora — to the reference's source, and the ELRA1 checkpoint
bytes to the reference's own writer and reader.

Bars: the reference composition runs in fp32; each output must be as close to the
float64 oracle as the fp32 oracle is (within 4x its error, or under 1e-5)."""

import ctypes
import os

import numpy as np
import pytest

from brosoundml_b200 import config, synth
from oracle import lora_oracle as lo
from oracle.oracle import Oracle
from tests.conftest import ROOT
from tests.helpers import random_params, rel_l2

LIB = os.path.join(ROOT, "oracle", "_ref", "libref_compose.so")
pytestmark = pytest.mark.skipif(not os.path.exists(LIB), reason="built by build() where the reference checkout is present")

P = ctypes.c_void_p
FACTOR, FLOOR = 4.0, 1e-5


def _lib():
    L = ctypes.CDLL(LIB)
    I, F, I64, S = ctypes.c_int, ctypes.c_float, ctypes.c_int64, ctypes.c_char_p
    L.refc_last_error.restype = S
    L.refc_decoder_run.argtypes = [P, I, S, P, P, P, I, I, P, P, P, P, I, P, P, P, P]
    L.refc_lora_run.argtypes = [P, I, S, P, P, P, I, P, P, P, P, P, I, I, F, P, I64, I64, P, P, P, P, P, P, S]
    L.refc_lora_load.argtypes = [P, I, S, P, P, P, I, S, I64, I64, P, P, P, P]
    for f in (L.refc_decoder_run, L.refc_lora_run, L.refc_lora_load):
        f.restype = I
    return L


def _p(a):
    return a.ctypes.data_as(P) if a is not None else None


def _table(o):
    names = b"".join(e["name"].encode() + b"\0" for e in o.table)
    offs = np.array([e["offset"] for e in o.table], np.int64)
    nums = np.array([e["numel"] for e in o.table], np.int64)
    return names, offs, nums


def _cfg(cfg):
    from brosoundml_b200 import _lib as bl
    return bl.make_config(cfg)


def _check(got, r32, r64, what):
    e, e32 = rel_l2(got, r64), rel_l2(r32, r64)
    assert e <= max(FLOOR, FACTOR * e32), (what, e, e32)
    return e


CASES = [("miniature", 2, 4), ("kokoro_82m", 1, 3)]


@pytest.mark.parametrize("which,B,T", CASES)
def test_decoder_composition_matches_the_reference(which, B, T):
    """Reference mode (caller-supplied (gamma, beta) per AdaIN, as DecoderLora drives
    the assemblies): audio and every AdaIN's (dgamma, dbeta)."""
    cfg = getattr(config, which)()
    o = Oracle(cfg)
    if which == "miniature":
        params = random_params(o.table, o.n_params, 4).astype(np.float32)
        frames = 33
    else:
        params = synth.init_params(o.table, o.n_params, 0)
        frames = config.har_frames(cfg, T)
    x = synth.make_inputs(cfg, B, T, 3)
    rng = np.random.default_rng(11)
    har = rng.uniform(-0.4, 0.4, (B, cfg["har_ch"], frames)).astype(np.float32)
    aff = rng.uniform(-0.4, 0.4, B * o.aff_per_clip).astype(np.float32)
    S = cfg["hop"] * (frames - 1)
    da = rng.normal(0, 1e-3, (B, S)).astype(np.float32)
    L = _lib()
    names, offs, nums = _table(o)
    c = _cfg(cfg)
    audio = np.zeros((B, S), np.float32)
    daff = np.zeros(B * o.aff_per_clip, np.float32)
    rc = L.refc_decoder_run(ctypes.byref(c), len(o.table), names, _p(offs), _p(nums), _p(params), B, T,
                            _p(x["asr"]), _p(x["F0"]), _p(x["N"]), _p(har), frames, _p(aff), _p(da), _p(audio),
                            _p(daff))
    assert rc == 0, L.refc_last_error()
    kw = dict(har=har, aff_in=aff, daudio=da, want_aff=True)
    r64 = o.run(params, x["asr"], x["F0"], x["N"], x["style"], dtype=np.float64, **kw)
    r32 = o.run(params, x["asr"], x["F0"], x["N"], x["style"], **kw)
    ea = _check(audio, r32["audio"], r64["audio"], "audio")
    ed = _check(daff, r32["d_aff"], r64["d_aff"], "d_aff")
    print(f"{which}: reference composition vs float64 oracle: audio {ea:.2e}, d_aff {ed:.2e}")


def _lora_case(seed=5):
    cfg = config.miniature()
    o = Oracle(cfg)
    params = random_params(o.table, o.n_params, seed).astype(np.float32)
    T, frames, rank, scale = 4, 33, 4, 1.5
    x = synth.make_inputs(cfg, 1, T, seed)
    rng = np.random.default_rng(seed)
    har = rng.uniform(-0.4, 0.4, (1, cfg["har_ch"], frames)).astype(np.float32)
    ref_s = rng.normal(0, 0.5, (1, 2 * cfg["style_dim"])).astype(np.float32)
    lay = lo.LoraLayout(o.aff_C, rank, cfg["style_dim"])
    lp = rng.uniform(-0.2, 0.2, lay.n_params).astype(np.float32)
    cond = np.array([0.5, -0.3, 0.7], np.float32)
    return cfg, o, params, x, har, ref_s, lay, lp, cond, T, frames, rank, scale


def _lora_offsets(lay):
    return np.array(lay.off_A, np.int64), np.array(lay.off_B, np.int64)


def test_lora_composition_matches_the_reference(tmp_path):
    """DecoderLora::forward / backward of the reference (adapters and gate set to the
    same values) against the float64 LoRA oracle: audio and every adapter / gate gradient."""
    cfg, o, params, x, har, ref_s, lay, lp, cond, T, frames, rank, scale = _lora_case()
    S = cfg["hop"] * (frames - 1)
    da = np.random.default_rng(2).normal(0, 1e-3, (1, S)).astype(np.float32)
    L = _lib()
    names, offs, nums = _table(o)
    c = _cfg(cfg)
    oA, oB = _lora_offsets(lay)
    audio = np.zeros((1, S), np.float32)
    grad = np.zeros(lay.n_params, np.float32)
    rc = L.refc_lora_run(ctypes.byref(c), len(o.table), names, _p(offs), _p(nums), _p(params), T, _p(x["asr"]),
                         _p(x["F0"]), _p(x["N"]), _p(ref_s), _p(har), frames, rank, scale, _p(lp),
                         lay.off_W1, lay.off_W2, _p(oA), _p(oB), _p(cond), _p(da), _p(audio), _p(grad), None)
    assert rc == 0, L.refc_last_error()
    style = ref_s[:, :cfg["style_dim"]]
    r64 = lo.run(o, lay, params, lp, x["asr"], x["F0"], x["N"], style, cond[None], scale, har=har, daudio=da)
    assert rel_l2(audio, r64["audio"]) < 1e-5
    assert rel_l2(grad, r64["grads"]) < 1e-4
    for a in (0, len(lay.aff_C) - 1):   # first backbone and last generator adapter
        sA = slice(lay.off_A[a], lay.off_A[a] + rank * cfg["style_dim"])
        assert rel_l2(grad[sA], r64["grads"][sA]) < 1e-4


def test_elra1_bytes_match_the_reference_writer(tmp_path):
    """The reference's DecoderLora::save writes exactly what oracle.lora_oracle.read_elra1
    reads, and the reference's DecoderLora::load restores a file whose bytes this
    repository's format description (ELRA1) produces."""
    cfg, o, params, x, har, ref_s, lay, lp, cond, T, frames, rank, scale = _lora_case(6)
    S = cfg["hop"] * (frames - 1)
    L = _lib()
    names, offs, nums = _table(o)
    c = _cfg(cfg)
    oA, oB = _lora_offsets(lay)
    path = str(tmp_path / "ref.elra")
    audio = np.zeros((1, S), np.float32)
    rc = L.refc_lora_run(ctypes.byref(c), len(o.table), names, _p(offs), _p(nums), _p(params), T, _p(x["asr"]),
                         _p(x["F0"]), _p(x["N"]), _p(ref_s), _p(har), frames, rank, scale, _p(lp),
                         lay.off_W1, lay.off_W2, _p(oA), _p(oB), _p(cond), None, _p(audio), None, path.encode())
    assert rc == 0, L.refc_last_error()
    r, sd, sc, hidden, W1, W2, ads = lo.read_elra1(path)
    assert (r, sd, hidden) == (rank, cfg["style_dim"], 16) and abs(sc - scale) < 1e-7
    assert np.array_equal(W1, lay.W1(lp)) and np.array_equal(W2, lay.W2(lp))
    assert [C for C, _, _ in ads] == list(lay.aff_C)
    for a, (C, A, B) in enumerate(ads):
        assert np.array_equal(A, lay.A(lp, a)) and np.array_equal(B, lay.B(lp, a))
    # the reference reads it back into a fresh object
    back = np.zeros(lay.n_params, np.float32)
    sc2 = ctypes.c_float(0)
    rc = L.refc_lora_load(ctypes.byref(c), len(o.table), names, _p(offs), _p(nums), _p(params), rank, path.encode(),
                          lay.off_W1, lay.off_W2, _p(oA), _p(oB), _p(back), ctypes.byref(sc2))
    assert rc == 0, L.refc_last_error()
    assert np.array_equal(back, lp) and abs(sc2.value - scale) < 1e-7
