"""CPU tests of the C-ABI library: it loads, exports every symbol the header
declares, its parameter layout equals the oracle's, and it fails loudly
(status + message, never a CPU fallback) where there is no GPU."""

import ctypes
import os
import re

import pytest

from brosoundml_b200 import _lib, config
from oracle.oracle import Oracle
from tests.conftest import ROOT, cuda_available

HEADER = os.path.join(ROOT, "include", "bsml_decoder.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(bsml_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    syms = declared_symbols()
    assert len(syms) >= 25
    for s in syms:
        assert hasattr(L, s), s
    # and the Python binding types every one of them
    assert set(syms) == set(_lib.SIGNATURES), set(syms) ^ set(_lib.SIGNATURES)


@pytest.mark.parametrize("which", ["kokoro_82m", "miniature"])
def test_param_layout_matches_oracle(which):
    cfg = getattr(config, which)()
    n, table, affc, apc = _lib.layout(cfg)
    o = Oracle(cfg)
    assert n == o.n_params
    assert affc == o.aff_C and apc == o.aff_per_clip
    assert len(table) == len(o.table)
    for a, b in zip(table, o.table):
        assert a == b, (a, b)


def test_kokoro_param_count():
    n, table, affc, _ = _lib.layout(config.kokoro_82m())
    assert sum(e["numel"] for e in table) == 53251204
    assert len(affc) == 58   # 2 per backbone block, 6 per AdaINResBlock1 (decoder_lora.cpp:119-137)


def test_bad_config_is_rejected():
    cfg = config.with_overrides(config.kokoro_82m(), n_fft=21)
    with pytest.raises(_lib.BsmlError, match="brosoundml: bsml_decoder_create: n_fft"):
        _lib.layout(cfg)


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU error path")
def test_create_without_gpu_fails_loudly():
    L = _lib.lib()
    c = _lib.make_config(config.kokoro_82m())
    h = ctypes.c_void_p()
    rc = L.bsml_decoder_create(ctypes.byref(c), 0, ctypes.byref(h))
    assert rc != 0
    assert L.bsml_last_error().decode().startswith("brosoundml: ")


@pytest.mark.parametrize("fn", ["bsml_conv1d_backward_weight", "bsml_conv1d_backward_weight_noalloc",
                                "bsml_conv1d_forward"])
def test_conv_shorter_than_kernel_is_rejected(fn):
    """L + 2p - d(k-1) - 1 < 0 (L=2, k=7, p=0, stride 6) has no output. The shape
    check runs before any device work, so this holds with or without a GPU."""
    L = _lib.lib()
    z = ctypes.c_void_p(16)   # never dereferenced: the arguments are rejected first
    if fn == "bsml_conv1d_forward":
        rc = L.bsml_conv1d_forward(z, 1, 4, 2, z, None, 4, 7, 6, 0, 1, z, None)
    else:
        rc = getattr(L, fn)(z, z, 1, 4, 2, 4, 7, 6, 0, 1, z, None, None)
    assert rc != 0
    assert "bad argument" in L.bsml_last_error().decode()


def test_math_mode_names_match_the_header():
    """The Python mode names map to the header's BSML_MATH_* values."""
    from brosoundml_b200.decoder import MATH
    text = open(HEADER).read()
    enum = re.search(r"enum \{\s*(BSML_MATH_FP32_SIMT = 0[^}]*)\}", text).group(1)
    vals = {k.strip(): int(v) for k, v in (e.split("=") for e in enum.split(","))}
    names = {"fp32": "BSML_MATH_FP32_SIMT", "tf32x3": "BSML_MATH_TF32X3", "bf16": "BSML_MATH_BF16",
             "bf16x3": "BSML_MATH_BF16X3", "tf32x3w": "BSML_MATH_TF32X3W", "tf32x3f": "BSML_MATH_TF32X3F"}
    assert {m: vals[names[m]] for m in names} == MATH
