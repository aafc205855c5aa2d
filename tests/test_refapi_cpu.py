"""The reference-signature C++ layer (libbsml_ref.so; include/brotensor/*.h,
include/brosoundml/*.h, include/kokoro_decoder_backward.h) without a GPU: it
loads, exports every entry point of the reference's headers it stands in for
(src/kokoro_decoder_backward.h:37-293, include/brosoundml/decoder_lora.h:36-164),
and fails loudly ("brosoundml: ..." as std::runtime_error) where there is no
device, never computing on the CPU."""

import ctypes
import os
import shutil
import subprocess

import pytest

from brosoundml_b200 import _lib
from tests.conftest import ROOT, cuda_available

LIB = os.path.join(ROOT, "brosoundml_b200", "libbsml_ref.so")

EXPECTED = [
    "brosoundml::detail::adain_affine_forward(",
    "brosoundml::detail::adain_affine_backward(",
    "brosoundml::detail::adain_resblk_1d_forward_train(",
    "brosoundml::detail::adain_resblk_1d_backward(",
    "brosoundml::detail::adain_resblock1_forward_train(",
    "brosoundml::detail::adain_resblock1_backward(",
    "brosoundml::detail::spectral_head_forward_train(",
    "brosoundml::detail::spectral_head_backward(",
    "brosoundml::detail::decoder_backbone_forward_train(",
    "brosoundml::detail::decoder_backbone_backward(",
    "brosoundml::detail::generator_forward_train(",
    "brosoundml::detail::generator_backward(",
    "brosoundml::DecoderLora::make(",
    "brosoundml::DecoderLora::forward(",
    "brosoundml::DecoderLora::backward(",
    "brosoundml::DecoderLora::zero_grad(",
    "brosoundml::DecoderLora::adam_step(",
    "brosoundml::DecoderLora::save(",
    "brosoundml::DecoderLora::load(",
    "brosoundml::DecoderLora::adapters(",
    "brosoundml::ConditioningGate::make(",
    "brosoundml::ConditioningGate::forward(",
    "brosoundml::ConditioningGate::backward(",
    "brosoundml::ConditioningGate::zero_grad(",
    "brosoundml::DecoderBackbone::forward(",
    "brosoundml::Generator::forward(",
    "brosoundml::HarmonicSource::forward(",
    "brosoundml::Conv1d::forward(",
    "brosoundml::Linear::forward(",
    "brotensor::Tensor::from_host_on(",
    "brotensor::Tensor::zeros_on(",
    "brotensor::copy_d2d(",
    "brotensor::init(",
]


def test_reference_layer_loads_and_exports():
    assert os.path.exists(LIB), "libbsml_ref.so is built by __graft_entry__.build()"
    _lib.lib()
    ctypes.CDLL(LIB)
    if shutil.which("nm") is None:
        pytest.skip("needs nm")
    out = subprocess.run(["nm", "-DC", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    missing = [s for s in EXPECTED if s not in out]
    assert not missing, missing


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU error path")
@pytest.mark.parametrize("name", ["test_decoder_lora", "test_kokoro_decoder_backward"])
def test_reference_tests_fail_loudly_without_gpu(name, tmp_path):
    exe = os.path.join(ROOT, "oracle", "_ref", name)
    if not os.path.exists(exe):
        pytest.skip("the reference's tests are built only where the reference checkout is present")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120, cwd=str(tmp_path))
    assert r.returncode != 0
    assert "brosoundml: " in r.stderr, r.stderr
