"""The C++ layer on the GPU: DecoderLora::make / forward / backward / adam_step /
save / load through include/bsml_decoder.hpp, with the reference's properties
(neutral identity at gate zero, include/brosoundml/decoder_lora.h:23-26; grads
accumulate; checkpoint round trip; move-only ownership)."""

import pytest

from brosoundml_b200 import config
from tests.conftest import cuda_available
from tests.test_cpp_shim_cpu import build_shim, write_cfg

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not cuda_available(), reason="needs a CUDA device")]


def test_cpp_layer_decoder_lora_on_gpu(tmp_path):
    import subprocess
    exe = build_shim(tmp_path, gpu=True)
    r = subprocess.run([exe, "gpu", write_cfg(tmp_path, config.miniature()), str(tmp_path)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and "OK" in r.stdout, r.stdout + r.stderr
