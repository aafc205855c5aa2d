"""B200-native Kokoro decoder training path (forward + backward), sm_100a CUDA
behind a C ABI (include/bsml_decoder.h)."""

from . import config, synth  # noqa: F401

__all__ = ["config", "synth"]
