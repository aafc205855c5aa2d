"""Decoder architecture descriptions.

A config is a plain dict whose keys match ``bsml_decoder_config`` in
include/bsml_decoder.h. ``kokoro_82m()`` is the Kokoro-82M iSTFTNet decoder
as the reference loads it (DecoderBackbone::load_from,
src/kokoro_modules.cpp:1021-1063; Generator::load_from, :1237-1347;
HarmonicSource::load_from, :1556-1572). ``miniature()`` is the tiny
backbone+generator the reference's own end-to-end LoRA test builds
(tests/test_kokoro_decoder_backward.cpp:467-497).
"""

from __future__ import annotations

import copy


def kokoro_82m() -> dict:
    return dict(
        asr_dim=512, style_dim=128, asr_res_dim=64, enc_dim=1024,
        n_decode=4, dec_out=[1024, 1024, 1024, 512], upsample_block=3,
        n_ups=2, init_ch=512, ups_rate=[10, 6], ups_kernel=[20, 12],
        # noise_convs: k = 2*prod(later rates), s = prod(later rates), p = (s+1)//2; last stage 1x1
        noise_kernel=[12, 1], noise_stride=[6, 1], noise_pad=[3, 0],
        nr_kernel=[7, 11], nr_dil=[[1, 3, 5], [1, 3, 5]],
        n_kernels=3, rb_kernel=[3, 7, 11], rb_dil=[[1, 3, 5], [1, 3, 5], [1, 3, 5]],
        har_ch=22, n_fft=20, hop=5, post_kernel=7, harmonic_num=8,
        sample_rate=24000, upsample_scale=300,
    )


def miniature() -> dict:
    """Reference test miniature: asr 6 ch, encode 8->10, decode 16->10, 16->8 (2x up),
    generator 8->4->2 (k4 s2 p1), 2 kernels k3 dil (1,2,3), n_fft 8 / hop 4, har 1 ch."""
    return dict(
        asr_dim=6, style_dim=128, asr_res_dim=4, enc_dim=10,
        n_decode=2, dec_out=[10, 8], upsample_block=1,
        n_ups=2, init_ch=8, ups_rate=[2, 2], ups_kernel=[4, 4],
        noise_kernel=[4, 3], noise_stride=[2, 1], noise_pad=[1, 1],
        nr_kernel=[3, 3], nr_dil=[[1, 2, 3], [1, 2, 3]],
        n_kernels=2, rb_kernel=[3, 3], rb_dil=[[1, 2, 3], [1, 2, 3]],
        har_ch=1, n_fft=8, hop=4, post_kernel=7, harmonic_num=8,
        sample_rate=24000, upsample_scale=16,
    )


def with_overrides(cfg: dict, **kw) -> dict:
    c = copy.deepcopy(cfg)
    c.update(kw)
    return c


def audio_len(cfg: dict, T: int) -> int:
    """Samples of audio produced from T asr frames when har comes from the harmonic source."""
    frames = (2 * T * cfg["upsample_scale"]) // cfg["hop"] + 1
    return cfg["hop"] * (frames - 1)


def har_frames(cfg: dict, T: int) -> int:
    return (2 * T * cfg["upsample_scale"]) // cfg["hop"] + 1
