// brotensor/ops/concat.h — the one copy op the reference's callers use directly
// (bt::copy_d2d, e.g. tests/test_kokoro_decoder_backward.cpp:502 and
// src/decoder_lora.cpp:187-199): n floats from src[src_off ...] to
// dst[dst_off ...], on the device; bounds are checked.
#pragma once

#include <brotensor/tensor.h>

namespace brotensor {

void copy_d2d(const Tensor& src, int src_off, Tensor& dst, int dst_off, int n);

}  // namespace brotensor
