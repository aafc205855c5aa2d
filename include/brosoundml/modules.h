// brosoundml/modules.h — the generic modules the decoder's weight structs are
// built from, with the reference's members (include/brosoundml/modules.h:27-81
// in the reference): Linear (y = W x + b) and Conv1d (NCL). Their forwards run on
// the GPU through this build's C ABI (include/bsml_decoder.h).
#pragma once

#include <brotensor/tensor.h>

namespace brosoundml {

// y = W x + b. W (out, in); b (out, 1), empty when the bias is disabled.
struct Linear {
    int in_features = 0;
    int out_features = 0;
    brotensor::Tensor W;
    brotensor::Tensor b;

    // x (in, 1) -> y (out, 1)
    void forward(const brotensor::Tensor& x, brotensor::Tensor& y) const;
    // X (B, in) -> Y (B, out)
    void forward_batched(const brotensor::Tensor& X, brotensor::Tensor& Y) const;
};

// Conv1d over NCL activations. W (out, (in/groups) * kernel_size); b (out, 1),
// empty when the bias is disabled. This build supports groups == 1.
struct Conv1d {
    int in_channels = 0;
    int out_channels = 0;
    int kernel_size = 0;
    int stride = 1;
    int padding = 0;
    int dilation = 1;
    int groups = 1;
    brotensor::Tensor W;
    brotensor::Tensor b;

    // X (N, in_channels * L) -> Y (N, out_channels * L_out)
    void forward(const brotensor::Tensor& X, int N, int L, brotensor::Tensor& Y) const;
    // L_out for an input of length L
    int out_len(int L) const { return (L + 2 * padding - dilation * (kernel_size - 1) - 1) / stride + 1; }
};

}  // namespace brosoundml
