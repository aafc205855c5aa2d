// brosoundml/kokoro_modules.h — the Kokoro decoder's weight structs with the
// reference's members (include/brosoundml/kokoro_modules.h:109-340 in the
// reference) and the inference forwards the decoder training path is checked
// against: DecoderBackbone::forward, HarmonicSource::forward and
// Generator::forward. The forwards run on the GPU engine of this build
// (include/bsml_decoder.h); the structs hold the weights in brotensor::Tensor,
// so code that fills them the reference's way (a checkpoint loader, a test's
// random initialisation) works unchanged. Loading from safetensors goes through
// bsml_params_from_safetensors instead of load_from().
#pragma once

#include <brotensor/tensor.h>

#include <array>
#include <cstdint>
#include <functional>
#include <vector>

#include "brosoundml/modules.h"

namespace brosoundml {

// checked between generator stages; true aborts the forward (audio left empty)
using CancelCheck = std::function<bool()>;

// AdaIN1d: y = (1 + gamma(s)) * InstanceNorm1d(x) + beta(s); fc: style -> (gamma ; beta)
struct AdaIN1dWeights {
    int channels = 0;
    int style_dim = 0;
    float eps = 1e-5f;
    Linear fc;   // (2 * channels, style_dim)
};

// The StyleTTS2 AdaIN residual block (iSTFTNet decoder): conv1 / conv2 k3 p1,
// optional x2 upsampling (depthwise ConvTranspose1d pool, k3 s2 p1 op1) and a
// learned 1x1 shortcut when channels_in != channels_out.
struct AdainResBlk1dWeights {
    int channels_in = 0;
    int channels_out = 0;
    bool upsample = false;
    bool learned_sc = false;
    AdaIN1dWeights norm1;
    AdaIN1dWeights norm2;
    Conv1d conv1;
    Conv1d conv2;
    Conv1d conv1x1;
    brotensor::Tensor pool_W;   // (channels_in, 3)
    brotensor::Tensor pool_b;   // (channels_in, 1)
};

// The generator's residual block: three (Snake, dilated conv, Snake, conv) pairs
struct AdaINResBlock1Weights {
    int channels = 0;
    int kernel_size = 0;
    std::vector<int> dilations;   // length 3
    std::array<Conv1d, 3> convs1;
    std::array<Conv1d, 3> convs2;
    std::array<AdaIN1dWeights, 3> adain1;
    std::array<AdaIN1dWeights, 3> adain2;
    std::array<brotensor::Tensor, 3> alpha1;   // (channels, 1)
    std::array<brotensor::Tensor, 3> alpha2;
};

// Everything of the decoder up to the generator (F0 / N stride-2 convs, the asr
// 1x1 projection, the encode block and the decode blocks).
struct DecoderBackbone {
    Conv1d F0_conv;
    Conv1d N_conv;
    Conv1d asr_res;
    AdainResBlk1dWeights encode;
    std::vector<AdainResBlk1dWeights> decode;

    // asr (1, C_asr * T), F0_pred / N_pred (1, 2T), ref_s (1, 2 * style_dim): the
    // style is its first style_dim values. gen_in (1, C_gen * L_gen).
    void forward(const brotensor::Tensor& asr, const brotensor::Tensor& F0_pred, const brotensor::Tensor& N_pred,
                 const brotensor::Tensor& ref_s, int T, brotensor::Tensor& gen_in) const;
};

// The deterministic sine source (upsampled F0 -> harmonics -> l_linear + tanh ->
// STFT magnitude and phase). This build reproduces the reference's fp32
// per-sample phase accumulation (kokoro_modules.cpp:1601-1616) bit for bit.
struct HarmonicSource {
    int sample_rate = 24000;
    int harmonic_num = 8;
    int upsample_scale = 0;
    int n_fft = 0;
    int hop_size = 0;
    int win_size = 0;
    float sine_amp = 0.1f;
    Linear l_linear;   // (1, harmonic_num + 1)

    // F0_pred (1, frame_count) -> har (1, (n_fft + 2) * stft_frames)
    void forward(const brotensor::Tensor& F0_pred, int frame_count, int& signal_len, int& stft_frames,
                 brotensor::Tensor& har) const;
};

// The iSTFTNet generator: ConvTranspose1d upsamplers, the noise branch, the
// AdaINResBlock1 stacks, conv_post and the iSTFT.
struct Generator {
    int n_fft = 0;
    int hop_size = 0;
    int win_size = 0;
    int num_upsamples = 0;
    int num_kernels = 0;
    std::vector<brotensor::Tensor> ups_W;   // each (C_in, C_out * k)
    std::vector<brotensor::Tensor> ups_b;   // each (C_out, 1)
    std::vector<int> ups_C_in, ups_C_out, ups_k, ups_stride, ups_pad;
    std::vector<Conv1d> noise_convs;
    std::vector<AdaINResBlock1Weights> noise_res;   // num_upsamples
    std::vector<AdaINResBlock1Weights> resblocks;   // num_upsamples * num_kernels
    Conv1d conv_post;

    // gen_in (1, C * L_in), har (1, har_ch * frames), style (1, style_dim) ->
    // audio (1, hop_size * (frames - 1))
    void forward(const brotensor::Tensor& gen_in, int L_in, const brotensor::Tensor& har, int frames,
                 const brotensor::Tensor& style, brotensor::Tensor& audio, const CancelCheck& cancel = {}) const;
};

}  // namespace brosoundml
