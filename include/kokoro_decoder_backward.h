// kokoro_decoder_backward.h — the reference's decoder backward atoms
// (src/kokoro_decoder_backward.h:37-293 in the reference, namespace
// brosoundml::detail) with their exact argument lists, cache structs and output
// semantics (outputs overwritten and resized), run on this build's GPU engine.
//
// Each *_forward_train fills its caller-owned cache and the matching *_backward
// reads it, as in the reference. Beyond the reference's named intermediates,
// every cache carries `state`: the GPU engine that ran the forward, which holds
// the intermediates the backward needs in device memory. The named tensor fields
// this build does not need are left empty; `x`-like inputs and the integer
// bookkeeping are filled. A cache may be reused across calls (the engine is kept
// while the architecture matches).
//
// Layout: N = 1, channel-major NCL (1, C * L), element (c, l) at c * L + l; the
// "sequence" layout is (L, C). (gamma, beta) are (C, 1). The weights are read on
// every call (they may change between calls); conv / convT / shortcut weights
// are frozen (no weight gradients), as in the reference.
#pragma once

#include <brotensor/tensor.h>

#include <array>
#include <memory>
#include <vector>

#include "brosoundml/kokoro_modules.h"

namespace brosoundml {
namespace detail {

// ─── AdaIN affine: y = (1 + gamma) * InstanceNorm(x) + beta ──────────────────
// x_ncl (1, C*L), gamma / beta (C, 1) -> y_ncl (1, C*L); x_seq_cache receives the
// normalised input in (L, C) sequence layout.
void adain_affine_forward(const brotensor::Tensor& x_ncl, const brotensor::Tensor& gamma,
                          const brotensor::Tensor& beta, int C, int L, float eps, brotensor::Tensor& y_ncl,
                          brotensor::Tensor& x_seq_cache);

// dY_ncl -> dX_ncl, dGamma, dBeta (overwritten); statistics recomputed from x_ncl
void adain_affine_backward(const brotensor::Tensor& x_ncl, const brotensor::Tensor& x_seq_cache,
                           const brotensor::Tensor& gamma, const brotensor::Tensor& dY_ncl, int C, int L, float eps,
                           brotensor::Tensor& dX_ncl, brotensor::Tensor& dGamma, brotensor::Tensor& dBeta);

// ─── AdainResBlk1d ──────────────────────────────────────────────────────────
struct AdainResBlkCache {
    brotensor::Tensor x;          // block input (1, C_in*L_in)
    brotensor::Tensor x_seq1;     // (left empty: the engine keeps its statistics)
    brotensor::Tensor r_pre;
    brotensor::Tensor conv1_out;
    brotensor::Tensor x_seq2;
    brotensor::Tensor n2_pre;
    int L_in = 0;
    int L_out = 0;
    std::shared_ptr<void> state;  // the engine holding this forward's intermediates
};

void adain_resblk_1d_forward_train(const AdainResBlk1dWeights& w, const brotensor::Tensor& x, int L_in,
                                   const brotensor::Tensor& gamma1, const brotensor::Tensor& beta1,
                                   const brotensor::Tensor& gamma2, const brotensor::Tensor& beta2, float eps,
                                   int& L_out, brotensor::Tensor& y, AdainResBlkCache& cache);

void adain_resblk_1d_backward(const AdainResBlk1dWeights& w, const AdainResBlkCache& cache,
                              const brotensor::Tensor& gamma1, const brotensor::Tensor& gamma2,
                              const brotensor::Tensor& dY, float eps, brotensor::Tensor& dX,
                              brotensor::Tensor& dGamma1, brotensor::Tensor& dBeta1, brotensor::Tensor& dGamma2,
                              brotensor::Tensor& dBeta2);

// ─── AdaINResBlock1 (Snake) ─────────────────────────────────────────────────
struct AdainResBlock1Cache {
    std::array<brotensor::Tensor, 3> x_in;   // x_in[0] = the block input; the rest left empty
    std::array<brotensor::Tensor, 3> x_seq1;
    std::array<brotensor::Tensor, 3> s1_pre;
    std::array<brotensor::Tensor, 3> c1_out;
    std::array<brotensor::Tensor, 3> x_seq2;
    std::array<brotensor::Tensor, 3> s2_pre;
    int C = 0;
    int L = 0;
    std::shared_ptr<void> state;
};

void adain_resblock1_forward_train(const AdaINResBlock1Weights& w, const brotensor::Tensor& x_in, int C, int L,
                                   const std::array<brotensor::Tensor, 3>& g1,
                                   const std::array<brotensor::Tensor, 3>& b1,
                                   const std::array<brotensor::Tensor, 3>& g2,
                                   const std::array<brotensor::Tensor, 3>& b2, brotensor::Tensor& x_out,
                                   AdainResBlock1Cache& cache);

void adain_resblock1_backward(const AdaINResBlock1Weights& w, const AdainResBlock1Cache& cache,
                              const std::array<brotensor::Tensor, 3>& g1,
                              const std::array<brotensor::Tensor, 3>& g2, const brotensor::Tensor& dX_out,
                              brotensor::Tensor& dX_in, std::array<brotensor::Tensor, 3>& dG1,
                              std::array<brotensor::Tensor, 3>& dB1, std::array<brotensor::Tensor, 3>& dG2,
                              std::array<brotensor::Tensor, 3>& dB2);

// ─── Spectral head: leaky 0.01 -> conv_post -> exp / sin polar -> iSTFT ─────
// window: the periodic Hann window of length win (this build requires
// win == n_fft and checks the values).
struct SpectralHeadCache {
    brotensor::Tensor x_pre;   // input to the final leaky_relu (1, C*L)
    brotensor::Tensor post;    // conv_post output (1, (n_fft+2)*L)
    int C = 0;
    int L = 0;
};

void spectral_head_forward_train(const Conv1d& conv_post, const brotensor::Tensor& x, int C, int L,
                                 const brotensor::Tensor& window, int n_fft, int hop, int win,
                                 brotensor::Tensor& audio, SpectralHeadCache& cache);

void spectral_head_backward(const Conv1d& conv_post, const SpectralHeadCache& cache,
                            const brotensor::Tensor& window, int n_fft, int hop, int win,
                            const brotensor::Tensor& dAudio, brotensor::Tensor& dX);

// ─── DecoderBackbone assembly ───────────────────────────────────────────────
struct BlockAffines {
    brotensor::Tensor g1, b1;   // affine1 (channels_in)
    brotensor::Tensor g2, b2;   // affine2 (channels_out)
};

struct BackboneCache {
    AdainResBlkCache encode;                  // (left empty: the engine in `state` holds the blocks)
    std::vector<AdainResBlkCache> decode;
    std::vector<char> res_applied;            // per decode block: [x, asr_res, F0, N] concatenated
    std::vector<int> x_channels;              // x channels before that block's concatenation
    int T = 0;
    std::shared_ptr<void> state;
};

// affines[0] = encode, affines[1 + i] = decode[i]; eps = 1e-5 (Kokoro)
void decoder_backbone_forward_train(const DecoderBackbone& bb, const brotensor::Tensor& asr,
                                    const brotensor::Tensor& F0_pred, const brotensor::Tensor& N_pred, int T,
                                    const std::vector<BlockAffines>& affines, float eps, brotensor::Tensor& gen_in,
                                    BackboneCache& cache);

// dAffines resized to the block count and filled; no asr / F0 / N / style grads
void decoder_backbone_backward(const DecoderBackbone& bb, const BackboneCache& cache,
                               const std::vector<BlockAffines>& affines, const brotensor::Tensor& dGenIn, float eps,
                               std::vector<BlockAffines>& dAffines);

// ─── Generator assembly ─────────────────────────────────────────────────────
struct ResBlock1Affines {
    std::array<brotensor::Tensor, 3> g1, b1;   // adain1[0..2]
    std::array<brotensor::Tensor, 3> g2, b2;   // adain2[0..2]
};

struct GenStageCache {
    brotensor::Tensor x_in;
    AdainResBlock1Cache noise;
    std::vector<AdainResBlock1Cache> res;
    int C_in = 0, L_in = 0;
    int C_out = 0, L_out = 0;
};

struct GeneratorCache {
    std::vector<GenStageCache> stages;   // shapes filled; tensors left empty
    SpectralHeadCache head;
    brotensor::Tensor window;
    std::shared_ptr<void> state;
};

// noise_aff[i] feeds noise_res[i]; res_aff[i*K + j] feeds resblocks[i*K + j]
void generator_forward_train(const Generator& gen, const brotensor::Tensor& gen_in, int L_in,
                             const brotensor::Tensor& har, int frames,
                             const std::vector<ResBlock1Affines>& noise_aff,
                             const std::vector<ResBlock1Affines>& res_aff, brotensor::Tensor& audio,
                             GeneratorCache& cache);

void generator_backward(const Generator& gen, const GeneratorCache& cache,
                        const std::vector<ResBlock1Affines>& noise_aff, const std::vector<ResBlock1Affines>& res_aff,
                        const brotensor::Tensor& dAudio, brotensor::Tensor& dGenIn,
                        std::vector<ResBlock1Affines>& dNoise_aff, std::vector<ResBlock1Affines>& dRes_aff);

}  // namespace detail
}  // namespace brosoundml
