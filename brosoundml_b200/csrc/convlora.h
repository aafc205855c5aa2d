// Conv-weight LoRA (the fine-tune of every conv weight; no counterpart in the reference): a rank-r
// adapter on every Conv1d / ConvTranspose1d weight of the decoder, base weights
// frozen. A weight stored as (d0, d1, k) is viewed as the matrix [d0][d1*k] and
// adapted as W + scale * B A, with A [rank][d1*k] and B [d0][rank]. Each forward
// folds the adapters into a private copy of the parameters; the backward turns
// the engine's weight gradients dW into dA = scale B^T dW and dB = scale dW A^T.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "engine.h"

namespace bsml {

struct ConvLoraW {
    int64_t w;      // weight offset in the decoder parameters
    int rows, cols; // the [d0][d1*k] matrix view
    int64_t offA, offB;
};

class ConvLora {
   public:
    ConvLora(Engine& eng, int rank, float scale, uint64_t seed);
    ~ConvLora();
    ConvLora(const ConvLora&) = delete;
    ConvLora& operator=(const ConvLora&) = delete;

    int64_t n_params() const { return n_params_; }
    int rank() const { return rank_; }
    float scale() const { return scale_; }
    int step() const { return step_; }
    const std::vector<ConvLoraW>& weights() const { return ws_; }
    float* params() { return P_; }
    float* grads() { return G_; }

    void forward(int B, int T, const float* base, const float* asr, const float* F0, const float* N,
                 const float* style, const float* har, int frames, float* audio, cudaStream_t st);
    // accumulates dA, dB (until zero_grad)
    void backward(const float* daudio, cudaStream_t st);
    void zero_grad(cudaStream_t st);
    void adam_step(float lr, float b1, float b2, float eps, cudaStream_t st);
    // full training state (ECLR1): parameters, Adam moments and step; synchronous
    void save(const std::string& path) const;
    void load(const std::string& path);

   private:
    Engine& eng_;
    int device_ = 0, rank_ = 0, step_ = 0;
    float scale_ = 1.f;
    int64_t n_params_ = 0, n_dec_ = 0;
    std::vector<ConvLoraW> ws_;
    ConvLoraW* d_ws_ = nullptr;
    float *P_ = nullptr, *G_ = nullptr, *M_ = nullptr, *V_ = nullptr;
    float* eff_ = nullptr;     // decoder parameters with the adapters folded in
    float* dgrad_ = nullptr;   // full decoder gradient of the last backward
    bool fwd_done_ = false;
};

}  // namespace bsml
