// DecoderLora on the GPU: per-AdaIN LoRA adapters on the frozen style -> (gamma, beta)
// projections, the shared conditioning gate, Adam and the ELRA1 checkpoint of the
// reference (src/decoder_lora.cpp, include/brosoundml/decoder_lora.h), batched over
// clips. The decoder engine runs in reference mode: these adapters supply every
// AdaIN's (gamma, beta), the engine returns their gradients, the base weights stay
// frozen (no weight gradients are formed).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "engine.h"

namespace bsml {

// ConditioningGate on its own (decoder_lora.cpp:28-78), batched over B condition
// vectors v (B, in_dim): act = tanh(W1 v), g = W2 act; the backward accumulates
// dW1, dW2 (+=) from dG (B, gate_dim).
void gate_forward(const float* W1, const float* W2, const float* v, int B, int in_dim, int hidden, int gate_dim,
                  float* act, float* g, cudaStream_t st);
void gate_backward(const float* W2, const float* v, const float* act, const float* dG, int B, int in_dim,
                   int hidden, int gate_dim, float* dW1, float* dW2, cudaStream_t st);

// Per adapter (one per AdaIN, DecoderLora::adapters() order), device side.
struct LoraAd {
    int64_t fw, fb;        // base fc weight [2C][S] / bias [2C] in the decoder parameters
    int64_t aff_base;      // per-clip offset of this AdaIN's (gamma ; beta) block
    int64_t offA, offB;    // A [rank][S], B [2C][rank] in the LoRA parameter vector
    int C;
};

class Lora {
   public:
    static constexpr int kInDim = 3;     // condition width (ConditioningGate::in_dim)
    static constexpr int kHidden = 16;   // gate hidden width (DecoderLora::make)

    Lora(Engine& eng, int rank, float scale, uint64_t seed);
    ~Lora();
    Lora(const Lora&) = delete;
    Lora& operator=(const Lora&) = delete;

    // Flat parameter vector (grads and Adam moments share the layout):
    //   gate W1 [kHidden][kInDim], gate W2 [rank][kHidden], then per adapter A, B.
    int64_t n_params() const { return n_params_; }
    int n_adapters() const { return (int)ads_.size(); }
    int rank() const { return rank_; }
    int style_dim() const { return S_; }
    float scale() const { return scale_; }
    int step() const { return step_; }
    float* params() { return P_; }
    float* grads() { return G_; }
    float* moment1() { return M_; }
    float* moment2() { return V_; }
    int64_t off_W1() const { return 0; }
    int64_t off_W2() const { return (int64_t)kHidden * kInDim; }
    const std::vector<LoraAd>& adapters() const { return ads_; }

    // DecoderLora::forward, batched: style_b = ref_s[b*ref_stride .. + S), cond (B, kInDim).
    void forward(int B, int T, const float* params, const float* asr, const float* F0, const float* N,
                 const float* ref_s, int ref_stride, const float* har, int frames, const float* cond, float* audio,
                 cudaStream_t st);
    // DecoderLora::backward: accumulates the adapter and gate gradients.
    void backward(const float* daudio, cudaStream_t st);
    void zero_grad(cudaStream_t st);
    void adam_step(float lr, float b1, float b2, float eps, cudaStream_t st);
    // ELRA1 checkpoint (DecoderLora::save / load, src/decoder_lora.cpp:324-396); synchronous.
    // full_state: Adam's moments and step follow the ELRA1 body (a resume point;
    // the reference format drops them, and its reader stops before them)
    void save(const std::string& path, bool full_state = false) const;
    void load(const std::string& path, bool full_state = false);

   private:
    void ensure_batch(int B);

    Engine& eng_;
    int device_ = 0;
    int rank_ = 0, S_ = 0;
    float scale_ = 1.f;
    int step_ = 0;
    int64_t n_params_ = 0;
    std::vector<LoraAd> ads_;
    int total_rows_ = 0;          // sum over adapters of 2C
    int64_t aff_per_clip_ = 0;
    float *P_ = nullptr, *G_ = nullptr, *M_ = nullptr, *V_ = nullptr;
    LoraAd* d_ads_ = nullptr;     // device copy of ads_
    int* d_row_ad_ = nullptr;     // adapter of each global row
    // per-batch state of the last forward
    int B_ = 0, B_cap_ = 0;
    bool fwd_done_ = false;
    float *style_ = nullptr, *cond_ = nullptr, *act_ = nullptr, *g_ = nullptr, *h_ = nullptr, *dG_ = nullptr;
    float *aff_ = nullptr, *daff_ = nullptr;
    double* dhg_ = nullptr;
};

}  // namespace bsml
