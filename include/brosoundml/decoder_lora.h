// brosoundml/decoder_lora.h — the trainable LoRA over the Kokoro decoder's AdaIN
// style -> (gamma, beta) projections, with the reference's classes, members and
// signatures (include/brosoundml/decoder_lora.h:36-164 in the reference):
// ConditioningGate, DecoderLoraAdapter, DecoderLoraContext and DecoderLora.
//
// The arithmetic runs on the GPU (this build's bsml_lora_* and bsml_gate_* entry
// points, include/bsml_decoder.h). The brotensor::Tensor members are the
// caller-visible copies of the parameters and gradients: DecoderLora writes the
// parameter tensors (A, B, gate W1 / W2) to the device before every call that
// reads them and brings back parameters, gradients and Adam moments after every
// call that changes them, so a caller may read or edit them between calls as with
// the reference.
#pragma once

#include <brotensor/tensor.h>

#include <array>
#include <cstdint>
#include <string>
#include <vector>

namespace brosoundml {

struct Linear;
struct DecoderBackbone;
struct Generator;

// g(v) = W2 tanh(W1 v), no biases (so g(0) = 0); W2 zero at creation.
//   v (in_dim, 1), W1 (hidden, in_dim), W2 (gate_dim, hidden), g (gate_dim, 1)
struct ConditioningGate {
    brotensor::Tensor W1, W2;
    brotensor::Tensor dW1, dW2;   // accumulated until zero_grad()
    int in_dim = 3;
    int hidden = 0;
    int gate_dim = 0;

    brotensor::Tensor pre1_;      // W1 v (not kept by this build: the backward reads act_)
    brotensor::Tensor act_;       // cached by forward(): tanh(W1 v)

    // W1 xavier-uniform from `seed` (0: a fixed default), W2 zero
    static ConditioningGate make(int gate_dim, int hidden, brotensor::Device dev, std::uint64_t seed);
    void zero_grad();
    void forward(const brotensor::Tensor& v, brotensor::Tensor& g);
    // accumulates dW1, dW2 from dG (gate_dim, 1); v as in the matching forward
    void backward(const brotensor::Tensor& v, const brotensor::Tensor& dG);
};

// One adapter on one AdaIN fc: (gamma, beta) = fc(s) + scale * B (g(v) * (A s)).
struct DecoderLoraAdapter {
    const Linear* fc = nullptr;        // the frozen base projection (2C outputs)
    int C = 0;
    brotensor::Tensor A, B;            // (rank, style_dim), (2C, rank)
    brotensor::Tensor mA, vA, mB, vB;  // Adam moments
    brotensor::Tensor dA, dB;          // gradient accumulators
    brotensor::Tensor h, hg;           // bottleneck of the last forward (not filled by this build)
};

// The frozen decoder inputs of one clip; pointers are borrowed for the call.
struct DecoderLoraContext {
    const brotensor::Tensor* asr = nullptr;      // (1, C_asr * T)
    const brotensor::Tensor* F0_pred = nullptr;  // (1, 2T)
    const brotensor::Tensor* N_pred = nullptr;   // (1, 2T)
    const brotensor::Tensor* ref_s = nullptr;    // (1, 2 * style_dim): style = first style_dim
    const brotensor::Tensor* har = nullptr;      // (1, har_ch * frames)
    int total = 0;                               // T
    int frames = 0;                              // har frames
};

// Adapters on every AdaIN fc of the backbone (2 per block) and the generator (6
// per AdaINResBlock1), the shared gate, Adam, ELRA1 checkpoints.
class DecoderLora {
   public:
    static DecoderLora make(const DecoderBackbone& bb, const Generator& gen, int rank, float scale,
                            brotensor::Device dev, std::uint64_t seed);

    DecoderLora() = default;
    ~DecoderLora();
    DecoderLora(DecoderLora&&) noexcept;
    DecoderLora& operator=(DecoderLora&&) noexcept;
    DecoderLora(const DecoderLora&) = delete;
    DecoderLora& operator=(const DecoderLora&) = delete;

    // decode ctx under the condition cond (in_dim, 1) -> audio (1, S); cond = 0
    // reproduces the base decoder
    void forward(const DecoderBackbone& bb, const Generator& gen, const DecoderLoraContext& ctx,
                 const brotensor::Tensor& cond, brotensor::Tensor& audio);
    // accumulates every adapter and gate gradient from dAudio; follows the
    // matching forward (same cond)
    void backward(const DecoderBackbone& bb, const Generator& gen, const brotensor::Tensor& cond,
                  const brotensor::Tensor& dAudio);

    void zero_grad();
    void adam_step(float lr, float beta1 = 0.9f, float beta2 = 0.999f, float eps = 1e-8f);

    void save(const std::string& path) const;
    void load(const std::string& path);

    int rank() const { return rank_; }
    float scale() const { return scale_; }
    ConditioningGate& gate() { return gate_; }
    const ConditioningGate& gate() const { return gate_; }
    // every adapter, backbone then generator (noise_res, then resblocks)
    std::vector<DecoderLoraAdapter*> adapters();

   private:
    int rank_ = 0;
    float scale_ = 1.0f;
    int style_dim_ = 0;
    brotensor::Device dev_ = brotensor::Device::CPU;
    ConditioningGate gate_;
    std::vector<DecoderLoraAdapter> ads_;   // adapters() order
    brotensor::Tensor gW1_m_, gW1_v_, gW2_m_, gW2_v_;
    void* impl_ = nullptr;                  // the device-side model (opaque)

    void push_params() const;
    void pull(bool params, bool grads, bool moments);
};

}  // namespace brosoundml
