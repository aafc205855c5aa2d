// ConditioningGate and DecoderLora with the reference's interface
// (include/brosoundml/decoder_lora.h) over this build's bsml_gate_* and
// bsml_lora_* entry points. The brotensor::Tensor members mirror the device-side
// parameter, gradient and moment vectors; see decoder_lora.h.
#include "brosoundml/decoder_lora.h"

#include <cmath>
#include <utility>

#include "brosoundml/kokoro_modules.h"
#include "internal.h"

namespace brosoundml {

namespace bt = brotensor;
using refapi::check;
using refapi::fail;
using refapi::need;
using refapi::need_size;
using refapi::shape_out;
using refapi::sync;

// ─── ConditioningGate ───────────────────────────────────────────────────────
namespace {

// splitmix64 -> xavier-uniform U(-a, a), a = sqrt(6 / (fan_in + fan_out)): parameter
// initialisation, run on the host as the reference's is (decoder_lora.cpp:31-44)
void xavier(bt::Tensor& W, std::uint64_t seed) {
    std::uint64_t s = seed;
    auto next = [&s]() {
        std::uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    const double a = std::sqrt(6.0 / (double)(W.rows + W.cols));
    std::vector<float> h((size_t)W.size());
    for (auto& v : h) v = (float)((((next() >> 40) * (1.0 / 16777216.0)) * 2.0 - 1.0) * a);
    W = bt::Tensor::from_host_on(W.device, h.data(), W.rows, W.cols);
}

}  // namespace

ConditioningGate ConditioningGate::make(int gate_dim, int hidden, bt::Device dev, std::uint64_t seed) {
    need(gate_dim > 0 && gate_dim <= 64 && hidden > 0 && hidden <= 64, "ConditioningGate::make",
         "gate and hidden widths in [1, 64]");
    ConditioningGate g;
    g.gate_dim = gate_dim;
    g.hidden = hidden;
    g.in_dim = 3;
    g.W1 = bt::Tensor::zeros_on(dev, hidden, g.in_dim);
    xavier(g.W1, seed ? seed : 0x9E3779B97F4A7C15ull);
    g.W2 = bt::Tensor::zeros_on(dev, gate_dim, hidden);
    return g;
}

void ConditioningGate::zero_grad() {
    dW1 = bt::Tensor::zeros_on(W1.device, hidden, in_dim);
    dW2 = bt::Tensor::zeros_on(W1.device, gate_dim, hidden);
}

void ConditioningGate::forward(const bt::Tensor& v, bt::Tensor& g) {
    const char* where = "ConditioningGate::forward";
    need_size(v, in_dim, where, "v");
    need_size(W1, (std::int64_t)hidden * in_dim, where, "W1");
    need_size(W2, (std::int64_t)gate_dim * hidden, where, "W2");
    shape_out(act_, hidden, 1, W1);
    shape_out(g, gate_dim, 1, W1);
    // act_ = tanh(W1 v) is what the backward reads; pre1_ (W1 v) is not kept by this build
    check(bsml_gate_forward(W1.f32(), W2.f32(), v.f32(), 1, in_dim, hidden, gate_dim, act_.f32(), g.f32(), nullptr));
    sync();
}

void ConditioningGate::backward(const bt::Tensor& v, const bt::Tensor& dG) {
    const char* where = "ConditioningGate::backward";
    need_size(v, in_dim, where, "v");
    need_size(dG, gate_dim, where, "dG");
    need_size(act_, hidden, where, "the cached activation (no matching forward)");
    if (dW1.size() != (std::int64_t)hidden * in_dim) dW1 = bt::Tensor::zeros_on(W1.device, hidden, in_dim);
    if (dW2.size() != (std::int64_t)gate_dim * hidden) dW2 = bt::Tensor::zeros_on(W1.device, gate_dim, hidden);
    check(bsml_gate_backward(W2.f32(), v.f32(), act_.f32(), dG.f32(), 1, in_dim, hidden, gate_dim, dW1.f32(),
                             dW2.f32(), nullptr));
    sync();
}

// ─── DecoderLora ────────────────────────────────────────────────────────────
namespace {

struct LoraImpl {
    bsml_decoder* h = nullptr;
    bsml_lora* l = nullptr;
    refapi::ParamBuf params;          // the frozen decoder weights, refilled per call
    float *P = nullptr, *G = nullptr, *M = nullptr, *V = nullptr;
    std::int64_t off_W1 = 0, off_W2 = 0;
    std::vector<std::int64_t> offA, offB;
    int hop = 0;
    ~LoraImpl() {
        if (l) bsml_lora_destroy(l);
        if (h) bsml_decoder_destroy(h);
    }
};

LoraImpl& impl(void* p, const char* where) {
    if (!p) fail(where, "the DecoderLora is empty (made by default or moved from)");
    return *static_cast<LoraImpl*>(p);
}

void to_dev(float* dst, const bt::Tensor& t, std::int64_t n, const char* where, const char* what) {
    need_size(t, n, where, what);
    refapi::copy_floats(dst, t.f32(), n);
}

void from_dev(bt::Tensor& t, const float* src) { refapi::copy_floats(t.f32(), src, t.size()); }

}  // namespace

DecoderLora DecoderLora::make(const DecoderBackbone& bb, const Generator& gen, int rank, float scale,
                              bt::Device dev, std::uint64_t seed) {
    const char* where = "DecoderLora::make";
    const bsml_decoder_config cfg = refapi::config_of(&bb, &gen);
    auto* I = new LoraImpl;
    DecoderLora m;
    m.impl_ = I;   // owned by m from here (freed by its destructor on a throw)
    check(bsml_decoder_create(&cfg, 0, &I->h));
    check(bsml_decoder_set_math(I->h, BSML_MATH_TF32X3));
    I->params.init(I->h);
    check(bsml_lora_create(I->h, rank, scale, seed, &I->l));
    std::int64_t n = 0;
    int n_ad = 0, r = 0, S = 0;
    check(bsml_lora_layout(I->l, &n, &n_ad, &r, &S, nullptr, nullptr, nullptr, nullptr, nullptr));
    I->offA.resize(n_ad);
    I->offB.resize(n_ad);
    std::vector<int> C(n_ad);
    check(bsml_lora_layout(I->l, &n, &n_ad, &r, &S, &I->off_W1, &I->off_W2, I->offA.data(), I->offB.data(),
                           C.data()));
    check(bsml_lora_buffers(I->l, &I->P, &I->G));
    check(bsml_lora_moments(I->l, &I->M, &I->V));
    I->hop = gen.hop_size;
    m.rank_ = rank;
    m.scale_ = scale;
    m.style_dim_ = S;
    m.dev_ = dev;
    // adapters in the reference's order (decoder_lora.cpp:173-179), each on its fc
    std::vector<const Linear*> fcs;
    auto blk = [&](const AdainResBlk1dWeights& w) {
        fcs.push_back(&w.norm1.fc);
        fcs.push_back(&w.norm2.fc);
    };
    blk(bb.encode);
    for (const auto& d : bb.decode) blk(d);
    auto rb1 = [&](const AdaINResBlock1Weights& w) {
        for (int j = 0; j < 3; ++j) fcs.push_back(&w.adain1[j].fc);
        for (int j = 0; j < 3; ++j) fcs.push_back(&w.adain2[j].fc);
    };
    for (const auto& w : gen.noise_res) rb1(w);
    for (const auto& w : gen.resblocks) rb1(w);
    need((int)fcs.size() == n_ad, where, "adapter count mismatch");
    m.ads_.resize(n_ad);
    for (int a = 0; a < n_ad; ++a) {
        DecoderLoraAdapter& ad = m.ads_[a];
        ad.fc = fcs[a];
        ad.C = C[a];
        ad.A = bt::Tensor::zeros_on(dev, rank, S);
        ad.B = bt::Tensor::zeros_on(dev, 2 * C[a], rank);
        ad.mA = bt::Tensor::zeros_on(dev, rank, S);
        ad.vA = bt::Tensor::zeros_on(dev, rank, S);
        ad.mB = bt::Tensor::zeros_on(dev, 2 * C[a], rank);
        ad.vB = bt::Tensor::zeros_on(dev, 2 * C[a], rank);
        ad.dA = bt::Tensor::zeros_on(dev, rank, S);
        ad.dB = bt::Tensor::zeros_on(dev, 2 * C[a], rank);
    }
    m.gate_.gate_dim = rank;
    m.gate_.hidden = 16;
    m.gate_.in_dim = 3;
    m.gate_.W1 = bt::Tensor::zeros_on(dev, 16, 3);
    m.gate_.W2 = bt::Tensor::zeros_on(dev, rank, 16);
    m.gate_.zero_grad();
    m.gW1_m_ = bt::Tensor::zeros_on(dev, 16, 3);
    m.gW1_v_ = bt::Tensor::zeros_on(dev, 16, 3);
    m.gW2_m_ = bt::Tensor::zeros_on(dev, rank, 16);
    m.gW2_v_ = bt::Tensor::zeros_on(dev, rank, 16);
    m.pull(true, true, true);
    return m;
}

DecoderLora::~DecoderLora() { delete static_cast<LoraImpl*>(impl_); }

DecoderLora::DecoderLora(DecoderLora&& o) noexcept { *this = std::move(o); }

DecoderLora& DecoderLora::operator=(DecoderLora&& o) noexcept {
    if (this != &o) {
        delete static_cast<LoraImpl*>(impl_);
        rank_ = o.rank_;
        scale_ = o.scale_;
        style_dim_ = o.style_dim_;
        dev_ = o.dev_;
        gate_ = std::move(o.gate_);
        ads_ = std::move(o.ads_);
        gW1_m_ = std::move(o.gW1_m_);
        gW1_v_ = std::move(o.gW1_v_);
        gW2_m_ = std::move(o.gW2_m_);
        gW2_v_ = std::move(o.gW2_v_);
        impl_ = o.impl_;
        o.impl_ = nullptr;
    }
    return *this;
}

std::vector<DecoderLoraAdapter*> DecoderLora::adapters() {
    std::vector<DecoderLoraAdapter*> v;
    for (auto& a : ads_) v.push_back(&a);
    return v;
}

void DecoderLora::push_params() const {
    const char* where = "DecoderLora";
    LoraImpl& I = impl(impl_, where);
    to_dev(I.P + I.off_W1, gate_.W1, 16 * 3, where, "gate W1");
    to_dev(I.P + I.off_W2, gate_.W2, (std::int64_t)rank_ * 16, where, "gate W2");
    for (size_t a = 0; a < ads_.size(); ++a) {
        to_dev(I.P + I.offA[a], ads_[a].A, (std::int64_t)rank_ * style_dim_, where, "adapter A");
        to_dev(I.P + I.offB[a], ads_[a].B, (std::int64_t)2 * ads_[a].C * rank_, where, "adapter B");
    }
}

void DecoderLora::pull(bool params, bool grads, bool moments) {
    LoraImpl& I = impl(impl_, "DecoderLora");
    auto one = [&](const float* base, bt::Tensor& W1, bt::Tensor& W2, auto pick) {
        from_dev(W1, base + I.off_W1);
        from_dev(W2, base + I.off_W2);
        for (size_t a = 0; a < ads_.size(); ++a) {
            from_dev(pick(ads_[a]).first, base + I.offA[a]);
            from_dev(pick(ads_[a]).second, base + I.offB[a]);
        }
    };
    if (params)
        one(I.P, gate_.W1, gate_.W2, [](DecoderLoraAdapter& d) { return std::pair<bt::Tensor&, bt::Tensor&>(d.A, d.B); });
    if (grads)
        one(I.G, gate_.dW1, gate_.dW2,
            [](DecoderLoraAdapter& d) { return std::pair<bt::Tensor&, bt::Tensor&>(d.dA, d.dB); });
    if (moments) {
        one(I.M, gW1_m_, gW2_m_,
            [](DecoderLoraAdapter& d) { return std::pair<bt::Tensor&, bt::Tensor&>(d.mA, d.mB); });
        one(I.V, gW1_v_, gW2_v_,
            [](DecoderLoraAdapter& d) { return std::pair<bt::Tensor&, bt::Tensor&>(d.vA, d.vB); });
    }
    sync();
}

void DecoderLora::forward(const DecoderBackbone& bb, const Generator& gen, const DecoderLoraContext& ctx,
                          const bt::Tensor& cond, bt::Tensor& audio) {
    const char* where = "DecoderLora::forward";
    LoraImpl& I = impl(impl_, where);
    need(ctx.asr && ctx.F0_pred && ctx.N_pred && ctx.ref_s && ctx.har, where, "the context needs every tensor");
    need(ctx.total > 0 && ctx.frames > 1, where, "the context needs total > 0 and frames > 1");
    need_size(cond, 3, where, "cond");
    need(ctx.ref_s->size() >= style_dim_, where, "ref_s is shorter than the style width");
    refapi::fill_backbone(I.params, bb, where);
    refapi::fill_generator(I.params, gen, where);
    push_params();
    shape_out(audio, 1, I.hop * (ctx.frames - 1), *ctx.asr);
    check(bsml_lora_forward(I.l, 1, ctx.total, I.params.data(), ctx.asr->f32(), ctx.F0_pred->f32(),
                            ctx.N_pred->f32(), ctx.ref_s->f32(), (int)ctx.ref_s->size(), ctx.har->f32(),
                            ctx.frames, cond.f32(), audio.f32(), nullptr));
    sync();
}

void DecoderLora::backward(const DecoderBackbone& /*bb*/, const Generator& /*gen*/, const bt::Tensor& cond,
                           const bt::Tensor& dAudio) {
    const char* where = "DecoderLora::backward";
    LoraImpl& I = impl(impl_, where);
    need_size(cond, 3, where, "cond");
    // the engine and the adapters keep the matching forward's activations (cond included)
    check(bsml_lora_backward(I.l, dAudio.f32(), nullptr));
    pull(false, true, false);
}

void DecoderLora::zero_grad() {
    LoraImpl& I = impl(impl_, "DecoderLora::zero_grad");
    check(bsml_lora_zero_grad(I.l, nullptr));
    pull(false, true, false);
}

void DecoderLora::adam_step(float lr, float beta1, float beta2, float eps) {
    LoraImpl& I = impl(impl_, "DecoderLora::adam_step");
    push_params();
    check(bsml_lora_adam_step(I.l, lr, beta1, beta2, eps, nullptr));
    pull(true, false, true);
}

void DecoderLora::save(const std::string& path) const {
    LoraImpl& I = impl(impl_, "DecoderLora::save");
    push_params();
    sync();
    check(bsml_lora_save(I.l, path.c_str()));
}

void DecoderLora::load(const std::string& path) {
    LoraImpl& I = impl(impl_, "DecoderLora::load");
    check(bsml_lora_load(I.l, path.c_str()));
    int step = 0;
    check(bsml_lora_state(I.l, &scale_, &step));
    pull(true, false, false);
}

}  // namespace brosoundml
