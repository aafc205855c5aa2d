// bsml_decoder.hpp — batched C++ layer over the C ABI in bsml_decoder.h
// (namespace brosoundml::b200), with class and function names modelled on the
// reference's (wlejon/brosoundml: include/brosoundml/decoder_lora.h,
// src/kokoro_decoder_backward.h) for callers that train many clips per call.
// Callers of the reference's own signatures use the reference-signature layer
// instead (include/brosoundml/decoder_lora.h, include/kokoro_decoder_backward.h,
// libbsml_ref.so), which takes brotensor::Tensor and runs one clip per call.
//
// Header-only; needs no CUDA header (streams are void*, tensors are device
// float pointers). Differences from the reference interface, all from batching
// and device pointers:
//  * tensors are device pointers with explicit sizes, NCL with a leading batch
//    axis B (B = 1 is the reference's case);
//  * (gamma, beta) travel packed per clip as (B, 2C) rows, and the affines of a
//    block or decoder as one buffer [a][B][2*C_a] in DecoderLora::adapters() order;
//  * the forward caches (AdainResBlkCache, AdainResBlock1Cache, BackboneCache,
//    GeneratorCache) live inside the Block / Decoder object, not in caller structs;
//  * every call takes an optional stream; nothing synchronises except save/load.
// Errors throw std::runtime_error with the library's message, already in the
// reference's format "brosoundml: <where>: <reason>" (src/kokoro_modules.cpp:90-92).
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "bsml_decoder.h"

namespace brosoundml {
namespace b200 {

inline void check(int rc) {
    if (rc < 0) throw std::runtime_error(bsml_last_error());
}

enum class Math {
    FP32 = BSML_MATH_FP32_SIMT,
    TF32X3 = BSML_MATH_TF32X3,
    BF16 = BSML_MATH_BF16,
    BF16X3 = BSML_MATH_BF16X3,
    TF32X3W = BSML_MATH_TF32X3W,
    TF32X3F = BSML_MATH_TF32X3F
};

// Parameter table of an engine handle (names, offsets into the flat buffer).
struct ParamLayout {
    int64_t n_params = 0;
    int64_t aff_per_clip = 0;
    std::vector<bsml_param_entry> table;
    std::vector<int> affine_channels;   // per AdaIN, DecoderLora::adapters() order
};

namespace impl {
inline ParamLayout read_layout(const bsml_decoder* h) {
    ParamLayout L;
    int ne = 0, na = 0;
    check(bsml_decoder_param_count(h, &L.n_params, &ne, &na, &L.aff_per_clip));
    L.table.resize(ne);
    L.affine_channels.resize(na);
    check(bsml_decoder_param_table(h, L.table.data(), ne, L.affine_channels.data()));
    return L;
}

// Owns one bsml_decoder handle (a whole decoder or a single block); move-only.
class Handle {
   public:
    Handle() = default;
    explicit Handle(bsml_decoder* h) : h_(h) {}
    ~Handle() { reset(); }
    Handle(Handle&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
    Handle& operator=(Handle&& o) noexcept {
        if (this != &o) {
            reset();
            h_ = std::exchange(o.h_, nullptr);
        }
        return *this;
    }
    Handle(const Handle&) = delete;
    Handle& operator=(const Handle&) = delete;
    bsml_decoder* get() const { return h_; }
    void reset() {
        if (h_) bsml_decoder_destroy(h_);
        h_ = nullptr;
    }

   private:
    bsml_decoder* h_ = nullptr;
};
}  // namespace impl

// ─── the whole decoder back half ─────────────────────────────────────────────
// forward = decoder_backbone_forward_train + generator_forward_train, backward =
// generator_backward + decoder_backbone_backward (src/kokoro_decoder_backward.h:
// 213-293), batched, with weight gradients beyond the reference's affine grads.
class Decoder {
   public:
    Decoder(const bsml_decoder_config& cfg, int device, Math math = Math::TF32X3) {
        bsml_decoder* h = nullptr;
        check(bsml_decoder_create(&cfg, device, &h));
        h_ = impl::Handle(h);
        check(bsml_decoder_set_math(h, static_cast<int>(math)));
        layout_ = impl::read_layout(h);
        cfg_ = cfg;
    }
    // the parameter layout of a config without a device
    static ParamLayout layout_of(const bsml_decoder_config& cfg) {
        ParamLayout L;
        int ne = 0, na = 0;
        check(bsml_config_param_count(&cfg, &L.n_params, &ne, &na, &L.aff_per_clip));
        L.table.resize(ne);
        L.affine_channels.resize(na);
        check(bsml_config_param_table(&cfg, L.table.data(), ne, L.affine_channels.data()));
        return L;
    }

    const ParamLayout& layout() const { return layout_; }
    const bsml_decoder_config& config() const { return cfg_; }
    bsml_decoder* handle() const { return h_.get(); }
    void set_math(Math m) { check(bsml_decoder_set_math(h_.get(), static_cast<int>(m))); }
    // samples per clip for T asr frames (frames = 0: har from the harmonic source)
    int64_t audio_len(int T, int frames = 0) const {
        const int f = frames > 0 ? frames : (2 * T * cfg_.upsample_scale) / cfg_.hop + 1;
        return (int64_t)cfg_.hop * (f - 1);
    }

    // params: the frozen weights, borrowed until backward() has been enqueued.
    // style (B, style_dim) or aff_in (reference mode); har NULL = harmonic source.
    void forward(int B, int T, const float* params, const float* asr, const float* F0, const float* N,
                 const float* style, const float* har, int frames, float* audio, const float* aff_in = nullptr,
                 float* aff_out = nullptr, void* stream = nullptr) {
        check(bsml_decoder_forward(h_.get(), B, T, params, asr, F0, N, style, har, frames, aff_in, audio, aff_out,
                                   stream));
    }
    // grads (n_params) overwritten; the rest optional
    void backward(const float* daudio, float* grads, float* d_asr = nullptr, float* d_style = nullptr,
                  float* d_aff = nullptr, void* stream = nullptr) {
        check(bsml_decoder_backward(h_.get(), daudio, grads, d_asr, d_style, d_aff, stream));
    }
    // Kokoro::Impl::decode_back_half (src/kokoro.cpp:352-407), batched; ref_s rows of
    // ref_s_stride floats (0 = 2 * style_dim), har from the harmonic source
    void decode(int B, int T, const float* params, const float* ref_s, const float* asr, const float* F0,
                const float* N, float* audio, int ref_s_stride = 0, void* stream = nullptr) {
        check(bsml_decoder_decode(h_.get(), B, T, params, ref_s, ref_s_stride > 0 ? ref_s_stride : 2 * cfg_.style_dim,
                                  asr, F0, N, audio, stream));
    }

   private:
    impl::Handle h_;
    ParamLayout layout_;
    bsml_decoder_config cfg_{};
};

// ─── one block: AdainResBlk1d or AdaINResBlock1 ──────────────────────────────
class Block {
   public:
    Block(const bsml_block_spec& spec, int device, Math math = Math::TF32X3) : spec_(spec) {
        bsml_decoder* h = nullptr;
        check(bsml_block_create(&spec, device, &h));
        h_ = impl::Handle(h);
        check(bsml_decoder_set_math(h, static_cast<int>(math)));
        layout_ = impl::read_layout(h);
    }
    const ParamLayout& layout() const { return layout_; }
    const bsml_block_spec& spec() const { return spec_; }
    int out_len(int L) const { return spec_.kind == BSML_BLOCK_RESBLK1D && spec_.upsample ? 2 * L : L; }
    void forward(int B, int L, const float* params, const float* x, const float* style, float* y,
                 const float* aff_in = nullptr, float* aff_out = nullptr, void* stream = nullptr) {
        check(bsml_block_forward(h_.get(), B, L, params, x, style, aff_in, y, aff_out, stream));
    }
    void backward(const float* dy, float* grads, float* dx, float* d_style = nullptr, float* d_aff = nullptr,
                  void* stream = nullptr) {
        check(bsml_block_backward(h_.get(), dy, grads, dx, d_style, d_aff, stream));
    }

   private:
    impl::Handle h_;
    ParamLayout layout_;
    bsml_block_spec spec_{};
};

// ─── CUDA graph of library calls (capture between begin and end on one stream) ─
class Graph {
   public:
    explicit Graph(void* stream) : stream_(stream) { check(bsml_graph_begin(stream)); }
    ~Graph() {
        if (g_) bsml_graph_destroy(g_);
    }
    Graph(const Graph&) = delete;
    Graph& operator=(const Graph&) = delete;
    void end() { check(bsml_graph_end(stream_, &g_)); }
    void launch(void* stream) const { check(bsml_graph_launch(g_, stream)); }
    int64_t kernels() const {
        int64_t n = 0;
        check(bsml_graph_kernel_count(g_, &n));
        return n;
    }

   private:
    void* stream_ = nullptr;
    bsml_graph* g_ = nullptr;
};

// ─── safetensors checkpoint (host) → flat parameter vector ───────────────────
class SafeTensors {
   public:
    explicit SafeTensors(const std::string& path) { check(bsml_st_open(path.c_str(), &f_)); }
    ~SafeTensors() { bsml_st_close(f_); }
    SafeTensors(const SafeTensors&) = delete;
    SafeTensors& operator=(const SafeTensors&) = delete;
    // host vector in the layout's order; weight-norm pairs fused
    std::vector<float> params(const ParamLayout& L, const std::string& prefix = "decoder.module.") const {
        std::vector<float> p(L.n_params, 0.f);
        check(bsml_params_from_safetensors(f_, L.table.data(), (int)L.table.size(), prefix.c_str(), p.data(),
                                           L.n_params));
        return p;
    }
    std::vector<float> read(const std::string& name, int64_t n) const {
        std::vector<float> v(n);
        check(bsml_st_read_f32(f_, name.c_str(), v.data(), n));
        return v;
    }

   private:
    bsml_st* f_ = nullptr;
};


// ─── DecoderLora (include/brosoundml/decoder_lora.h:36-164) ─────────────────

// Pre-decoder context for B clips; pointers are borrowed for the call
// (decoder_lora.h:82-90). ref_s rows are ref_s_stride floats apart (0 = 2 *
// style_dim, the reference's (1, 2*style_dim) layout); style = the first style_dim.
struct DecoderLoraContext {
    const float* asr = nullptr;       // (B, hidden, T)
    const float* F0_pred = nullptr;   // (B, 2T)
    const float* N_pred = nullptr;    // (B, 2T)
    const float* ref_s = nullptr;     // (B, ref_s_stride)
    const float* har = nullptr;       // (B, har_ch, frames) or NULL: the harmonic source
    int total = 0;                    // T (asr frames)
    int frames = 0;                   // har frames
    int batch = 1;
    int ref_s_stride = 0;
};

// The conditioning gate g(v) = W2 tanh(W1 v) (decoder_lora.h:36-61), as views of
// the DecoderLora's device parameter and gradient vectors.
struct ConditioningGate {
    float* W1 = nullptr;    // (hidden, in_dim)
    float* W2 = nullptr;    // (gate_dim, hidden)
    float* dW1 = nullptr;
    float* dW2 = nullptr;
    int in_dim = 3;
    int hidden = 16;
    int gate_dim = 0;
};

// One adapter (decoder_lora.h:68-77): views of A (rank, style_dim), B (2C, rank)
// and their gradients; the frozen fc stays in the decoder weights.
struct DecoderLoraAdapter {
    int C = 0;
    float* A = nullptr;
    float* B = nullptr;
    float* dA = nullptr;
    float* dB = nullptr;
};

class DecoderLora {
   public:
    // DecoderLora::make (decoder_lora.cpp:115-147) over a decoder engine, which
    // must outlive the returned object. seed 0 = the reference default.
    static DecoderLora make(b200::Decoder& dec, int rank, float scale, std::uint64_t seed) {
        DecoderLora d;
        b200::check(bsml_lora_create(dec.handle(), rank, scale, seed, &d.h_));
        int64_t n = 0, w1 = 0, w2 = 0;
        int na = 0, r = 0, sd = 0;
        b200::check(bsml_lora_layout(d.h_, &n, &na, &r, &sd, &w1, &w2, nullptr, nullptr, nullptr));
        d.off_A_.resize(na);
        d.off_B_.resize(na);
        d.C_.resize(na);
        b200::check(bsml_lora_layout(d.h_, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, d.off_A_.data(),
                                     d.off_B_.data(), d.C_.data()));
        b200::check(bsml_lora_buffers(d.h_, &d.P_, &d.G_));
        d.n_params_ = n;
        d.rank_ = r;
        d.style_dim_ = sd;
        d.off_W1_ = w1;
        d.off_W2_ = w2;
        return d;
    }

    DecoderLora() = default;
    ~DecoderLora() {
        if (h_) bsml_lora_destroy(h_);
    }
    DecoderLora(DecoderLora&& o) noexcept { *this = std::move(o); }
    DecoderLora& operator=(DecoderLora&& o) noexcept {
        if (this != &o) {
            if (h_) bsml_lora_destroy(h_);
            h_ = std::exchange(o.h_, nullptr);
            P_ = o.P_;
            G_ = o.G_;
            n_params_ = o.n_params_;
            rank_ = o.rank_;
            style_dim_ = o.style_dim_;
            off_W1_ = o.off_W1_;
            off_W2_ = o.off_W2_;
            off_A_ = std::move(o.off_A_);
            off_B_ = std::move(o.off_B_);
            C_ = std::move(o.C_);
            weights_ = o.weights_;
            cond_ = o.cond_;
        }
        return *this;
    }
    DecoderLora(const DecoderLora&) = delete;
    DecoderLora& operator=(const DecoderLora&) = delete;

    // Cached forward of ctx.batch clips under conditions cond (B, in_dim) -> audio
    // (B, S). weights = the frozen decoder parameters (the reference's bb + gen),
    // borrowed until the matching backward.
    void forward(const float* weights, const DecoderLoraContext& ctx, const float* cond, float* audio,
                 void* stream = nullptr) {
        const int stride = ctx.ref_s_stride > 0 ? ctx.ref_s_stride : 2 * style_dim_;
        b200::check(bsml_lora_forward(h_, ctx.batch, ctx.total, weights, ctx.asr, ctx.F0_pred, ctx.N_pred, ctx.ref_s,
                                      stride, ctx.har, ctx.frames, cond, audio, stream));
        weights_ = weights;
        cond_ = cond;
    }
    // Backward of the last forward: accumulates every LoRA + gate gradient. The
    // weights and the condition buffer must be the forward's (the gate's
    // activations are cached by the forward, as in the reference).
    void backward(const float* weights, const float* cond, const float* dAudio, void* stream = nullptr) {
        if (weights != weights_)
            throw std::runtime_error("brosoundml: DecoderLora::backward: weights differ from the forward's");
        if (cond != cond_)
            throw std::runtime_error("brosoundml: DecoderLora::backward: cond differs from the forward's");
        b200::check(bsml_lora_backward(h_, dAudio, stream));
    }
    void zero_grad(void* stream = nullptr) { b200::check(bsml_lora_zero_grad(h_, stream)); }
    void adam_step(float lr, float beta1 = 0.9f, float beta2 = 0.999f, float eps = 1e-8f, void* stream = nullptr) {
        b200::check(bsml_lora_adam_step(h_, lr, beta1, beta2, eps, stream));
    }
    void save(const std::string& path) const { b200::check(bsml_lora_save(h_, path.c_str())); }
    void load(const std::string& path) { b200::check(bsml_lora_load(h_, path.c_str())); }
    // ELRA1 plus Adam's moments and step (a resume point; still readable by load())
    void save_state(const std::string& path) const { b200::check(bsml_lora_save_state(h_, path.c_str())); }
    void load_state(const std::string& path) { b200::check(bsml_lora_load_state(h_, path.c_str())); }

    int rank() const { return rank_; }
    float scale() const {
        float s = 0.f;
        int st = 0;
        b200::check(bsml_lora_state(h_, &s, &st));
        return s;
    }
    int step() const {
        float s = 0.f;
        int st = 0;
        b200::check(bsml_lora_state(h_, &s, &st));
        return st;
    }
    ConditioningGate gate() const {
        ConditioningGate g;
        g.W1 = P_ + off_W1_;
        g.W2 = P_ + off_W2_;
        g.dW1 = G_ + off_W1_;
        g.dW2 = G_ + off_W2_;
        g.gate_dim = rank_;
        return g;
    }
    // every adapter (backbone then generator), decoder_lora.cpp:173-179 order
    std::vector<DecoderLoraAdapter> adapters() const {
        std::vector<DecoderLoraAdapter> v(C_.size());
        for (size_t a = 0; a < C_.size(); ++a) {
            v[a].C = C_[a];
            v[a].A = P_ + off_A_[a];
            v[a].B = P_ + off_B_[a];
            v[a].dA = G_ + off_A_[a];
            v[a].dB = G_ + off_B_[a];
        }
        return v;
    }
    // the flat device parameter / gradient vectors (gate W1, W2, then A, B per adapter)
    float* params() const { return P_; }
    float* grads() const { return G_; }
    int64_t n_params() const { return n_params_; }

   private:
    bsml_lora* h_ = nullptr;
    float* P_ = nullptr;
    float* G_ = nullptr;
    int64_t n_params_ = 0, off_W1_ = 0, off_W2_ = 0;
    int rank_ = 0, style_dim_ = 0;
    std::vector<int64_t> off_A_, off_B_;
    std::vector<int> C_;
    const float* weights_ = nullptr;
    const float* cond_ = nullptr;
};

// ─── the reference's detail:: atoms (src/kokoro_decoder_backward.h) ─────────
namespace detail {

// :37-43. gamma_beta (B, 2C) = (gamma ; beta) per clip.
inline void adain_affine_forward(const float* x_ncl, const float* gamma_beta, int B, int C, int L, float eps,
                                 float* y_ncl, void* stream = nullptr) {
    b200::check(bsml_adain_affine_forward(x_ncl, gamma_beta, B, C, L, eps, y_ncl, stream));
}
// :49-56. The instance-norm statistics are recomputed from x (no x_seq cache needed).
inline void adain_affine_backward(const float* x_ncl, const float* gamma_beta, const float* dY_ncl, int B, int C,
                                  int L, float eps, float* dX_ncl, float* dGammaBeta, void* stream = nullptr) {
    b200::check(bsml_adain_affine_backward(x_ncl, gamma_beta, dY_ncl, B, C, L, eps, dX_ncl, dGammaBeta, stream));
}

// :82-111. The cache is the Block (kind BSML_BLOCK_RESBLK1D); affines packed
// [norm1, norm2][B][2C]; eps is the engine's 1e-5.
inline void adain_resblk_1d_forward_train(b200::Block& blk, const float* weights, const float* x, int B, int L_in,
                                          const float* affines, int& L_out, float* y, void* stream = nullptr) {
    blk.forward(B, L_in, weights, x, nullptr, y, affines, nullptr, stream);
    L_out = blk.out_len(L_in);
}
inline void adain_resblk_1d_backward(b200::Block& blk, const float* dY, float* dX, float* dAffines,
                                     float* weight_grads = nullptr, void* stream = nullptr) {
    blk.backward(dY, weight_grads, dX, nullptr, dAffines, stream);
}

// :125-144. The cache is the Block (kind BSML_BLOCK_RESBLOCK1); affines packed
// [adain1[0..2], adain2[0..2]][B][2C].
inline void adain_resblock1_forward_train(b200::Block& blk, const float* weights, const float* x_in, int B, int L,
                                          const float* affines, float* x_out, void* stream = nullptr) {
    blk.forward(B, L, weights, x_in, nullptr, x_out, affines, nullptr, stream);
}
inline void adain_resblock1_backward(b200::Block& blk, const float* dX_out, float* dX_in, float* dAffines,
                                     float* weight_grads = nullptr, void* stream = nullptr) {
    blk.backward(dX_out, weight_grads, dX_in, nullptr, dAffines, stream);
}

// :213-293. One engine runs both assemblies and the spectral head; the affines
// of every AdaIN are packed in adapters() order (reference mode).
inline void decoder_forward_train(b200::Decoder& dec, const float* weights, const float* asr, const float* F0_pred,
                                  const float* N_pred, int B, int T, const float* har, int frames,
                                  const float* affines, float* audio, void* stream = nullptr) {
    dec.forward(B, T, weights, asr, F0_pred, N_pred, nullptr, har, frames, audio, affines, nullptr, stream);
}
inline void decoder_backward(b200::Decoder& dec, const float* dAudio, float* dAffines,
                             float* weight_grads = nullptr, void* stream = nullptr) {
    dec.backward(dAudio, weight_grads, nullptr, nullptr, dAffines, stream);
}

}  // namespace detail
}  // namespace b200
}  // namespace brosoundml
