// The reference's decoder entry points (brosoundml::detail atoms and assemblies,
// the inference forwards of DecoderBackbone / HarmonicSource / Generator) on the
// GPU engine, through the C ABI (include/bsml_decoder.h).
#include <brotensor/tensor.h>

#include <cmath>
#include <map>
#include <mutex>

#include "internal.h"
#include "kokoro_decoder_backward.h"

namespace brosoundml {

namespace bt = brotensor;
using refapi::check;
using refapi::EngineState;
using refapi::fail;
using refapi::need;
using refapi::need_size;
using refapi::shape_out;
using refapi::sync;

namespace {

constexpr float kEps = 1e-5f;   // the engine's instance-norm epsilon (Kokoro's)

void need_eps(float eps, const char* where) {
    if (std::fabs(eps - kEps) > 1e-9f) fail(where, "this build's fused norms use eps = 1e-5 (Kokoro's)");
}

// (gamma ; beta) of one AdaIN into the packed affine buffer at float offset `off`
void put_affine(EngineState& s, std::int64_t off, int C, const bt::Tensor& g, const bt::Tensor& b, const char* where) {
    need_size(g, C, where, "gamma");
    need_size(b, C, where, "beta");
    refapi::copy_floats(s.aff + off, g.f32(), C);
    refapi::copy_floats(s.aff + off + C, b.f32(), C);
}

void get_affine(const EngineState& s, std::int64_t off, int C, const bt::Tensor& like, bt::Tensor& dg,
                bt::Tensor& db) {
    shape_out(dg, C, 1, like);
    shape_out(db, C, 1, like);
    refapi::copy_floats(dg.f32(), s.daff + off, C);
    refapi::copy_floats(db.f32(), s.daff + off + C, C);
}

// packed offset of each AdaIN (B = 1: the per-clip bases)
std::vector<std::int64_t> aff_offsets(const EngineState& s) {
    std::vector<std::int64_t> o(s.aff_C.size());
    std::int64_t q = 0;
    for (size_t a = 0; a < s.aff_C.size(); ++a) {
        o[a] = q;
        q += 2 * s.aff_C[a];
    }
    return o;
}

EngineState& state_of(const std::shared_ptr<void>& p, const char* where) {
    if (!p) fail(where, "no matching forward (the cache holds no forward state)");
    return *std::static_pointer_cast<EngineState>(p);
}

}  // namespace

namespace detail {

// ─── AdaIN affine ───────────────────────────────────────────────────────────
void adain_affine_forward(const bt::Tensor& x_ncl, const bt::Tensor& gamma, const bt::Tensor& beta, int C, int L,
                          float eps, bt::Tensor& y_ncl, bt::Tensor& x_seq_cache) {
    const char* where = "adain_affine_forward";
    need(C > 0 && L > 0, where, "C and L must be positive");
    need_size(x_ncl, (std::int64_t)C * L, where, "x");
    need_size(gamma, C, where, "gamma");
    need_size(beta, C, where, "beta");
    bt::Tensor gb = bt::Tensor::zeros_on(x_ncl.device, 1, 2 * C);
    refapi::copy_floats(gb.f32(), gamma.f32(), C);
    refapi::copy_floats(gb.f32() + C, beta.f32(), C);
    shape_out(y_ncl, 1, C * L, x_ncl);
    check(bsml_adain_affine_forward(x_ncl.f32(), gb.f32(), 1, C, L, eps, y_ncl.f32(), nullptr));
    // the normalised input in (L, C) sequence layout: the affine with gamma = beta = 0, transposed
    bt::Tensor z = bt::Tensor::zeros_on(x_ncl.device, 1, 2 * C);
    bt::Tensor xn = bt::Tensor::zeros_on(x_ncl.device, 1, C * L);
    check(bsml_adain_affine_forward(x_ncl.f32(), z.f32(), 1, C, L, eps, xn.f32(), nullptr));
    shape_out(x_seq_cache, L, C, x_ncl);
    check(bsml_transpose(xn.f32(), 1, C, L, x_seq_cache.f32(), nullptr));
    sync();
}

void adain_affine_backward(const bt::Tensor& x_ncl, const bt::Tensor& /*x_seq_cache*/, const bt::Tensor& gamma,
                           const bt::Tensor& dY_ncl, int C, int L, float eps, bt::Tensor& dX_ncl, bt::Tensor& dGamma,
                           bt::Tensor& dBeta) {
    const char* where = "adain_affine_backward";
    need(C > 0 && L > 0, where, "C and L must be positive");
    need_size(x_ncl, (std::int64_t)C * L, where, "x");
    need_size(dY_ncl, (std::int64_t)C * L, where, "dY");
    need_size(gamma, C, where, "gamma");
    // the statistics are recomputed from x, as in the reference; beta does not enter the backward
    bt::Tensor gb = bt::Tensor::zeros_on(x_ncl.device, 1, 2 * C);
    refapi::copy_floats(gb.f32(), gamma.f32(), C);
    bt::Tensor dgb = bt::Tensor::zeros_on(x_ncl.device, 1, 2 * C);
    shape_out(dX_ncl, 1, C * L, x_ncl);
    check(bsml_adain_affine_backward(x_ncl.f32(), gb.f32(), dY_ncl.f32(), 1, C, L, eps, dX_ncl.f32(), dgb.f32(),
                                     nullptr));
    shape_out(dGamma, C, 1, x_ncl);
    shape_out(dBeta, C, 1, x_ncl);
    refapi::copy_floats(dGamma.f32(), dgb.f32(), C);
    refapi::copy_floats(dBeta.f32(), dgb.f32() + C, C);
    sync();
}

// ─── AdainResBlk1d ──────────────────────────────────────────────────────────
void adain_resblk_1d_forward_train(const AdainResBlk1dWeights& w, const bt::Tensor& x, int L_in,
                                   const bt::Tensor& gamma1, const bt::Tensor& beta1, const bt::Tensor& gamma2,
                                   const bt::Tensor& beta2, float eps, int& L_out, bt::Tensor& y,
                                   AdainResBlkCache& cache) {
    const char* where = "adain_resblk_1d_forward_train";
    need_eps(eps, where);
    need(L_in > 0, where, "L_in must be positive");
    need_size(x, (std::int64_t)w.channels_in * L_in, where, "x");
    auto s = refapi::block_state(refapi::spec_of(w), cache.state);
    refapi::fill_block(s->params, "", w, where);
    put_affine(*s, 0, w.channels_in, gamma1, beta1, where);
    put_affine(*s, 2 * w.channels_in, w.channels_out, gamma2, beta2, where);
    L_out = w.upsample ? 2 * L_in : L_in;
    shape_out(y, 1, w.channels_out * L_out, x);
    check(bsml_block_forward(s->h, 1, L_in, s->params.data(), x.f32(), nullptr, s->aff, y.f32(), nullptr, nullptr));
    cache.state = s;
    cache.x = x;
    cache.L_in = L_in;
    cache.L_out = L_out;
    sync();
}

void adain_resblk_1d_backward(const AdainResBlk1dWeights& w, const AdainResBlkCache& cache,
                              const bt::Tensor& /*gamma1*/, const bt::Tensor& /*gamma2*/, const bt::Tensor& dY,
                              float eps, bt::Tensor& dX, bt::Tensor& dGamma1, bt::Tensor& dBeta1,
                              bt::Tensor& dGamma2, bt::Tensor& dBeta2) {
    const char* where = "adain_resblk_1d_backward";
    need_eps(eps, where);
    EngineState& s = state_of(cache.state, where);
    need_size(dY, (std::int64_t)w.channels_out * cache.L_out, where, "dY");
    shape_out(dX, 1, w.channels_in * cache.L_in, dY);
    // the (gamma1, gamma2) of the matching forward are in the engine's caches
    check(bsml_block_backward(s.h, dY.f32(), nullptr, dX.f32(), nullptr, s.daff, nullptr));
    get_affine(s, 0, w.channels_in, dY, dGamma1, dBeta1);
    get_affine(s, 2 * w.channels_in, w.channels_out, dY, dGamma2, dBeta2);
    sync();
}

// ─── AdaINResBlock1 ─────────────────────────────────────────────────────────
void adain_resblock1_forward_train(const AdaINResBlock1Weights& w, const bt::Tensor& x_in, int C, int L,
                                   const std::array<bt::Tensor, 3>& g1, const std::array<bt::Tensor, 3>& b1,
                                   const std::array<bt::Tensor, 3>& g2, const std::array<bt::Tensor, 3>& b2,
                                   bt::Tensor& x_out, AdainResBlock1Cache& cache) {
    const char* where = "adain_resblock1_forward_train";
    need(C == w.channels && L > 0, where, "C must equal the block's channels and L be positive");
    need_size(x_in, (std::int64_t)C * L, where, "x_in");
    for (int i = 0; i < 3; ++i) {
        need_eps(w.adain1[i].eps, where);
        need_eps(w.adain2[i].eps, where);
    }
    auto s = refapi::block_state(refapi::spec_of(w), cache.state);
    refapi::fill_rb1(s->params, "", w, where);
    for (int i = 0; i < 3; ++i) put_affine(*s, (std::int64_t)2 * C * i, C, g1[i], b1[i], where);
    for (int i = 0; i < 3; ++i) put_affine(*s, (std::int64_t)2 * C * (3 + i), C, g2[i], b2[i], where);
    shape_out(x_out, 1, C * L, x_in);
    check(bsml_block_forward(s->h, 1, L, s->params.data(), x_in.f32(), nullptr, s->aff, x_out.f32(), nullptr,
                             nullptr));
    cache.state = s;
    cache.x_in[0] = x_in;
    cache.C = C;
    cache.L = L;
    sync();
}

void adain_resblock1_backward(const AdaINResBlock1Weights& w, const AdainResBlock1Cache& cache,
                              const std::array<bt::Tensor, 3>& /*g1*/, const std::array<bt::Tensor, 3>& /*g2*/,
                              const bt::Tensor& dX_out, bt::Tensor& dX_in, std::array<bt::Tensor, 3>& dG1,
                              std::array<bt::Tensor, 3>& dB1, std::array<bt::Tensor, 3>& dG2,
                              std::array<bt::Tensor, 3>& dB2) {
    const char* where = "adain_resblock1_backward";
    EngineState& s = state_of(cache.state, where);
    const int C = cache.C;
    need(C == w.channels, where, "the cache belongs to another block");
    need_size(dX_out, (std::int64_t)C * cache.L, where, "dX_out");
    shape_out(dX_in, 1, C * cache.L, dX_out);
    check(bsml_block_backward(s.h, dX_out.f32(), nullptr, dX_in.f32(), nullptr, s.daff, nullptr));
    for (int i = 0; i < 3; ++i) get_affine(s, (std::int64_t)2 * C * i, C, dX_out, dG1[i], dB1[i]);
    for (int i = 0; i < 3; ++i) get_affine(s, (std::int64_t)2 * C * (3 + i), C, dX_out, dG2[i], dB2[i]);
    sync();
}

// ─── Spectral head ──────────────────────────────────────────────────────────
namespace {
void check_window(const bt::Tensor& window, int n_fft, int win, const char* where) {
    need(win == n_fft, where, "this build's iSTFT uses a window of length n_fft (win == n_fft)");
    need_size(window, win, where, "window");
    const std::vector<float> w = window.to_host_vector();
    for (int n = 0; n < win; ++n) {
        const double h = 0.5 - 0.5 * std::cos(2.0 * 3.14159265358979323846 * n / win);
        if (std::fabs(w[n] - h) > 1e-6)
            fail(where, "this build's iSTFT uses the periodic Hann window (the reference's)");
    }
}
}  // namespace

void spectral_head_forward_train(const Conv1d& conv_post, const bt::Tensor& x, int C, int L,
                                 const bt::Tensor& window, int n_fft, int hop, int win, bt::Tensor& audio,
                                 SpectralHeadCache& cache) {
    const char* where = "spectral_head_forward_train";
    need(C > 0 && L > 1 && hop > 0, where, "C, L and hop must be positive (L at least 2)");
    need_size(x, (std::int64_t)C * L, where, "x");
    check_window(window, n_fft, win, where);
    need(conv_post.in_channels == C && conv_post.out_channels == n_fft + 2 && conv_post.stride == 1 &&
             conv_post.dilation == 1 && conv_post.groups == 1 &&
             conv_post.padding == (conv_post.kernel_size - 1) / 2,
         where, "conv_post must map C to n_fft + 2 channels with 'same' padding");
    need_size(conv_post.W, (std::int64_t)(n_fft + 2) * C * conv_post.kernel_size, where, "conv_post.W");
    cache.x_pre = x;
    cache.C = C;
    cache.L = L;
    shape_out(cache.post, 1, (n_fft + 2) * L, x);
    shape_out(audio, 1, hop * (L - 1), x);
    check(bsml_spectral_head_forward(x.f32(), 1, C, L, conv_post.W.f32(),
                                     conv_post.b.empty() ? nullptr : conv_post.b.f32(), n_fft, hop,
                                     conv_post.kernel_size, cache.post.f32(), audio.f32(), nullptr));
    sync();
}

void spectral_head_backward(const Conv1d& conv_post, const SpectralHeadCache& cache, const bt::Tensor& window,
                            int n_fft, int hop, int win, const bt::Tensor& dAudio, bt::Tensor& dX) {
    const char* where = "spectral_head_backward";
    check_window(window, n_fft, win, where);
    need(cache.C > 0 && cache.L > 1, where, "no matching forward");
    need_size(dAudio, (std::int64_t)hop * (cache.L - 1), where, "dAudio");
    need_size(cache.post, (std::int64_t)(n_fft + 2) * cache.L, where, "cache.post");
    shape_out(dX, 1, cache.C * cache.L, dAudio);
    check(bsml_spectral_head_backward(cache.x_pre.f32(), cache.post.f32(), dAudio.f32(), 1, cache.C, cache.L,
                                      conv_post.W.f32(), n_fft, hop, conv_post.kernel_size, dX.f32(), nullptr));
    sync();
}

// ─── DecoderBackbone assembly ───────────────────────────────────────────────
void decoder_backbone_forward_train(const DecoderBackbone& bb, const bt::Tensor& asr, const bt::Tensor& F0_pred,
                                    const bt::Tensor& N_pred, int T, const std::vector<BlockAffines>& affines,
                                    float eps, bt::Tensor& gen_in, BackboneCache& cache) {
    const char* where = "decoder_backbone_forward_train";
    need_eps(eps, where);
    need(T > 0, where, "T must be positive");
    const bsml_decoder_config cfg = refapi::config_of(&bb, nullptr);
    need_size(asr, (std::int64_t)cfg.asr_dim * T, where, "asr");
    need_size(F0_pred, 2 * (std::int64_t)T, where, "F0_pred");
    need_size(N_pred, 2 * (std::int64_t)T, where, "N_pred");
    need(affines.size() == 1 + bb.decode.size(), where, "one BlockAffines per block (encode first)");
    auto s = refapi::decoder_state(cfg, cache.state);
    refapi::fill_backbone(s->params, bb, where);
    const auto off = aff_offsets(*s);
    for (size_t k = 0; k < affines.size(); ++k) {
        const AdainResBlk1dWeights& w = k == 0 ? bb.encode : bb.decode[k - 1];
        put_affine(*s, off[2 * k], w.channels_in, affines[k].g1, affines[k].b1, where);
        put_affine(*s, off[2 * k + 1], w.channels_out, affines[k].g2, affines[k].b2, where);
    }
    int L = 0;
    check(bsml_backbone_out_len(s->h, T, &L));
    shape_out(gen_in, 1, cfg.dec_out[cfg.n_decode - 1] * L, asr);
    check(bsml_backbone_forward(s->h, 1, T, s->params.data(), asr.f32(), F0_pred.f32(), N_pred.f32(), nullptr, 0,
                                s->aff, gen_in.f32(), nullptr, nullptr));
    s->part_T = T;
    cache.state = s;
    cache.T = T;
    // the concatenation bookkeeping of the reference's cache
    cache.res_applied.assign(bb.decode.size(), 0);
    cache.x_channels.assign(bb.decode.size(), 0);
    bool res = true;
    int Cx = bb.encode.channels_out;
    for (size_t i = 0; i < bb.decode.size(); ++i) {
        cache.res_applied[i] = res ? 1 : 0;
        cache.x_channels[i] = Cx;
        Cx = bb.decode[i].channels_out;
        if (bb.decode[i].upsample) res = false;
    }
    sync();
}

void decoder_backbone_backward(const DecoderBackbone& bb, const BackboneCache& cache,
                               const std::vector<BlockAffines>& /*affines*/, const bt::Tensor& dGenIn, float eps,
                               std::vector<BlockAffines>& dAffines) {
    const char* where = "decoder_backbone_backward";
    need_eps(eps, where);
    EngineState& s = state_of(cache.state, where);
    int L = 0;
    check(bsml_backbone_out_len(s.h, cache.T, &L));
    need_size(dGenIn, (std::int64_t)bb.decode.back().channels_out * L, where, "dGenIn");
    check(bsml_backbone_backward(s.h, dGenIn.f32(), nullptr, nullptr, nullptr, s.daff, nullptr));
    const auto off = aff_offsets(s);
    dAffines.resize(1 + bb.decode.size());
    for (size_t k = 0; k < dAffines.size(); ++k) {
        const AdainResBlk1dWeights& w = k == 0 ? bb.encode : bb.decode[k - 1];
        get_affine(s, off[2 * k], w.channels_in, dGenIn, dAffines[k].g1, dAffines[k].b1);
        get_affine(s, off[2 * k + 1], w.channels_out, dGenIn, dAffines[k].g2, dAffines[k].b2);
    }
    sync();
}

// ─── Generator assembly ─────────────────────────────────────────────────────
namespace {
// generator AdaINs follow the backbone's: noise_res[i] (adain1[0..2], adain2[0..2]),
// then resblocks[k], in the packed order
void put_rb1_affines(EngineState& s, const std::vector<std::int64_t>& off, size_t& a, int C,
                     const ResBlock1Affines& r, const char* where) {
    for (int i = 0; i < 3; ++i) put_affine(s, off[a++], C, r.g1[i], r.b1[i], where);
    for (int i = 0; i < 3; ++i) put_affine(s, off[a++], C, r.g2[i], r.b2[i], where);
}
void get_rb1_affines(const EngineState& s, const std::vector<std::int64_t>& off, size_t& a, int C,
                     const bt::Tensor& like, ResBlock1Affines& r) {
    for (int i = 0; i < 3; ++i) get_affine(s, off[a++], C, like, r.g1[i], r.b1[i]);
    for (int i = 0; i < 3; ++i) get_affine(s, off[a++], C, like, r.g2[i], r.b2[i]);
}
}  // namespace

void generator_forward_train(const Generator& gen, const bt::Tensor& gen_in, int L_in, const bt::Tensor& har,
                             int frames, const std::vector<ResBlock1Affines>& noise_aff,
                             const std::vector<ResBlock1Affines>& res_aff, bt::Tensor& audio,
                             GeneratorCache& cache) {
    const char* where = "generator_forward_train";
    need(L_in > 0 && frames > 1, where, "L_in must be positive and frames at least 2");
    const bsml_decoder_config cfg = refapi::config_of(nullptr, &gen);
    need_size(gen_in, (std::int64_t)cfg.init_ch * L_in, where, "gen_in");
    need_size(har, (std::int64_t)cfg.har_ch * frames, where, "har");
    need((int)noise_aff.size() == gen.num_upsamples && res_aff.size() == gen.resblocks.size(), where,
         "one ResBlock1Affines per noise_res and per resblock");
    auto s = refapi::decoder_state(cfg, cache.state);
    refapi::fill_generator(s->params, gen, where);
    const auto off = aff_offsets(*s);
    size_t a = 2 * (1 + (size_t)cfg.n_decode);   // past the (stand-in) backbone's AdaINs
    for (int i = 0; i < gen.num_upsamples; ++i) put_rb1_affines(*s, off, a, gen.ups_C_out[i], noise_aff[i], where);
    for (size_t k = 0; k < res_aff.size(); ++k)
        put_rb1_affines(*s, off, a, gen.ups_C_out[k / gen.num_kernels], res_aff[k], where);
    shape_out(audio, 1, gen.hop_size * (frames - 1), gen_in);
    check(bsml_generator_forward(s->h, 1, L_in, s->params.data(), gen_in.f32(), har.f32(), frames, nullptr, 0,
                                 s->aff, audio.f32(), nullptr, nullptr));
    s->part_T = L_in;
    cache.state = s;
    // shapes of the reference's per-stage bookkeeping
    cache.stages.assign(gen.num_upsamples, GenStageCache{});
    int L = L_in;
    for (int i = 0; i < gen.num_upsamples; ++i) {
        GenStageCache& g = cache.stages[i];
        g.C_in = gen.ups_C_in[i];
        g.L_in = L;
        g.C_out = gen.ups_C_out[i];
        L = (L - 1) * gen.ups_stride[i] - 2 * gen.ups_pad[i] + gen.ups_k[i] + (i + 1 == gen.num_upsamples ? 1 : 0);
        g.L_out = L;
    }
    cache.head.C = cfg.init_ch >> cfg.n_ups;
    cache.head.L = L;
    sync();
}

void generator_backward(const Generator& gen, const GeneratorCache& cache,
                        const std::vector<ResBlock1Affines>& /*noise_aff*/,
                        const std::vector<ResBlock1Affines>& /*res_aff*/, const bt::Tensor& dAudio,
                        bt::Tensor& dGenIn, std::vector<ResBlock1Affines>& dNoise_aff,
                        std::vector<ResBlock1Affines>& dRes_aff) {
    const char* where = "generator_backward";
    EngineState& s = state_of(cache.state, where);
    need_size(dAudio, (std::int64_t)gen.hop_size * (cache.head.L - 1), where, "dAudio");
    shape_out(dGenIn, 1, gen.ups_C_in[0] * s.part_T, dAudio);
    check(bsml_generator_backward(s.h, dAudio.f32(), nullptr, dGenIn.f32(), nullptr, s.daff, nullptr));
    const auto off = aff_offsets(s);
    std::int64_t n_decode = 0;
    {
        const bsml_decoder_config cfg = refapi::config_of(nullptr, &gen);
        n_decode = cfg.n_decode;
    }
    size_t a = 2 * (1 + (size_t)n_decode);
    dNoise_aff.resize(gen.num_upsamples);
    dRes_aff.resize(gen.resblocks.size());
    for (int i = 0; i < gen.num_upsamples; ++i) get_rb1_affines(s, off, a, gen.ups_C_out[i], dAudio, dNoise_aff[i]);
    for (size_t k = 0; k < gen.resblocks.size(); ++k)
        get_rb1_affines(s, off, a, gen.ups_C_out[k / gen.num_kernels], dAudio, dRes_aff[k]);
    sync();
}

}  // namespace detail

// ─── inference forwards ─────────────────────────────────────────────────────
namespace {

// engines of the const inference forwards, by the calling object's address (the
// architecture is checked on every call, the weights re-read)
std::mutex g_inf_mu;
std::map<const void*, std::shared_ptr<void>> g_inf;

std::shared_ptr<EngineState> inference_state(const void* obj, const bsml_decoder_config& cfg) {
    std::lock_guard<std::mutex> lk(g_inf_mu);
    if (g_inf.size() > 16) g_inf.clear();
    auto s = refapi::decoder_state(cfg, g_inf[obj]);
    g_inf[obj] = s;
    return s;
}

}  // namespace

void DecoderBackbone::forward(const bt::Tensor& asr, const bt::Tensor& F0_pred, const bt::Tensor& N_pred,
                              const bt::Tensor& ref_s, int T, bt::Tensor& gen_in) const {
    const char* where = "DecoderBackbone::forward";
    need(T > 0, where, "T must be positive");
    const bsml_decoder_config cfg = refapi::config_of(this, nullptr);
    need_size(asr, (std::int64_t)cfg.asr_dim * T, where, "asr");
    need_size(F0_pred, 2 * (std::int64_t)T, where, "F0_pred");
    need_size(N_pred, 2 * (std::int64_t)T, where, "N_pred");
    need(ref_s.size() >= cfg.style_dim, where, "ref_s is shorter than the style width");
    auto s = inference_state(this, cfg);
    refapi::fill_backbone(s->params, *this, where);
    int L = 0;
    check(bsml_backbone_out_len(s->h, T, &L));
    shape_out(gen_in, 1, cfg.dec_out[cfg.n_decode - 1] * L, asr);
    check(bsml_backbone_forward(s->h, 1, T, s->params.data(), asr.f32(), F0_pred.f32(), N_pred.f32(), ref_s.f32(),
                                0, nullptr, gen_in.f32(), nullptr, nullptr));
    sync();
}

void Generator::forward(const bt::Tensor& gen_in, int L_in, const bt::Tensor& har, int frames,
                        const bt::Tensor& style, bt::Tensor& audio, const CancelCheck& cancel) const {
    const char* where = "Generator::forward";
    // one engine call covers every stage: the cancel check runs before it
    if (cancel && cancel()) {
        audio = bt::Tensor();
        return;
    }
    need(L_in > 0 && frames > 1, where, "L_in must be positive and frames at least 2");
    const bsml_decoder_config cfg = refapi::config_of(nullptr, this);
    need_size(gen_in, (std::int64_t)cfg.init_ch * L_in, where, "gen_in");
    need_size(har, (std::int64_t)cfg.har_ch * frames, where, "har");
    need(style.size() >= cfg.style_dim, where, "style is shorter than the style width");
    auto s = inference_state(this, cfg);
    refapi::fill_generator(s->params, *this, where);
    shape_out(audio, 1, hop_size * (frames - 1), gen_in);
    check(bsml_generator_forward(s->h, 1, L_in, s->params.data(), gen_in.f32(), har.f32(), frames, style.f32(), 0,
                                 nullptr, audio.f32(), nullptr, nullptr));
    sync();
}

void HarmonicSource::forward(const bt::Tensor& F0_pred, int frame_count, int& signal_len, int& stft_frames,
                             bt::Tensor& har) const {
    const char* where = "HarmonicSource::forward";
    need(frame_count > 0 && upsample_scale > 0 && hop_size > 0, where, "frame_count, upsample_scale, hop_size");
    need(win_size == n_fft, where, "win_size must equal n_fft");
    need(std::fabs(sine_amp - 0.1f) < 1e-9f, where, "this build's source uses sine_amp = 0.1 (Kokoro's)");
    need_size(F0_pred, frame_count, where, "F0_pred");
    need_size(l_linear.W, harmonic_num + 1, where, "l_linear.W");
    need_size(l_linear.b, 1, where, "l_linear.b");
    bsml_decoder_config c{};
    c.upsample_scale = upsample_scale;
    c.harmonic_num = harmonic_num;
    c.sample_rate = sample_rate;
    c.n_fft = n_fft;
    c.hop = hop_size;
    c.har_ch = n_fft + 2;
    signal_len = frame_count * upsample_scale;
    stft_frames = signal_len / hop_size + 1;
    shape_out(har, 1, (n_fft + 2) * stft_frames, F0_pred);
    check(bsml_harmonic_source(&c, F0_pred.f32(), 1, frame_count, l_linear.W.f32(), l_linear.b.f32(), har.f32(),
                               nullptr));
    sync();
}

}  // namespace brosoundml
