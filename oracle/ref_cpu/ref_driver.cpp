// Runs the reference's own decoder composition — src/kokoro_decoder_backward.cpp
// and src/decoder_lora.cpp, compiled unchanged from the reference checkout
// against the CPU brotensor stand-ins in this directory — on parameters laid out
// like this repository's flat parameter vector, for the Python tests
// (tests/test_ref_compose_cpu.py) that check oracle/kokoro_oracle.cpp against it.
// Test infrastructure only: nothing in the product loads it.
//
// C entry points (ctypes):
//   refc_decoder_run  the reference's reference-mode decoder (caller-supplied
//                     (gamma, beta) per AdaIN), clip by clip: audio and the
//                     per-AdaIN gradients (decoder_backbone_* + generator_*)
//   refc_lora_run     DecoderLora::make / forward / backward with given adapter
//                     and gate values: audio and every LoRA gradient; optionally
//                     DecoderLora::save to a path (the reference's ELRA1 writer)
//   refc_lora_load    DecoderLora::load from a path (the reference's reader)
#include <cstdio>
#include <cstring>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/bsml_decoder.h"   // bsml_decoder_config (plain C struct)
#include "brosoundml/decoder_lora.h"
#include "brosoundml/kokoro_modules.h"
#include "kokoro_decoder_backward.h"

namespace bt = brotensor;
using namespace brosoundml;

namespace {

thread_local std::string g_err;

struct Params {
    std::map<std::string, const float*> by_name;
    std::map<std::string, int64_t> numel;
    const float* get(const std::string& n, int64_t want) const {
        auto it = by_name.find(n);
        if (it == by_name.end()) throw std::runtime_error("no parameter " + n);
        if (numel.at(n) != want)
            throw std::runtime_error(n + ": " + std::to_string(numel.at(n)) + " != " + std::to_string(want));
        return it->second;
    }
    bt::Tensor t(const std::string& n, int r, int c) const {
        return bt::Tensor::from_host_on(bt::Device::CPU, get(n, (int64_t)r * c), r, c);
    }
};

Params params_of(int n_entries, const char* names, const int64_t* offsets, const int64_t* numels, const float* p) {
    Params P;
    const char* s = names;
    for (int i = 0; i < n_entries; ++i) {
        const std::string n(s);
        s += n.size() + 1;
        P.by_name[n] = p + offsets[i];
        P.numel[n] = numels[i];
    }
    return P;
}

std::string sub(const std::string& p, const std::string& n) { return p.empty() ? n : p + "." + n; }

Conv1d conv(const Params& P, const std::string& n, int cin, int cout, int k, int s, int p, int d, bool bias) {
    Conv1d c;
    c.in_channels = cin; c.out_channels = cout; c.kernel_size = k;
    c.stride = s; c.padding = p; c.dilation = d; c.groups = 1;
    c.W = P.t(n + ".weight", cout, cin * k);
    if (bias) c.b = P.t(n + ".bias", cout, 1);
    return c;
}

AdaIN1dWeights adain(const Params& P, const std::string& n, int C, int S) {
    AdaIN1dWeights a;
    a.channels = C; a.style_dim = S; a.eps = 1e-5f;
    a.fc.in_features = S; a.fc.out_features = 2 * C;
    a.fc.W = P.t(n + ".fc.weight", 2 * C, S);
    a.fc.b = P.t(n + ".fc.bias", 2 * C, 1);
    return a;
}

AdainResBlk1dWeights block(const Params& P, const std::string& n, int cin, int cout, bool up, int S) {
    AdainResBlk1dWeights w;
    w.channels_in = cin; w.channels_out = cout; w.upsample = up; w.learned_sc = cin != cout;
    w.norm1 = adain(P, sub(n, "norm1"), cin, S);
    w.norm2 = adain(P, sub(n, "norm2"), cout, S);
    w.conv1 = conv(P, sub(n, "conv1"), cin, cout, 3, 1, 1, 1, true);
    w.conv2 = conv(P, sub(n, "conv2"), cout, cout, 3, 1, 1, 1, true);
    if (w.learned_sc) w.conv1x1 = conv(P, sub(n, "conv1x1"), cin, cout, 1, 1, 0, 1, false);
    if (up) {
        w.pool_W = P.t(sub(n, "pool.weight"), cin, 3);
        w.pool_b = P.t(sub(n, "pool.bias"), cin, 1);
    }
    return w;
}

AdaINResBlock1Weights rb1(const Params& P, const std::string& n, int C, int k, const int* dil, int S) {
    AdaINResBlock1Weights w;
    w.channels = C; w.kernel_size = k; w.dilations = {dil[0], dil[1], dil[2]};
    for (int i = 0; i < 3; ++i) {
        const std::string s = std::to_string(i);
        w.convs1[i] = conv(P, sub(n, "convs1." + s), C, C, k, 1, (k * dil[i] - dil[i]) / 2, dil[i], true);
        w.convs2[i] = conv(P, sub(n, "convs2." + s), C, C, k, 1, (k - 1) / 2, 1, true);
        w.adain1[i] = adain(P, sub(n, "adain1." + s), C, S);
        w.adain2[i] = adain(P, sub(n, "adain2." + s), C, S);
        w.alpha1[i] = P.t(sub(n, "alpha1." + s), C, 1);
        w.alpha2[i] = P.t(sub(n, "alpha2." + s), C, 1);
    }
    return w;
}

void build(const bsml_decoder_config& c, const Params& P, DecoderBackbone& bb, Generator& gen) {
    const int S = c.style_dim;
    bb.F0_conv = conv(P, "F0_conv", 1, 1, 3, 2, 1, 1, true);
    bb.N_conv = conv(P, "N_conv", 1, 1, 3, 2, 1, 1, true);
    bb.asr_res = conv(P, "asr_res.0", c.asr_dim, c.asr_res_dim, 1, 1, 0, 1, true);
    bb.encode = block(P, "encode", c.asr_dim + 2, c.enc_dim, false, S);
    int x_ch = c.enc_dim;
    bool res = true;
    for (int i = 0; i < c.n_decode; ++i) {
        const int cin = res ? x_ch + c.asr_res_dim + 2 : x_ch;
        const bool up = i == c.upsample_block;
        bb.decode.push_back(block(P, "decode." + std::to_string(i), cin, c.dec_out[i], up, S));
        x_ch = c.dec_out[i];
        if (up) res = false;
    }
    gen.n_fft = c.n_fft; gen.hop_size = c.hop; gen.win_size = c.n_fft;
    gen.num_upsamples = c.n_ups; gen.num_kernels = c.n_kernels;
    for (int i = 0; i < c.n_ups; ++i) {
        const int ci = c.init_ch >> i, co = c.init_ch >> (i + 1), k = c.ups_kernel[i], s = c.ups_rate[i];
        gen.ups_C_in.push_back(ci); gen.ups_C_out.push_back(co);
        gen.ups_k.push_back(k); gen.ups_stride.push_back(s); gen.ups_pad.push_back((k - s) / 2);
        gen.ups_W.push_back(P.t("generator.ups." + std::to_string(i) + ".weight", ci, co * k));
        gen.ups_b.push_back(P.t("generator.ups." + std::to_string(i) + ".bias", co, 1));
        gen.noise_convs.push_back(conv(P, "generator.noise_convs." + std::to_string(i), c.har_ch, co,
                                       c.noise_kernel[i], c.noise_stride[i], c.noise_pad[i], 1, true));
        gen.noise_res.push_back(rb1(P, "generator.noise_res." + std::to_string(i), co, c.nr_kernel[i], c.nr_dil[i], S));
    }
    for (int i = 0; i < c.n_ups; ++i)
        for (int j = 0; j < c.n_kernels; ++j)
            gen.resblocks.push_back(rb1(P, "generator.resblocks." + std::to_string(i * c.n_kernels + j),
                                        c.init_ch >> (i + 1), c.rb_kernel[j], c.rb_dil[j], S));
    gen.conv_post = conv(P, "generator.conv_post", c.init_ch >> c.n_ups, c.n_fft + 2, c.post_kernel, 1,
                         (c.post_kernel - 1) / 2, 1, true);
}

bt::Tensor col(const float* p, int n) { return bt::Tensor::from_host_on(bt::Device::CPU, p, n, 1); }

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // namespace

extern "C" {

const char* refc_last_error() { return g_err.c_str(); }

// aff_in / d_aff: packed [a][B][2 C_a] in DecoderLora::adapters() order (backbone
// blocks norm1, norm2; then noise_res / resblocks adain1[0..2], adain2[0..2])
int refc_decoder_run(const bsml_decoder_config* c, int n_entries, const char* names, const int64_t* offsets,
                     const int64_t* numels, const float* params, int B, int T, const float* asr, const float* F0,
                     const float* N, const float* har, int frames, const float* aff_in, const float* daudio,
                     float* audio, float* d_aff) {
    return guarded([&] {
        const Params P = params_of(n_entries, names, offsets, numels, params);
        DecoderBackbone bb;
        Generator gen;
        build(*c, P, bb, gen);
        // AdaIN channel counts in packing order
        std::vector<int> C;
        C.push_back(bb.encode.channels_in); C.push_back(bb.encode.channels_out);
        for (auto& d : bb.decode) { C.push_back(d.channels_in); C.push_back(d.channels_out); }
        for (size_t r = 0; r < gen.noise_res.size() + gen.resblocks.size(); ++r) {
            const int ch = r < gen.noise_res.size() ? gen.noise_res[r].channels
                                                    : gen.resblocks[r - gen.noise_res.size()].channels;
            for (int q = 0; q < 6; ++q) C.push_back(ch);
        }
        std::vector<int64_t> base(C.size());
        int64_t tot = 0;
        for (size_t a = 0; a < C.size(); ++a) { base[a] = tot; tot += (int64_t)B * 2 * C[a]; }
        const int S_len = c->hop * (frames - 1);
        for (int b = 0; b < B; ++b) {
            auto gb = [&](size_t a, int which) {   // gamma (0) or beta (1) of AdaIN a, clip b
                return col(aff_in + base[a] + (int64_t)b * 2 * C[a] + which * C[a], C[a]);
            };
            std::vector<detail::BlockAffines> bba(1 + bb.decode.size());
            size_t a = 0;
            for (auto& x : bba) {
                x.g1 = gb(a, 0); x.b1 = gb(a, 1); ++a;
                x.g2 = gb(a, 0); x.b2 = gb(a, 1); ++a;
            }
            auto rb_aff = [&](detail::ResBlock1Affines& r) {
                for (int i = 0; i < 3; ++i) { r.g1[i] = gb(a, 0); r.b1[i] = gb(a, 1); ++a; }
                for (int i = 0; i < 3; ++i) { r.g2[i] = gb(a, 0); r.b2[i] = gb(a, 1); ++a; }
            };
            std::vector<detail::ResBlock1Affines> na(gen.noise_res.size()), ra(gen.resblocks.size());
            for (auto& r : na) rb_aff(r);
            for (auto& r : ra) rb_aff(r);
            const bt::Tensor asr_b = bt::Tensor::from_host_on(bt::Device::CPU, asr + (int64_t)b * c->asr_dim * T, 1,
                                                              c->asr_dim * T);
            const bt::Tensor F0_b = bt::Tensor::from_host_on(bt::Device::CPU, F0 + (int64_t)b * 2 * T, 1, 2 * T);
            const bt::Tensor N_b = bt::Tensor::from_host_on(bt::Device::CPU, N + (int64_t)b * 2 * T, 1, 2 * T);
            const bt::Tensor har_b = bt::Tensor::from_host_on(
                bt::Device::CPU, har + (int64_t)b * c->har_ch * frames, 1, c->har_ch * frames);
            detail::BackboneCache bbc;
            detail::GeneratorCache gc;
            bt::Tensor gen_in, au;
            detail::decoder_backbone_forward_train(bb, asr_b, F0_b, N_b, T, bba, 1e-5f, gen_in, bbc);
            detail::generator_forward_train(gen, gen_in, 2 * T, har_b, frames, na, ra, au, gc);
            if (au.size() != S_len) throw std::runtime_error("audio length mismatch");
            std::memcpy(audio + (int64_t)b * S_len, au.f(), sizeof(float) * S_len);
            if (!daudio) continue;
            const bt::Tensor da = bt::Tensor::from_host_on(bt::Device::CPU, daudio + (int64_t)b * S_len, 1, S_len);
            bt::Tensor dgen;
            std::vector<detail::ResBlock1Affines> dna, dra;
            detail::generator_backward(gen, gc, na, ra, da, dgen, dna, dra);
            std::vector<detail::BlockAffines> dbb;
            detail::decoder_backbone_backward(bb, bbc, bba, dgen, 1e-5f, dbb);
            auto put = [&](size_t aa, const bt::Tensor& g, const bt::Tensor& be) {
                float* o = d_aff + base[aa] + (int64_t)b * 2 * C[aa];
                std::memcpy(o, g.f(), sizeof(float) * C[aa]);
                std::memcpy(o + C[aa], be.f(), sizeof(float) * C[aa]);
            };
            a = 0;
            for (auto& x : dbb) { put(a++, x.g1, x.b1); put(a++, x.g2, x.b2); }
            auto put_rb = [&](const detail::ResBlock1Affines& r) {
                for (int i = 0; i < 3; ++i) put(a++, r.g1[i], r.b1[i]);
                for (int i = 0; i < 3; ++i) put(a++, r.g2[i], r.b2[i]);
            };
            for (auto& r : dna) put_rb(r);
            for (auto& r : dra) put_rb(r);
        }
    });
}

// LoRA parameters / gradients in this repository's layout: gate W1 [16][3] at
// off_W1, W2 [rank][16] at off_W2, per adapter A [rank][S] at off_A[a], B [2C][rank]
// at off_B[a]. One clip; ref_s (2 * style_dim), cond (3).
int refc_lora_run(const bsml_decoder_config* c, int n_entries, const char* names, const int64_t* offsets,
                  const int64_t* numels, const float* params, int T, const float* asr, const float* F0,
                  const float* N, const float* ref_s, const float* har, int frames, int rank, float scale,
                  const float* lp, int64_t off_W1, int64_t off_W2, const int64_t* off_A, const int64_t* off_B,
                  const float* cond, const float* daudio, float* audio, float* lgrad, const char* save_path) {
    return guarded([&] {
        const Params P = params_of(n_entries, names, offsets, numels, params);
        DecoderBackbone bb;
        Generator gen;
        build(*c, P, bb, gen);
        DecoderLora lora = DecoderLora::make(bb, gen, rank, scale, bt::Device::CPU, 1);
        auto ads = lora.adapters();
        const int S = c->style_dim;
        for (size_t a = 0; a < ads.size(); ++a) {
            ads[a]->A = bt::Tensor::from_host_on(bt::Device::CPU, lp + off_A[a], rank, S);
            ads[a]->B = bt::Tensor::from_host_on(bt::Device::CPU, lp + off_B[a], 2 * ads[a]->C, rank);
        }
        lora.gate().W1 = bt::Tensor::from_host_on(bt::Device::CPU, lp + off_W1, 16, 3);
        lora.gate().W2 = bt::Tensor::from_host_on(bt::Device::CPU, lp + off_W2, rank, 16);
        const bt::Tensor asr_t = bt::Tensor::from_host_on(bt::Device::CPU, asr, 1, c->asr_dim * T);
        const bt::Tensor F0_t = bt::Tensor::from_host_on(bt::Device::CPU, F0, 1, 2 * T);
        const bt::Tensor N_t = bt::Tensor::from_host_on(bt::Device::CPU, N, 1, 2 * T);
        const bt::Tensor ref_t = bt::Tensor::from_host_on(bt::Device::CPU, ref_s, 1, 2 * S);
        const bt::Tensor har_t = bt::Tensor::from_host_on(bt::Device::CPU, har, 1, c->har_ch * frames);
        const bt::Tensor cond_t = bt::Tensor::from_host_on(bt::Device::CPU, cond, 3, 1);
        DecoderLoraContext ctx{&asr_t, &F0_t, &N_t, &ref_t, &har_t, T, frames};
        bt::Tensor au;
        lora.zero_grad();
        lora.forward(bb, gen, ctx, cond_t, au);
        std::memcpy(audio, au.f(), sizeof(float) * au.size());
        if (daudio) {
            const bt::Tensor da = bt::Tensor::from_host_on(bt::Device::CPU, daudio, 1, (int)au.size());
            lora.backward(bb, gen, cond_t, da);
            for (size_t a = 0; a < ads.size(); ++a) {
                std::memcpy(lgrad + off_A[a], ads[a]->dA.f(), sizeof(float) * ads[a]->dA.size());
                std::memcpy(lgrad + off_B[a], ads[a]->dB.f(), sizeof(float) * ads[a]->dB.size());
            }
            std::memcpy(lgrad + off_W1, lora.gate().dW1.f(), sizeof(float) * 48);
            std::memcpy(lgrad + off_W2, lora.gate().dW2.f(), sizeof(float) * rank * 16);
        }
        if (save_path && *save_path) lora.save(save_path);
    });
}

// DecoderLora::load of `path` into an object of the given architecture; the
// restored values in this repository's LoRA layout, and the file's scale
int refc_lora_load(const bsml_decoder_config* c, int n_entries, const char* names, const int64_t* offsets,
                   const int64_t* numels, const float* params, int rank, const char* path, int64_t off_W1,
                   int64_t off_W2, const int64_t* off_A, const int64_t* off_B, float* lp, float* scale) {
    return guarded([&] {
        const Params P = params_of(n_entries, names, offsets, numels, params);
        DecoderBackbone bb;
        Generator gen;
        build(*c, P, bb, gen);
        DecoderLora lora = DecoderLora::make(bb, gen, rank, 1.0f, bt::Device::CPU, 7);
        lora.load(path);
        auto ads = lora.adapters();
        for (size_t a = 0; a < ads.size(); ++a) {
            std::memcpy(lp + off_A[a], ads[a]->A.f(), sizeof(float) * ads[a]->A.size());
            std::memcpy(lp + off_B[a], ads[a]->B.f(), sizeof(float) * ads[a]->B.size());
        }
        std::memcpy(lp + off_W1, lora.gate().W1.f(), sizeof(float) * 48);
        std::memcpy(lp + off_W2, lora.gate().W2.f(), sizeof(float) * rank * 16);
        *scale = lora.scale();
    });
}

}  // extern "C"
