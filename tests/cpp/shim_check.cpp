// Exercises include/bsml_decoder.hpp (the C++ layer with the reference's names)
// through libbsml_b200.so. Test fixture: built and run by tests/test_cpp_shim_*.py.
//   shim_check layout <config.bin>   no device: layout queries and error paths
//   shim_check gpu <config.bin> <dir>  DecoderLora life cycle on device 0
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "bsml_decoder.hpp"

#ifdef SHIM_GPU
#include <cuda_runtime.h>
#endif

namespace bb = brosoundml::b200;

static bsml_decoder_config read_cfg(const char* path) {
    bsml_decoder_config c{};
    FILE* f = std::fopen(path, "rb");
    if (!f || std::fread(&c, sizeof(c), 1, f) != 1) {
        std::fprintf(stderr, "cannot read %s\n", path);
        std::exit(2);
    }
    std::fclose(f);
    return c;
}

#define EXPECT(cond)                                                      \
    do {                                                                  \
        if (!(cond)) {                                                    \
            std::fprintf(stderr, "FAILED %s at line %d\n", #cond, __LINE__); \
            return 1;                                                     \
        }                                                                 \
    } while (0)

static int layout_mode(const bsml_decoder_config& cfg) {
    const bb::ParamLayout L = bb::Decoder::layout_of(cfg);
    std::printf("n_params %lld entries %zu affines %zu\n", (long long)L.n_params, L.table.size(),
                L.affine_channels.size());
    bsml_block_spec bad{};
    bad.kind = 9;
    try {
        bb::Block blk(bad, 0);
        return 1;
    } catch (const std::runtime_error& e) {
        EXPECT(std::strncmp(e.what(), "brosoundml: ", 12) == 0);
        std::printf("block error: %s\n", e.what());
    }
    // without a device the engine cannot be created: a runtime_error, not a crash
    try {
        bb::Decoder d(cfg, 0);
        std::printf("decoder created\n");
    } catch (const std::runtime_error& e) {
        EXPECT(std::strncmp(e.what(), "brosoundml: ", 12) == 0);
        std::printf("decoder error: %s\n", e.what());
    }
    return 0;
}

#ifdef SHIM_GPU
struct Dev {
    float* p = nullptr;
    size_t n = 0;
    explicit Dev(size_t n_, const std::vector<float>* h = nullptr) : n(n_) {
        cudaMalloc(&p, sizeof(float) * (n ? n : 1));
        if (h) cudaMemcpy(p, h->data(), sizeof(float) * n, cudaMemcpyHostToDevice);
        else cudaMemset(p, 0, sizeof(float) * (n ? n : 1));
    }
    ~Dev() { cudaFree(p); }
    std::vector<float> host() const {
        std::vector<float> h(n);
        cudaMemcpy(h.data(), p, sizeof(float) * n, cudaMemcpyDeviceToHost);
        return h;
    }
};

static std::vector<float> rnd(size_t n, std::mt19937& g, float lo, float hi) {
    std::uniform_real_distribution<float> u(lo, hi);
    std::vector<float> v(n);
    for (auto& x : v) x = u(g);
    return v;
}

static int gpu_mode(const bsml_decoder_config& cfg, const std::string& dir) {
    std::mt19937 g(7);
    const int B = 2, T = 4;
    bb::Decoder dec(cfg, 0, bb::Math::FP32);
    const auto& L = dec.layout();
    std::vector<float> w = rnd(L.n_params, g, -0.3f, 0.3f);
    for (const auto& e : L.table)
        if (std::strstr(e.name, ".alpha")) std::fill(w.begin() + e.offset, w.begin() + e.offset + e.numel, 1.f);
    Dev W(L.n_params, &w);
    const int frames = (2 * T * cfg.upsample_scale) / cfg.hop + 1;
    std::vector<float> asr = rnd((size_t)B * cfg.asr_dim * T, g, -1, 1), F0 = rnd((size_t)B * 2 * T, g, 80, 300),
                       Nn = rnd((size_t)B * 2 * T, g, -1, 1), ref = rnd((size_t)B * 2 * cfg.style_dim, g, -1, 1),
                       har = rnd((size_t)B * cfg.har_ch * frames, g, -0.4f, 0.4f);
    Dev dA(asr.size(), &asr), dF(F0.size(), &F0), dN(Nn.size(), &Nn), dR(ref.size(), &ref), dH(har.size(), &har);
    const size_t S = (size_t)dec.audio_len(T, frames);
    Dev audio(B * S), audio_base(B * S), daudio(B * S);

    auto lora = bb::DecoderLora::make(dec, 4, 2.0f, 0);
    EXPECT(lora.rank() == 4 && std::fabs(lora.scale() - 2.0f) < 1e-6f);
    EXPECT(lora.adapters().size() == L.affine_channels.size());
    const bb::ConditioningGate gate = lora.gate();
    std::vector<float> w2(gate.gate_dim * gate.hidden);
    cudaMemcpy(w2.data(), gate.W2, sizeof(float) * w2.size(), cudaMemcpyDeviceToHost);
    for (float v : w2) EXPECT(v == 0.f);   // W2 = 0 at make

    bb::DecoderLoraContext ctx;
    ctx.asr = dA.p; ctx.F0_pred = dF.p; ctx.N_pred = dN.p; ctx.ref_s = dR.p; ctx.har = dH.p;
    ctx.total = T; ctx.frames = frames; ctx.batch = B;
    std::vector<float> c = rnd((size_t)B * 3, g, -1, 1);
    Dev cond(c.size(), &c);
    // neutral identity: with W2 = 0 the adapted decoder is the base decoder on fc(style)
    lora.forward(W.p, ctx, cond.p, audio.p);
    // the base decoder reads style = the first style_dim of each ref_s row
    std::vector<float> style((size_t)B * cfg.style_dim);
    for (int b = 0; b < B; ++b)
        std::memcpy(&style[(size_t)b * cfg.style_dim], &ref[(size_t)b * 2 * cfg.style_dim], sizeof(float) * cfg.style_dim);
    Dev dS(style.size(), &style);
    bb::Decoder base(cfg, 0, bb::Math::FP32);
    base.forward(B, T, W.p, dA.p, dF.p, dN.p, dS.p, dH.p, frames, audio_base.p);
    cudaDeviceSynchronize();
    const auto a1 = audio.host(), a0 = audio_base.host();
    double num = 0, den = 0;
    for (size_t i = 0; i < a1.size(); ++i) { num += (a1[i] - a0[i]) * (a1[i] - a0[i]); den += a0[i] * a0[i]; }
    std::printf("neutral identity rel %.3e\n", std::sqrt(num / den));
    EXPECT(std::sqrt(num / den) < 1e-5);

    // open the gate, one training step, checkpoint round trip
    std::vector<float> w2n = rnd(w2.size(), g, -0.3f, 0.3f);
    cudaMemcpy(gate.W2, w2n.data(), sizeof(float) * w2n.size(), cudaMemcpyHostToDevice);
    lora.forward(W.p, ctx, cond.p, audio.p);
    std::vector<float> da = rnd(B * S, g, -1, 1);
    cudaMemcpy(daudio.p, da.data(), sizeof(float) * da.size(), cudaMemcpyHostToDevice);
    lora.zero_grad();
    lora.backward(W.p, cond.p, daudio.p);
    try {
        lora.backward(audio_base.p, cond.p, daudio.p);
        return 1;
    } catch (const std::runtime_error& e) {
        EXPECT(std::strncmp(e.what(), "brosoundml: DecoderLora::backward", 33) == 0);
    }
    lora.adam_step(1e-3f);
    EXPECT(lora.step() == 1);
    std::vector<float> gW2(w2.size());
    cudaMemcpy(gW2.data(), gate.dW2, sizeof(float) * gW2.size(), cudaMemcpyDeviceToHost);
    double gn = 0;
    for (float v : gW2) gn += std::fabs(v);
    EXPECT(gn > 0);
    const std::string path = dir + "/shim.elra";
    lora.save(path);
    std::vector<float> saved(lora.n_params());
    cudaMemcpy(saved.data(), lora.params(), sizeof(float) * saved.size(), cudaMemcpyDeviceToHost);
    cudaMemset(lora.params(), 0, sizeof(float) * saved.size());
    lora.load(path);
    std::vector<float> back(lora.n_params());
    cudaMemcpy(back.data(), lora.params(), sizeof(float) * back.size(), cudaMemcpyDeviceToHost);
    EXPECT(std::memcmp(saved.data(), back.data(), sizeof(float) * saved.size()) == 0);
    // full training state: a fresh object resumes at the same step
    lora.save_state(dir + "/state.elra");
    auto resumed = bb::DecoderLora::make(dec, 4, 2.0f, 99);
    resumed.load_state(dir + "/state.elra");
    EXPECT(resumed.step() == lora.step());
    lora.load(dir + "/state.elra");   // the plain reader stops before the optimiser state
    // decode needs the built-in harmonic source, which this config (har_ch != n_fft + 2) cannot use
    try {
        base.decode(B, T, W.p, dR.p, dA.p, dF.p, dN.p, audio.p);
        return 1;
    } catch (const std::runtime_error& e) {
        EXPECT(std::strstr(e.what(), "harmonic source") != nullptr);
    }
    // a replayed graph of the base forward reproduces the eager audio
    cudaStream_t s = nullptr;
    cudaStreamCreate(&s);
    base.forward(B, T, W.p, dA.p, dF.p, dN.p, dS.p, dH.p, frames, audio_base.p, nullptr, nullptr, s);
    cudaStreamSynchronize(s);
    const auto e0 = audio_base.host();
    {
        bb::Graph g(s);
        base.forward(B, T, W.p, dA.p, dF.p, dN.p, dS.p, dH.p, frames, audio_base.p, nullptr, nullptr, s);
        g.end();
        EXPECT(g.kernels() > 10);
        cudaMemsetAsync(audio_base.p, 0, sizeof(float) * B * S, s);
        g.launch(s);
        cudaStreamSynchronize(s);
    }
    const auto e1 = audio_base.host();
    double dn = 0, dd = 0;
    for (size_t i = 0; i < e0.size(); ++i) { dn += (e1[i] - e0[i]) * (e1[i] - e0[i]); dd += e0[i] * e0[i]; }
    EXPECT(std::sqrt(dn / dd) < 1e-6);
    cudaStreamDestroy(s);
    // move-only ownership
    bb::DecoderLora moved = std::move(lora);
    EXPECT(moved.rank() == 4);
    std::printf("OK\n");
    return 0;
}
#endif

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    const bsml_decoder_config cfg = read_cfg(argv[2]);
    try {
        if (std::strcmp(argv[1], "layout") == 0) return layout_mode(cfg);
#ifdef SHIM_GPU
        if (std::strcmp(argv[1], "gpu") == 0 && argc > 3) return gpu_mode(cfg, argv[3]);
#endif
    } catch (const std::exception& e) {
        std::fprintf(stderr, "exception: %s\n", e.what());
        return 1;
    }
    return 2;
}
