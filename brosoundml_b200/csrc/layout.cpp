#include "layout.h"

#include <cstdio>
#include <cstring>

#include "common.cuh"

#include <atomic>

namespace bsml {

namespace {
std::atomic<int64_t> g_launches{0};
}
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
int64_t launch_count() { return g_launches.load(std::memory_order_relaxed); }

namespace {
// "a.b" module-key join; an empty prefix gives the block-relative key
std::string sub(const std::string& n, const std::string& s) { return n.empty() ? s : n + "." + s; }
}  // namespace

int64_t Layout::add(const std::string& name, int nd, int s0, int s1, int s2, bool train) {
    bsml_param_entry e{};
    std::snprintf(e.name, sizeof(e.name), "%s", name.c_str());
    e.ndim = nd;
    e.shape[0] = s0;
    e.shape[1] = s1;
    e.shape[2] = s2;
    e.numel = (int64_t)s0 * (nd > 1 ? s1 : 1) * (nd > 2 ? s2 : 1);
    e.trainable = train ? 1 : 0;
    e.offset = total;
    total += round_up(e.numel, 64);   // 256-byte aligned tensors
    table.push_back(e);
    return e.offset;
}

ConvP Layout::conv(const std::string& n, int cout, int cin, int k, int s, int p, int d, bool bias) {
    ConvP c;
    c.cout = cout; c.cin = cin; c.k = k; c.s = s; c.p = p; c.d = d;
    c.w = add(n + ".weight", 3, cout, cin, k, true);
    if (bias) c.b = add(n + ".bias", 1, cout, 1, 1, true);
    return c;
}

AdaP Layout::adain(const std::string& n, int C) {
    AdaP a;
    a.C = C;
    a.fw = add(n + ".fc.weight", 2, 2 * C, cfg.style_dim, 1, true);
    a.fb = add(n + ".fc.bias", 1, 2 * C, 1, 1, true);
    return a;
}

// AdainResBlk1d weights, kokoro_modules.cpp:747-767 (conv1x1 has no bias; pool is
// a depthwise ConvTranspose1d (C_in, 1, 3) with bias).
BlkP Layout::blk(const std::string& n, int cin, int cout, bool up) {
    BlkP b;
    b.cin = cin; b.cout = cout; b.up = up; b.sc = cin != cout;
    b.n1 = adain(sub(n, "norm1"), cin);
    b.n2 = adain(sub(n, "norm2"), cout);
    b.c1 = conv(sub(n, "conv1"), cout, cin, 3, 1, 1, 1, true);
    b.c2 = conv(sub(n, "conv2"), cout, cout, 3, 1, 1, 1, true);
    if (b.sc) b.c1x1 = conv(sub(n, "conv1x1"), cout, cin, 1, 1, 0, 1, false);
    if (up) {
        b.pool_w = add(sub(n, "pool.weight"), 3, cin, 1, 3, true);
        b.pool_b = add(sub(n, "pool.bias"), 1, cin, 1, 1, true);
    }
    return b;
}

// AdaINResBlock1 weights, kokoro_modules.cpp:1147-1195: convs1 dilated with
// padding (k*d - d)/2, convs2 dilation 1, adain1/adain2 fc, alpha1/alpha2 (1, C, 1).
RB1P Layout::rb1(const std::string& n, int C, int k, const int* dil) {
    RB1P r;
    r.C = C; r.k = k;
    for (int i = 0; i < 3; ++i) r.dil[i] = dil[i];
    for (int i = 0; i < 3; ++i)
        r.c1[i] = conv(sub(n, "convs1." + std::to_string(i)), C, C, k, 1, (k * dil[i] - dil[i]) / 2, dil[i], true);
    for (int i = 0; i < 3; ++i) r.c2[i] = conv(sub(n, "convs2." + std::to_string(i)), C, C, k, 1, (k - 1) / 2, 1, true);
    for (int i = 0; i < 3; ++i) r.a1[i] = adain(sub(n, "adain1." + std::to_string(i)), C);
    for (int i = 0; i < 3; ++i) r.a2[i] = adain(sub(n, "adain2." + std::to_string(i)), C);
    for (int i = 0; i < 3; ++i) r.al1[i] = add(sub(n, "alpha1." + std::to_string(i)), 3, 1, C, 1, true);
    for (int i = 0; i < 3; ++i) r.al2[i] = add(sub(n, "alpha2." + std::to_string(i)), 3, 1, C, 1, true);
    return r;
}

void validate_config(const bsml_decoder_config& c) {
    auto bad = [](const char* why) { fail("bsml_decoder_create", why); };
    if (c.asr_dim <= 0 || c.style_dim <= 0 || c.asr_res_dim <= 0 || c.enc_dim <= 0) bad("non-positive channel count");
    if (c.n_decode < 1 || c.n_decode > 8) bad("n_decode must be in [1, 8]");
    if (c.upsample_block >= c.n_decode) bad("upsample_block out of range");
    if (c.n_ups < 1 || c.n_ups > 4) bad("n_ups must be in [1, 4]");
    if (c.n_kernels < 1 || c.n_kernels > 4) bad("n_kernels must be in [1, 4]");
    if (c.n_fft < 2 || c.n_fft > 64 || (c.n_fft & 1)) bad("n_fft must be even and <= 64");
    if (c.hop < 1) bad("hop must be positive");
    if (c.init_ch >> c.n_ups < 1) bad("init_ch too small for n_ups halvings");
    if (c.dec_out[c.n_decode - 1] != c.init_ch) bad("last decode block must output init_ch channels");
    for (int i = 0; i < c.n_ups; ++i) {
        if (c.ups_rate[i] < 1 || c.ups_kernel[i] < c.ups_rate[i]) bad("bad upsample rate/kernel");
        if (c.noise_kernel[i] < 1 || c.noise_stride[i] < 1 || c.noise_pad[i] < 0) bad("bad noise conv");
        if (c.nr_kernel[i] < 1 || !(c.nr_kernel[i] & 1)) bad("noise_res kernels must be odd");
    }
    for (int j = 0; j < c.n_kernels; ++j)
        if (c.rb_kernel[j] < 1 || !(c.rb_kernel[j] & 1)) bad("resblock kernels must be odd");
    if (c.post_kernel < 1 || !(c.post_kernel & 1)) bad("post_kernel must be odd");
}

Layout::Layout(const bsml_decoder_config& c) : cfg(c) {
    validate_config(c);
    F0c = conv("F0_conv", 1, 1, 3, 2, 1, 1, true);
    Nc = conv("N_conv", 1, 1, 3, 2, 1, 1, true);
    asr_res = conv("asr_res.0", cfg.asr_res_dim, cfg.asr_dim, 1, 1, 0, 1, true);
    enc = blk("encode", cfg.asr_dim + 2, cfg.enc_dim, false);
    int x_ch = cfg.enc_dim;
    bool res = true;
    for (int i = 0; i < cfg.n_decode; ++i) {
        const int cin = res ? x_ch + cfg.asr_res_dim + 2 : x_ch;
        const bool up = (i == cfg.upsample_block);
        dec.push_back(blk("decode." + std::to_string(i), cin, cfg.dec_out[i], up));
        x_ch = cfg.dec_out[i];
        if (up) res = false;
    }
    llin_w = add("generator.m_source.l_linear.weight", 2, 1, cfg.harmonic_num + 1, 1, false);
    llin_b = add("generator.m_source.l_linear.bias", 1, 1, 1, 1, false);
    for (int i = 0; i < cfg.n_ups; ++i) {
        UpP u;
        u.cin = cfg.init_ch >> i;
        u.cout = cfg.init_ch >> (i + 1);
        u.k = cfg.ups_kernel[i];
        u.s = cfg.ups_rate[i];
        u.p = (u.k - u.s) / 2;   // kokoro_modules.cpp:1266
        u.w = add("generator.ups." + std::to_string(i) + ".weight", 3, u.cin, u.cout, u.k, true);
        u.b = add("generator.ups." + std::to_string(i) + ".bias", 1, u.cout, 1, 1, true);
        ups.push_back(u);
    }
    for (int i = 0; i < cfg.n_ups; ++i)
        noise.push_back(conv("generator.noise_convs." + std::to_string(i), cfg.init_ch >> (i + 1), cfg.har_ch,
                             cfg.noise_kernel[i], cfg.noise_stride[i], cfg.noise_pad[i], 1, true));
    for (int i = 0; i < cfg.n_ups; ++i)
        nres.push_back(rb1("generator.noise_res." + std::to_string(i), cfg.init_ch >> (i + 1), cfg.nr_kernel[i],
                           cfg.nr_dil[i]));
    for (int i = 0; i < cfg.n_ups; ++i)
        for (int j = 0; j < cfg.n_kernels; ++j)
            rbs.push_back(rb1("generator.resblocks." + std::to_string(i * cfg.n_kernels + j), cfg.init_ch >> (i + 1),
                              cfg.rb_kernel[j], cfg.rb_dil[j]));
    post = conv("generator.conv_post", cfg.n_fft + 2, cfg.init_ch >> cfg.n_ups, cfg.post_kernel, 1,
                (cfg.post_kernel - 1) / 2, 1, true);

    finish();
}

void validate_block(const bsml_block_spec& b) {
    auto bad = [](const char* why) { fail("bsml_block_create", why); };
    if (b.kind != BSML_BLOCK_RESBLK1D && b.kind != BSML_BLOCK_RESBLOCK1) bad("unknown block kind");
    if (b.style_dim <= 0 || b.cin <= 0 || b.cout <= 0) bad("non-positive channel count");
    if (b.kind == BSML_BLOCK_RESBLOCK1) {
        if (b.cin != b.cout) bad("an AdaINResBlock1 keeps its channel count (cin == cout)");
        if (b.kernel < 1 || !(b.kernel & 1)) bad("kernel must be odd");
        for (int i = 0; i < 3; ++i)
            if (b.dil[i] < 1) bad("dilations must be positive");
    }
}

// One block on its own: an AdainResBlk1d in `enc`, an AdaINResBlock1 in `rbs[0]`;
// parameter keys relative to the block
Layout::Layout(const bsml_block_spec& b) : block_kind(b.kind) {
    validate_block(b);
    cfg.style_dim = b.style_dim;
    if (b.kind == BSML_BLOCK_RESBLK1D) enc = blk("", b.cin, b.cout, b.upsample != 0);
    else rbs.push_back(rb1("", b.cin, b.kernel, b.dil));
    finish();
}

void Layout::finish() {
    // AdaIN order = DecoderLora::adapters() (decoder_lora.cpp:173-179)
    auto reg = [&](AdaP& a) {
        a.idx = (int)aff_C.size();
        adains.push_back(&a);
        aff_C.push_back(a.C);
        aff_base.push_back(aff_per_clip);
        aff_per_clip += 2 * a.C;
    };
    const bool decoder = block_kind == 0, with_enc = block_kind != BSML_BLOCK_RESBLOCK1;
    if (with_enc) { reg(enc.n1); reg(enc.n2); }
    for (auto& d : dec) { reg(d.n1); reg(d.n2); }
    for (auto& r : nres) { for (auto& a : r.a1) reg(a); for (auto& a : r.a2) reg(a); }
    for (auto& r : rbs) { for (auto& a : r.a1) reg(a); for (auto& a : r.a2) reg(a); }

    auto regc = [&](ConvP& cp) { cp.id = (int)convs.size(); convs.push_back(&cp); };
    if (decoder) { regc(F0c); regc(Nc); regc(asr_res); }
    auto regb = [&](BlkP& b) { regc(b.c1); regc(b.c2); if (b.sc) regc(b.c1x1); };
    if (with_enc) regb(enc);
    for (auto& d : dec) regb(d);
    for (auto& n : noise) regc(n);
    for (auto& r : nres) for (int i = 0; i < 3; ++i) { regc(r.c1[i]); regc(r.c2[i]); }
    for (auto& r : rbs) for (int i = 0; i < 3; ++i) { regc(r.c1[i]); regc(r.c2[i]); }
    if (decoder) regc(post);
    for (size_t i = 0; i < ups.size(); ++i) ups[i].id = (int)i;
}

}  // namespace bsml
