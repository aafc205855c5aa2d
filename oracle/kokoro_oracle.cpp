// CPU oracle for the Kokoro iSTFTNet decoder forward + backward.
//
// TEST INFRASTRUCTURE ONLY. This file restates, in plain C++ loops, the
// composition the reference library performs in
//   src/kokoro_decoder_backward.cpp   (the *_forward_train / *_backward atoms)
//   src/decoder_lora.cpp              (gate, adapters, Adam)
//   src/kokoro_modules.cpp            (inference forwards, harmonic source)
// of wlejon/brosoundml. Only tests/, __graft_entry__.smoke() and bench.py's
// CPU-baseline leg may load it; the product never does.
//
// PARITY STATUS: unpinned by reference artefacts. The reference delegates all
// arithmetic to the un-vendored `brotensor` library (no source, no golden
// vectors, no buildable copy here), so each brotensor op is restated from the
// PyTorch definition the upstream Kokoro model uses (F.conv1d,
// F.conv_transpose1d, F.instance_norm with eps 1e-5 and biased variance,
// torch.istft(center=True, hann periodic), torch.stft(center=True, reflect)).
// The restatement is pinned instead by (1) an independent PyTorch autograd
// model of the same decoder (oracle/torch_decoder.py) and (2) the reference's
// own finite-difference methodology (tests/test_kokoro_decoder_backward.cpp),
// run in float64 through the templated build below.
//
// Layout: NCL, element (b, c, l) at (b*C + c)*L + l — the reference's layout
// (src/kokoro_decoder_backward.h:15-17) with a leading batch axis.
//
// Beyond the reference (which trains only the AdaIN affines), the oracle also
// returns conv/convT weight and bias gradients, Snake alpha gradients, AdaIN
// fc gradients, and input gradients for asr and style; the reference-mode
// per-AdaIN (dGamma, dBeta) outputs are a subset of that.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {

// Architecture description. Field meanings follow the reference loaders:
// DecoderBackbone::load_from (kokoro_modules.cpp:1021-1063),
// Generator::load_from (kokoro_modules.cpp:1237-1347),
// HarmonicSource::load_from (kokoro_modules.cpp:1556-1572).
typedef struct orc_cfg {
    int asr_dim;          // 512  asr channels
    int style_dim;        // 128
    int asr_res_dim;      // 64   asr_res 1x1 projection
    int enc_dim;          // 1024 encode output channels
    int n_decode;         // 4
    int dec_out[8];       // per decode block output channels
    int upsample_block;   // decode block that upsamples 2x (3); blocks after it get no cat
    int n_ups;            // 2
    int init_ch;          // 512 generator input channels
    int ups_rate[4];      // 10, 6
    int ups_kernel[4];    // 20, 12
    int noise_kernel[4];  // 12, 1
    int noise_stride[4];  // 6, 1
    int noise_pad[4];     // 3, 0
    int nr_kernel[4];     // noise_res kernels 7, 11
    int nr_dil[4][3];     // noise_res dilations {1,3,5}
    int n_kernels;        // 3
    int rb_kernel[4];     // 3, 7, 11
    int rb_dil[4][3];     // {1,3,5} each
    int har_ch;           // n_fft + 2 = 22
    int n_fft;            // 20
    int hop;              // 5
    int post_kernel;      // 7
    int harmonic_num;     // 8
    int sample_rate;      // 24000
    int upsample_scale;   // prod(ups_rate) * hop = 300
} orc_cfg;

// One decoder block on its own (the reference's block-level atoms,
// src/kokoro_decoder_backward.h:82-144). kind 1 = AdainResBlk1d (cin, cout,
// upsample), kind 2 = AdaINResBlock1 (C = cin, kernel, dil).
typedef struct orc_block_spec {
    int kind;
    int style_dim;
    int cin, cout;
    int upsample;
    int kernel;
    int dil[3];
} orc_block_spec;

typedef struct orc_param {
    char name[96];
    int64_t offset;
    int64_t numel;
    int ndim;
    int shape[3];
    int trainable;
} orc_param;

}  // extern "C"

namespace orc {

// ─── parameter layout ───────────────────────────────────────────────────────

struct Conv { int64_t w = -1, b = -1; int cout = 0, cin = 0, k = 0, s = 1, p = 0, d = 1; };
struct AdaIN { int64_t fw = -1, fb = -1; int C = 0; int idx = 0; };
struct Blk {
    int cin = 0, cout = 0; bool up = false, sc = false;
    AdaIN n1, n2; Conv c1, c2, c1x1; int64_t pool_w = -1, pool_b = -1;
};
struct RB1 {
    int C = 0, k = 0; int dil[3] = {1, 1, 1};
    Conv c1[3], c2[3]; AdaIN a1[3], a2[3]; int64_t al1[3], al2[3];
};
struct Up { int64_t w = -1, b = -1; int cin = 0, cout = 0, k = 0, s = 1, p = 0; };

// "a.b" module-key join; an empty prefix gives the block-relative key
inline std::string sub(const std::string& n, const std::string& s) { return n.empty() ? s : n + "." + s; }

struct Layout {
    orc_cfg cfg;
    int kind = 0;   // 0 = full decoder, else orc_block_spec::kind
    std::vector<orc_param> table;
    int64_t total = 0;
    Conv F0c, Nc, asr_res;
    Blk enc;
    std::vector<Blk> dec;
    int64_t llin_w = -1, llin_b = -1;
    std::vector<Up> ups;
    std::vector<Conv> noise;
    std::vector<RB1> nres, rbs;
    Conv post;
    std::vector<int> aff_C;          // per AdaIN channel count, adapter order
    std::vector<int64_t> aff_base;   // per AdaIN: sum_{a'<a} 2*C_a' (per clip units)
    int64_t aff_per_clip = 0;

    int64_t add(const std::string& name, int nd, int s0, int s1, int s2, bool train) {
        orc_param p{};
        std::snprintf(p.name, sizeof(p.name), "%s", name.c_str());
        p.ndim = nd; p.shape[0] = s0; p.shape[1] = s1; p.shape[2] = s2;
        p.numel = (int64_t)s0 * (nd > 1 ? s1 : 1) * (nd > 2 ? s2 : 1);
        p.trainable = train ? 1 : 0;
        p.offset = total;
        total += (p.numel + 63) / 64 * 64;   // 256-byte aligned slots
        table.push_back(p);
        return p.offset;
    }
    Conv conv(const std::string& n, int cout, int cin, int k, int s, int p, int d, bool bias) {
        Conv c; c.cout = cout; c.cin = cin; c.k = k; c.s = s; c.p = p; c.d = d;
        c.w = add(n + ".weight", 3, cout, cin, k, true);
        if (bias) c.b = add(n + ".bias", 1, cout, 1, 1, true);
        return c;
    }
    AdaIN adain(const std::string& n, int C) {
        AdaIN a; a.C = C;
        a.fw = add(n + ".fc.weight", 2, 2 * C, cfg.style_dim, 1, true);
        a.fb = add(n + ".fc.bias", 1, 2 * C, 1, 1, true);
        return a;
    }
    Blk blk(const std::string& n, int cin, int cout, bool up) {
        Blk b; b.cin = cin; b.cout = cout; b.up = up; b.sc = cin != cout;
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
    RB1 rb1(const std::string& n, int C, int k, const int* dil) {
        RB1 r; r.C = C; r.k = k;
        for (int i = 0; i < 3; ++i) r.dil[i] = dil[i];
        for (int i = 0; i < 3; ++i)   // get_padding(k, d) = (k*d - d)/2, kokoro_modules.cpp:1155-1157
            r.c1[i] = conv(sub(n, "convs1." + std::to_string(i)), C, C, k, 1, (k * dil[i] - dil[i]) / 2, dil[i], true);
        for (int i = 0; i < 3; ++i)
            r.c2[i] = conv(sub(n, "convs2." + std::to_string(i)), C, C, k, 1, (k - 1) / 2, 1, true);
        for (int i = 0; i < 3; ++i) r.a1[i] = adain(sub(n, "adain1." + std::to_string(i)), C);
        for (int i = 0; i < 3; ++i) r.a2[i] = adain(sub(n, "adain2." + std::to_string(i)), C);
        for (int i = 0; i < 3; ++i) r.al1[i] = add(sub(n, "alpha1." + std::to_string(i)), 3, 1, C, 1, true);
        for (int i = 0; i < 3; ++i) r.al2[i] = add(sub(n, "alpha2." + std::to_string(i)), 3, 1, C, 1, true);
        return r;
    }

    explicit Layout(const orc_cfg& c) : cfg(c) {
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
            Up u; u.cin = cfg.init_ch >> i; u.cout = cfg.init_ch >> (i + 1);
            u.k = cfg.ups_kernel[i]; u.s = cfg.ups_rate[i]; u.p = (u.k - u.s) / 2;
            u.w = add("generator.ups." + std::to_string(i) + ".weight", 3, u.cin, u.cout, u.k, true);
            u.b = add("generator.ups." + std::to_string(i) + ".bias", 1, u.cout, 1, 1, true);
            ups.push_back(u);
        }
        for (int i = 0; i < cfg.n_ups; ++i)
            noise.push_back(conv("generator.noise_convs." + std::to_string(i), cfg.init_ch >> (i + 1),
                                 cfg.har_ch, cfg.noise_kernel[i], cfg.noise_stride[i], cfg.noise_pad[i], 1, true));
        for (int i = 0; i < cfg.n_ups; ++i)
            nres.push_back(rb1("generator.noise_res." + std::to_string(i), cfg.init_ch >> (i + 1),
                               cfg.nr_kernel[i], cfg.nr_dil[i]));
        for (int i = 0; i < cfg.n_ups; ++i)
            for (int j = 0; j < cfg.n_kernels; ++j)
                rbs.push_back(rb1("generator.resblocks." + std::to_string(i * cfg.n_kernels + j),
                                  cfg.init_ch >> (i + 1), cfg.rb_kernel[j], cfg.rb_dil[j]));
        post = conv("generator.conv_post", cfg.n_fft + 2, cfg.init_ch >> cfg.n_ups, cfg.post_kernel, 1,
                    (cfg.post_kernel - 1) / 2, 1, true);
        register_adains();
    }

    // a single block: AdainResBlk1d held in `enc`, AdaINResBlock1 in `rbs[0]`;
    // keys are block-relative ("norm1.fc.weight", "convs1.0.weight", ...)
    explicit Layout(const orc_block_spec& b) : cfg{}, kind(b.kind) {
        cfg.style_dim = b.style_dim;
        if (kind == 1) enc = blk("", b.cin, b.cout, b.upsample != 0);
        else rbs.push_back(rb1("", b.cin, b.kernel, b.dil));
        register_adains();
    }

    // AdaIN order = DecoderLora::adapters() order (decoder_lora.cpp:173-179).
    void register_adains() {
        auto reg = [&](AdaIN& a) {
            a.idx = (int)aff_C.size(); aff_C.push_back(a.C); aff_base.push_back(aff_per_clip);
            aff_per_clip += 2 * a.C;
        };
        if (kind != 2) { reg(enc.n1); reg(enc.n2); }
        for (auto& d : dec) { reg(d.n1); reg(d.n2); }
        for (auto& r : nres) { for (auto& a : r.a1) reg(a); for (auto& a : r.a2) reg(a); }
        for (auto& r : rbs) { for (auto& a : r.a1) reg(a); for (auto& a : r.a2) reg(a); }
    }
};

// ─── primitive ops (templated: float for parity, double for FD checks) ─────

template <class R> using Vec = std::vector<R>;

inline int conv_out_len(int L, int k, int s, int p, int d) { return (L + 2 * p - d * (k - 1) - 1) / s + 1; }

// F.conv1d semantics: y[b,co,o] = bias[co] + sum_{ci,t} W[co,ci,t] x[b,ci,o*s+t*d-p].
template <class R>
void conv_fwd(const R* x, int B, int Ci, int L, const R* W, const R* bias, int Co, int k, int s, int p, int d,
              R* y, int Lo) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
        for (int co = 0; co < Co; ++co) {
            R* yr = y + ((int64_t)b * Co + co) * Lo;
            const R bv = bias ? bias[co] : R(0);
            for (int o = 0; o < Lo; ++o) yr[o] = bv;
            for (int ci = 0; ci < Ci; ++ci) {
                const R* xr = x + ((int64_t)b * Ci + ci) * L;
                for (int t = 0; t < k; ++t) {
                    const R w = W[((int64_t)co * Ci + ci) * k + t];
                    const int off = t * d - p;
                    // o range with 0 <= o*s + off < L
                    int o0 = off >= 0 ? 0 : (-off + s - 1) / s;
                    int o1 = (L - 1 - off) >= 0 ? (L - 1 - off) / s + 1 : 0;
                    o1 = std::min(o1, Lo);
                    if (s == 1) {
                        const R* xs = xr + off;
                        for (int o = o0; o < o1; ++o) yr[o] += w * xs[o];
                    } else {
                        for (int o = o0; o < o1; ++o) yr[o] += w * xr[o * s + off];
                    }
                }
            }
        }
}

// Adjoint of conv_fwd w.r.t. x (conv1d_backward_input).
template <class R>
void conv_dgrad(const R* dy, int B, int Ci, int L, const R* W, int Co, int k, int s, int p, int d, R* dx, int Lo) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
        for (int ci = 0; ci < Ci; ++ci) {
            R* dr = dx + ((int64_t)b * Ci + ci) * L;
            for (int j = 0; j < L; ++j) dr[j] = R(0);
            for (int co = 0; co < Co; ++co) {
                const R* gr = dy + ((int64_t)b * Co + co) * Lo;
                for (int t = 0; t < k; ++t) {
                    const R w = W[((int64_t)co * Ci + ci) * k + t];
                    const int off = t * d - p;
                    int o0 = off >= 0 ? 0 : (-off + s - 1) / s;
                    int o1 = (L - 1 - off) >= 0 ? (L - 1 - off) / s + 1 : 0;
                    o1 = std::min(o1, Lo);
                    for (int o = o0; o < o1; ++o) dr[o * s + off] += w * gr[o];
                }
            }
        }
}

// Weight / bias gradient of conv_fwd (accumulates; double accumulators).
template <class R>
void conv_wgrad(const R* dy, const R* x, int B, int Ci, int L, int Co, int k, int s, int p, int d, int Lo,
                R* dW, R* db) {
#pragma omp parallel for schedule(dynamic)
    for (int co = 0; co < Co; ++co) {
        if (db) {
            double acc = 0;
            for (int b = 0; b < B; ++b) {
                const R* gr = dy + ((int64_t)b * Co + co) * Lo;
                for (int o = 0; o < Lo; ++o) acc += gr[o];
            }
            db[co] += (R)acc;
        }
        for (int ci = 0; ci < Ci; ++ci)
            for (int t = 0; t < k; ++t) {
                const int off = t * d - p;
                int o0 = off >= 0 ? 0 : (-off + s - 1) / s;
                int o1 = (L - 1 - off) >= 0 ? (L - 1 - off) / s + 1 : 0;
                o1 = std::min(o1, Lo);
                double acc = 0;
                for (int b = 0; b < B; ++b) {
                    const R* gr = dy + ((int64_t)b * Co + co) * Lo;
                    const R* xr = x + ((int64_t)b * Ci + ci) * L;
                    R part = 0;
                    for (int o = o0; o < o1; ++o) part += gr[o] * xr[o * s + off];
                    acc += part;
                }
                dW[((int64_t)co * Ci + ci) * k + t] += (R)acc;
            }
    }
}

// F.conv_transpose1d semantics, groups = 1, weight (Ci, Co, k):
//   y[b,co,j] = bias[co] + sum_{ci,l,t : j = l*s - p + t} W[ci,co,t] x[b,ci,l]
template <class R>
void convT_fwd(const R* x, int B, int Ci, int L, const R* W, const R* bias, int Co, int k, int s, int p, R* y,
               int Lo) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
        for (int co = 0; co < Co; ++co) {
            R* yr = y + ((int64_t)b * Co + co) * Lo;
            const R bv = bias ? bias[co] : R(0);
            for (int j = 0; j < Lo; ++j) yr[j] = bv;
            for (int ci = 0; ci < Ci; ++ci) {
                const R* xr = x + ((int64_t)b * Ci + ci) * L;
                for (int t = 0; t < k; ++t) {
                    const R w = W[((int64_t)ci * Co + co) * k + t];
                    for (int l = 0; l < L; ++l) {
                        const int j = l * s - p + t;
                        if (j >= 0 && j < Lo) yr[j] += w * xr[l];
                    }
                }
            }
        }
}

template <class R>
void convT_dgrad(const R* dy, int B, int Ci, int L, const R* W, int Co, int k, int s, int p, R* dx, int Lo) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
        for (int ci = 0; ci < Ci; ++ci) {
            R* dr = dx + ((int64_t)b * Ci + ci) * L;
            for (int l = 0; l < L; ++l) dr[l] = R(0);
            for (int co = 0; co < Co; ++co) {
                const R* gr = dy + ((int64_t)b * Co + co) * Lo;
                for (int t = 0; t < k; ++t) {
                    const R w = W[((int64_t)ci * Co + co) * k + t];
                    for (int l = 0; l < L; ++l) {
                        const int j = l * s - p + t;
                        if (j >= 0 && j < Lo) dr[l] += w * gr[j];
                    }
                }
            }
        }
}

template <class R>
void convT_wgrad(const R* dy, const R* x, int B, int Ci, int L, int Co, int k, int s, int p, int Lo, R* dW, R* db) {
    if (db) {
#pragma omp parallel for schedule(static)
        for (int co = 0; co < Co; ++co) {
            double acc = 0;
            for (int b = 0; b < B; ++b)
                for (int j = 0; j < Lo; ++j) acc += dy[((int64_t)b * Co + co) * Lo + j];
            db[co] += (R)acc;
        }
    }
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int ci = 0; ci < Ci; ++ci)
        for (int co = 0; co < Co; ++co)
            for (int t = 0; t < k; ++t) {
                double acc = 0;
                for (int b = 0; b < B; ++b) {
                    const R* xr = x + ((int64_t)b * Ci + ci) * L;
                    const R* gr = dy + ((int64_t)b * Co + co) * Lo;
                    R part = 0;
                    for (int l = 0; l < L; ++l) {
                        const int j = l * s - p + t;
                        if (j >= 0 && j < Lo) part += xr[l] * gr[j];
                    }
                    acc += part;
                }
                dW[((int64_t)ci * Co + co) * k + t] += (R)acc;
            }
}

// Depthwise ConvTranspose1d (groups = C), weight (C, 1, k): the AdainResBlk1d
// upsampling pool, kokoro_decoder_backward.cpp:176-180 (k3 s2 p1 op1).
template <class R>
void dwconvT_fwd(const R* x, int B, int C, int L, const R* W, const R* bias, int k, int s, int p, R* y, int Lo) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c) {
            R* yr = y + ((int64_t)b * C + c) * Lo;
            const R* xr = x + ((int64_t)b * C + c) * L;
            for (int j = 0; j < Lo; ++j) yr[j] = bias ? bias[c] : R(0);
            for (int t = 0; t < k; ++t)
                for (int l = 0; l < L; ++l) {
                    const int j = l * s - p + t;
                    if (j >= 0 && j < Lo) yr[j] += W[c * k + t] * xr[l];
                }
        }
}
template <class R>
void dwconvT_dgrad(const R* dy, int B, int C, int L, const R* W, int k, int s, int p, R* dx, int Lo) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int b = 0; b < B; ++b)
        for (int c = 0; c < C; ++c) {
            R* dr = dx + ((int64_t)b * C + c) * L;
            const R* gr = dy + ((int64_t)b * C + c) * Lo;
            for (int l = 0; l < L; ++l) {
                R acc = 0;
                for (int t = 0; t < k; ++t) {
                    const int j = l * s - p + t;
                    if (j >= 0 && j < Lo) acc += W[c * k + t] * gr[j];
                }
                dr[l] = acc;
            }
        }
}
template <class R>
void dwconvT_wgrad(const R* dy, const R* x, int B, int C, int L, int k, int s, int p, int Lo, R* dW, R* db) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < C; ++c) {
        double accb = 0;
        for (int b = 0; b < B; ++b)
            for (int j = 0; j < Lo; ++j) accb += dy[((int64_t)b * C + c) * Lo + j];
        if (db) db[c] += (R)accb;
        for (int t = 0; t < k; ++t) {
            double acc = 0;
            for (int b = 0; b < B; ++b) {
                const R* xr = x + ((int64_t)b * C + c) * L;
                const R* gr = dy + ((int64_t)b * C + c) * Lo;
                for (int l = 0; l < L; ++l) {
                    const int j = l * s - p + t;
                    if (j >= 0 && j < Lo) acc += (double)xr[l] * gr[j];
                }
            }
            dW[c * k + t] += (R)acc;
        }
    }
}

template <class R>
void leaky_fwd(const R* x, int64_t n, R slope, R* y) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) y[i] = x[i] > R(0) ? x[i] : slope * x[i];
}
template <class R>
void leaky_bwd(const R* x, const R* dy, int64_t n, R slope, R* dx) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) dx[i] = x[i] > R(0) ? dy[i] : slope * dy[i];
}

// Instance norm (GroupNorm with num_groups = C), biased variance, statistics in
// double. mean/rstd are (B, C).
template <class R>
void in_stats(const R* x, int B, int C, int L, R eps, R* mean, R* rstd) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)B * C; ++r) {
        const R* xr = x + r * L;
        double s = 0;
        for (int l = 0; l < L; ++l) s += xr[l];
        const double m = s / L;
        double v = 0;
        for (int l = 0; l < L; ++l) { const double dd = xr[l] - m; v += dd * dd; }
        v /= L;
        mean[r] = (R)m;
        rstd[r] = (R)(1.0 / std::sqrt(v + (double)eps));
    }
}

// AdaIN affine (kokoro_decoder_backward.cpp:100-120):
//   y = (1 + gamma) * (x - mean) * rstd + beta, gamma/beta per clip: gb[b][0:C] / gb[b][C:2C].
template <class R>
void adain_fwd(const R* x, int B, int C, int L, const R* gb, int64_t gb_stride, const R* mean, const R* rstd, R* y) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)B * C; ++r) {
        const int b = (int)(r / C), c = (int)(r % C);
        const R g1 = R(1) + gb[b * gb_stride + c], be = gb[b * gb_stride + C + c];
        const R m = mean[r], rs = rstd[r];
        const R* xr = x + r * L; R* yr = y + r * L;
        for (int l = 0; l < L; ++l) yr[l] = g1 * ((xr[l] - m) * rs) + be;
    }
}

// Backward of adain_fwd (modulate_backward + group_norm_backward,
// kokoro_decoder_backward.cpp:41-61, 122-150). dgb (dGamma, dBeta) overwritten.
template <class R>
void adain_bwd(const R* x, int B, int C, int L, const R* gb, int64_t gb_stride, const R* mean, const R* rstd,
               const R* dy, R* dx, R* dgb) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)B * C; ++r) {
        const int b = (int)(r / C), c = (int)(r % C);
        const R g1 = R(1) + gb[b * gb_stride + c];
        const R m = mean[r], rs = rstd[r];
        const R* xr = x + r * L; const R* gr = dy + r * L; R* dr = dx + r * L;
        double sg = 0, sgx = 0;
        for (int l = 0; l < L; ++l) { const double xh = (double)((xr[l] - m) * rs); sg += gr[l]; sgx += gr[l] * xh; }
        dgb[b * gb_stride + c] = (R)sgx;
        dgb[b * gb_stride + C + c] = (R)sg;
        // dxhat = g1*dy ; dx = rstd*(dxhat - mean(dxhat) - xhat*mean(dxhat*xhat))
        const R mdh = (R)(g1 * sg / L), mdhx = (R)(g1 * sgx / L);
        for (int l = 0; l < L; ++l) {
            const R xh = (xr[l] - m) * rs;
            dr[l] = rs * (g1 * gr[l] - mdh - xh * mdhx);
        }
    }
}

// Snake1D: y = x + sin(alpha x)^2 / alpha (kokoro_modules.h:253).
template <class R>
void snake_fwd(const R* x, int B, int C, int L, const R* alpha, R* y) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)B * C; ++r) {
        const R a = alpha[r % C];
        const R* xr = x + r * L; R* yr = y + r * L;
        for (int l = 0; l < L; ++l) { const R sn = std::sin(a * xr[l]); yr[l] = xr[l] + sn * sn / a; }
    }
}
// dx = dy * (1 + sin(2 a x)); dalpha += sum dy * (x sin(2ax)/a - sin(ax)^2/a^2)
template <class R>
void snake_bwd(const R* x, int B, int C, int L, const R* alpha, const R* dy, R* dx, R* dalpha) {
    std::vector<double> da((size_t)B * C, 0.0);
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)B * C; ++r) {
        const R a = alpha[r % C];
        const R* xr = x + r * L; const R* gr = dy + r * L; R* dr = dx + r * L;
        double acc = 0;
        for (int l = 0; l < L; ++l) {
            const R sn = std::sin(a * xr[l]), s2 = std::sin(R(2) * a * xr[l]);
            dr[l] = gr[l] * (R(1) + s2);
            acc += (double)gr[l] * (double)(xr[l] * s2 / a - sn * sn / (a * a));
        }
        da[r] = acc;
    }
    if (dalpha)
        for (int c = 0; c < C; ++c) {
            double s = 0;
            for (int b = 0; b < B; ++b) s += da[(size_t)b * C + c];
            dalpha[c] += (R)s;
        }
}

inline double two_pi() { return 6.28318530717958647692; }

// Periodic Hann window, kokoro_decoder_backward.cpp:581-588 (float arithmetic).
template <class R>
Vec<R> hann(int N) {
    Vec<R> w(N);
    constexpr float kTwoPi = 6.28318530717958647692f;
    for (int n = 0; n < N; ++n) w[n] = (R)(0.5f - 0.5f * std::cos(kTwoPi * (float)n / (float)N));
    return w;
}

// torch.istft(center=True, normalized=False, onesided, window=hann(n_fft),
// length omitted -> hop*(frames-1)). re/im: (B, n_freq, L) channel-major.
// audio: (B, hop*(L-1)).
template <class R>
void istft_fwd(const R* re, const R* im, int B, int n_fft, int hop, int L, const R* win, R* audio) {
    const int nf = n_fft / 2 + 1;
    const int S = hop * (L - 1);
    const int full = n_fft + hop * (L - 1);
    const int pad = n_fft / 2;
    // basis: frame[m] = sum_k c_k/N (Re_k cos(2pi k m/N) - Im_k sin(2pi k m/N))
    Vec<double> cb((size_t)nf * n_fft), sb((size_t)nf * n_fft);
    for (int k = 0; k < nf; ++k)
        for (int m = 0; m < n_fft; ++m) {
            const double ck = (k == 0 || 2 * k == n_fft) ? 1.0 : 2.0;
            const double ang = two_pi() * (double)k * (double)m / (double)n_fft;
            cb[(size_t)k * n_fft + m] = ck / n_fft * std::cos(ang);
            sb[(size_t)k * n_fft + m] = -ck / n_fft * std::sin(ang);
        }
    Vec<double> env(full, 0.0);
    for (int t = 0; t < L; ++t)
        for (int m = 0; m < n_fft; ++m) env[t * hop + m] += (double)win[m] * win[m];
#pragma omp parallel for schedule(static)
    for (int b = 0; b < B; ++b) {
        Vec<double> y(full, 0.0);
        for (int t = 0; t < L; ++t)
            for (int m = 0; m < n_fft; ++m) {
                double v = 0;
                for (int k = 0; k < nf; ++k) {
                    const int64_t ix = ((int64_t)b * nf + k) * L + t;
                    v += re[ix] * cb[(size_t)k * n_fft + m] + im[ix] * sb[(size_t)k * n_fft + m];
                }
                y[t * hop + m] += v * win[m];
            }
        for (int n = 0; n < S; ++n) audio[(int64_t)b * S + n] = (R)(y[n + pad] / env[n + pad]);
    }
}

template <class R>
void istft_bwd(const R* daudio, int B, int n_fft, int hop, int L, const R* win, R* dre, R* dim) {
    const int nf = n_fft / 2 + 1;
    const int S = hop * (L - 1);
    const int full = n_fft + hop * (L - 1);
    const int pad = n_fft / 2;
    Vec<double> cb((size_t)nf * n_fft), sb((size_t)nf * n_fft);
    for (int k = 0; k < nf; ++k)
        for (int m = 0; m < n_fft; ++m) {
            const double ck = (k == 0 || 2 * k == n_fft) ? 1.0 : 2.0;
            const double ang = two_pi() * (double)k * (double)m / (double)n_fft;
            cb[(size_t)k * n_fft + m] = ck / n_fft * std::cos(ang);
            sb[(size_t)k * n_fft + m] = -ck / n_fft * std::sin(ang);
        }
    Vec<double> env(full, 0.0);
    for (int t = 0; t < L; ++t)
        for (int m = 0; m < n_fft; ++m) env[t * hop + m] += (double)win[m] * win[m];
#pragma omp parallel for schedule(static)
    for (int b = 0; b < B; ++b) {
        Vec<double> g(full, 0.0);
        for (int n = 0; n < S; ++n) g[n + pad] = daudio[(int64_t)b * S + n] / env[n + pad];
        for (int t = 0; t < L; ++t)
            for (int k = 0; k < nf; ++k) {
                double ar = 0, ai = 0;
                for (int m = 0; m < n_fft; ++m) {
                    const double gw = g[t * hop + m] * win[m];
                    ar += gw * cb[(size_t)k * n_fft + m];
                    ai += gw * sb[(size_t)k * n_fft + m];
                }
                const int64_t ix = ((int64_t)b * nf + k) * L + t;
                dre[ix] = (R)ar;
                dim[ix] = (R)ai;
            }
    }
}

// Harmonic source, kokoro_modules.cpp:1574-1665: per-sample fp32 phase
// accumulator (reference arithmetic, single wrap), l_linear + tanh, then
// torch.stft(center=True, reflect pad n_fft/2, hann) -> [|X| ; angle X].
// F0: (B, F) frames. har: (B, 2*nf, S/hop + 1).
template <class R>
void harmonic_source(const R* F0, int B, int F, const R* lw, const R* lb, const orc_cfg& cfg, R* har) {
    const int dim = cfg.harmonic_num + 1;
    const int S = F * cfg.upsample_scale;
    const int n_fft = cfg.n_fft, hop = cfg.hop, nf = n_fft / 2 + 1;
    const int frames = S / hop + 1;
    const float sr_f = (float)cfg.sample_rate;
    const float kTwoPi = 6.28318530717958647692f;
    const Vec<R> win = hann<R>(n_fft);
#pragma omp parallel for schedule(static)
    for (int b = 0; b < B; ++b) {
        std::vector<float> phases(dim, 0.0f);
        Vec<R> src(S);
        for (int t = 0; t < S; ++t) {
            const int frame = t / cfg.upsample_scale;
            const float f0 = (float)F0[(int64_t)b * F + std::min(frame, F - 1)];
            const float uv = f0 > 0.0f ? 1.0f : 0.0f;
            double merged = (double)lb[0];
            float mf = 0.0f;
            for (int h = 0; h < dim; ++h) {
                const float omega = kTwoPi * (float)(h + 1) * f0 / sr_f;
                phases[h] += omega;
                if (phases[h] > kTwoPi) phases[h] -= kTwoPi;
                const float sw = std::sin(phases[h]) * 0.1f * uv;
                mf += (float)lw[h] * sw;
            }
            merged += mf;
            src[t] = (R)std::tanh(merged);
        }
        const int pad = n_fft / 2;
        auto xp = [&](int i) -> R {   // reflect padding
            int j = i - pad;
            if (j < 0) j = -j;
            if (j >= S) j = 2 * (S - 1) - j;
            return src[j];
        };
        for (int t = 0; t < frames; ++t)
            for (int k = 0; k < nf; ++k) {
                double xr = 0, xi = 0;
                for (int m = 0; m < n_fft; ++m) {
                    const double v = (double)win[m] * xp(t * hop + m);
                    const double ang = two_pi() * (double)k * (double)m / (double)n_fft;
                    xr += v * std::cos(ang);
                    xi -= v * std::sin(ang);
                }
                har[((int64_t)b * 2 * nf + k) * frames + t] = (R)std::sqrt(xr * xr + xi * xi);
                har[((int64_t)b * 2 * nf + nf + k) * frames + t] = (R)std::atan2(xi, xr);
            }
    }
}

// ─── the decoder ────────────────────────────────────────────────────────────

template <class R>
struct Decoder {
    const Layout& lay;
    const R* P;      // params
    R* G;            // param grads (may be null)
    int B, T;
    R eps = R(1e-5);
    const R* aff_in = nullptr;   // reference mode: (gamma, beta) per AdaIN, else fc(style)
    Vec<R> aff;                  // resolved (gamma, beta): [n_aff][B][2C]
    Vec<R> daff;                 // grads of the above
    const R* style = nullptr;

    Decoder(const Layout& l, const R* p, R* g, int b, int t) : lay(l), P(p), G(g), B(b), T(t) {}

    const R* aff_ptr(const AdaIN& a) const { return aff.data() + (int64_t)B * lay.aff_base[a.idx]; }
    R* daff_ptr(const AdaIN& a) { return daff.data() + (int64_t)B * lay.aff_base[a.idx]; }
    R* g(int64_t off) { return (G && off >= 0) ? G + off : nullptr; }

    // ── AdaIN fc: (gamma, beta)_b = W style_b + bias (compute_style_affine, kokoro_modules.cpp:563-572)
    void resolve_affines() {
        aff.assign((size_t)B * lay.aff_per_clip, R(0));
        daff.assign(aff.size(), R(0));
        auto one = [&](const AdaIN& a) {
            R* out = aff.data() + (int64_t)B * lay.aff_base[a.idx];
            const int n2 = 2 * a.C, S = lay.cfg.style_dim;
            if (aff_in) {
                std::memcpy(out, aff_in + (int64_t)B * lay.aff_base[a.idx], sizeof(R) * (size_t)B * n2);
                return;
            }
            for (int b = 0; b < B; ++b)
                for (int o = 0; o < n2; ++o) {
                    double acc = P[a.fb + o];
                    for (int i = 0; i < S; ++i) acc += (double)P[a.fw + (int64_t)o * S + i] * style[b * S + i];
                    out[b * n2 + o] = (R)acc;
                }
        };
        for_each_adain(one);
    }
    template <class F> void for_each_adain(F f) {
        if (lay.kind != 2) { f(lay.enc.n1); f(lay.enc.n2); }
        for (auto& d : lay.dec) { f(d.n1); f(d.n2); }
        for (auto& r : lay.nres) { for (auto& a : r.a1) f(a); for (auto& a : r.a2) f(a); }
        for (auto& r : lay.rbs) { for (auto& a : r.a1) f(a); for (auto& a : r.a2) f(a); }
    }
    void affine_backward(R* d_style) {
        if (aff_in) return;
        const int S = lay.cfg.style_dim;
        for_each_adain([&](const AdaIN& a) {
            const R* d = daff.data() + (int64_t)B * lay.aff_base[a.idx];
            const int n2 = 2 * a.C;
            if (G) {
                for (int o = 0; o < n2; ++o) {
                    double sb = 0;
                    for (int b = 0; b < B; ++b) sb += d[b * n2 + o];
                    G[a.fb + o] += (R)sb;
                    for (int i = 0; i < S; ++i) {
                        double acc = 0;
                        for (int b = 0; b < B; ++b) acc += (double)d[b * n2 + o] * style[b * S + i];
                        G[a.fw + (int64_t)o * S + i] += (R)acc;
                    }
                }
            }
            if (d_style)
                for (int b = 0; b < B; ++b)
                    for (int i = 0; i < S; ++i) {
                        double acc = 0;
                        for (int o = 0; o < n2; ++o) acc += (double)P[a.fw + (int64_t)o * S + i] * d[b * n2 + o];
                        d_style[b * S + i] += (R)acc;
                    }
        });
    }

    // ── conv helpers on Conv descriptors
    int out_len(const Conv& c, int L) const { return conv_out_len(L, c.k, c.s, c.p, c.d); }
    void cfwd(const Conv& c, const R* x, int L, R* y) {
        conv_fwd(x, B, c.cin, L, P + c.w, c.b >= 0 ? P + c.b : (const R*)nullptr, c.cout, c.k, c.s, c.p, c.d, y,
                 out_len(c, L));
    }
    void cbwd(const Conv& c, const R* x, int L, const R* dy, R* dx) {
        const int Lo = out_len(c, L);
        if (dx) conv_dgrad(dy, B, c.cin, L, P + c.w, c.cout, c.k, c.s, c.p, c.d, dx, Lo);
        if (G) conv_wgrad(dy, x, B, c.cin, L, c.cout, c.k, c.s, c.p, c.d, Lo, G + c.w, g(c.b));
    }

    // ── AdaIN + cache
    struct AdaCache { Vec<R> x, mean, rstd; };
    void adain_f(const AdaIN& a, const R* x, int C, int L, AdaCache& ac, R* y) {
        const int64_t n = (int64_t)B * C * L;
        ac.x.assign(x, x + n);
        ac.mean.resize((size_t)B * C); ac.rstd.resize((size_t)B * C);
        in_stats(x, B, C, L, eps, ac.mean.data(), ac.rstd.data());
        adain_fwd(x, B, C, L, aff_ptr(a), 2 * C, ac.mean.data(), ac.rstd.data(), y);
    }
    void adain_b(const AdaIN& a, const AdaCache& ac, int C, int L, const R* dy, R* dx) {
        adain_bwd(ac.x.data(), B, C, L, aff_ptr(a), 2 * C, ac.mean.data(), ac.rstd.data(), dy, dx, daff_ptr(a));
    }

    // ── AdainResBlk1d (kokoro_decoder_backward.cpp:152-285)
    struct BlkCache { AdaCache a1, a2; Vec<R> r_pre, pooled_in /*leaky(r_pre)*/, pooled, n2_pre, n2, shortx; int Lin, Lout; };
    void blk_f(const Blk& w, const R* x, int Lin, BlkCache& c, Vec<R>& y) {
        const int Lout = w.up ? 2 * Lin : Lin;
        c.Lin = Lin; c.Lout = Lout;
        const int64_t nin = (int64_t)B * w.cin * Lin, nout = (int64_t)B * w.cout * Lout;
        c.r_pre.resize(nin);
        adain_f(w.n1, x, w.cin, Lin, c.a1, c.r_pre.data());
        c.pooled_in.resize(nin);
        leaky_fwd(c.r_pre.data(), nin, R(0.2), c.pooled_in.data());
        if (w.up) {
            c.pooled.resize((int64_t)B * w.cin * Lout);
            dwconvT_fwd(c.pooled_in.data(), B, w.cin, Lin, P + w.pool_w, P + w.pool_b, 3, 2, 1, c.pooled.data(), Lout);
        } else {
            c.pooled = c.pooled_in;
        }
        Vec<R> c1((size_t)nout);
        cfwd(w.c1, c.pooled.data(), Lout, c1.data());
        c.n2_pre.resize(nout);
        adain_f(w.n2, c1.data(), w.cout, Lout, c.a2, c.n2_pre.data());
        c.n2.resize(nout);
        leaky_fwd(c.n2_pre.data(), nout, R(0.2), c.n2.data());
        y.assign((size_t)nout, R(0));
        cfwd(w.c2, c.n2.data(), Lout, y.data());
        // shortcut: nearest2x (kokoro_decoder_backward.cpp:67-81) then conv1x1
        if (w.up) {
            c.shortx.resize((int64_t)B * w.cin * Lout);
            for (int64_t r = 0; r < (int64_t)B * w.cin; ++r)
                for (int l = 0; l < Lin; ++l)
                    c.shortx[r * Lout + 2 * l] = c.shortx[r * Lout + 2 * l + 1] = x[r * Lin + l];
        } else {
            c.shortx.assign(x, x + nin);
        }
        const R inv = R(1) / std::sqrt(R(2));
        if (w.sc) {
            Vec<R> sc((size_t)nout);
            cfwd(w.c1x1, c.shortx.data(), Lout, sc.data());
            for (int64_t i = 0; i < nout; ++i) y[i] = (y[i] + sc[i]) * inv;
        } else {
            for (int64_t i = 0; i < nout; ++i) y[i] = (y[i] + c.shortx[i]) * inv;
        }
    }
    void blk_b(const Blk& w, BlkCache& c, const R* dY, Vec<R>& dX) {
        const int Lin = c.Lin, Lout = c.Lout;
        const int64_t nin = (int64_t)B * w.cin * Lin, nout = (int64_t)B * w.cout * Lout;
        const R inv = R(1) / std::sqrt(R(2));
        Vec<R> db((size_t)nout);
        for (int64_t i = 0; i < nout; ++i) db[i] = dY[i] * inv;
        Vec<R> dn2((size_t)nout), t1((size_t)nout);
        cbwd(w.c2, c.n2.data(), Lout, db.data(), dn2.data());
        leaky_bwd(c.n2_pre.data(), dn2.data(), nout, R(0.2), t1.data());
        Vec<R> dc1((size_t)nout);
        adain_b(w.n2, c.a2, w.cout, Lout, t1.data(), dc1.data());
        Vec<R> dpooled((size_t)B * w.cin * Lout);
        cbwd(w.c1, c.pooled.data(), Lout, dc1.data(), dpooled.data());
        Vec<R> dr((size_t)nin);
        if (w.up) {
            dwconvT_dgrad(dpooled.data(), B, w.cin, Lin, P + w.pool_w, 3, 2, 1, dr.data(), Lout);
            if (G) dwconvT_wgrad(dpooled.data(), c.pooled_in.data(), B, w.cin, Lin, 3, 2, 1, Lout, G + w.pool_w,
                                 G + w.pool_b);
        } else {
            dr = dpooled;
        }
        Vec<R> drp((size_t)nin);
        leaky_bwd(c.r_pre.data(), dr.data(), nin, R(0.2), drp.data());
        dX.assign((size_t)nin, R(0));
        adain_b(w.n1, c.a1, w.cin, Lin, drp.data(), dX.data());
        // shortcut branch
        Vec<R> dshort;
        if (w.sc) {
            dshort.resize((size_t)B * w.cin * Lout);
            cbwd(w.c1x1, c.shortx.data(), Lout, db.data(), dshort.data());
        } else {
            dshort = db;
        }
        if (w.up) {   // nearest2x adjoint, kokoro_decoder_backward.cpp:85-96
            for (int64_t r = 0; r < (int64_t)B * w.cin; ++r)
                for (int l = 0; l < Lin; ++l) dX[r * Lin + l] += dshort[r * Lout + 2 * l] + dshort[r * Lout + 2 * l + 1];
        } else {
            for (int64_t i = 0; i < nin; ++i) dX[i] += dshort[i];
        }
    }

    // ── AdaINResBlock1 (kokoro_decoder_backward.cpp:287-376)
    struct RB1Cache { AdaCache a1[3], a2[3]; Vec<R> s1[3], s2[3]; int L = 0; };
    void rb1_f(const RB1& w, const R* x_in, int L, RB1Cache& c, Vec<R>& x_out) {
        const int C = w.C;
        const int64_t n = (int64_t)B * C * L;
        c.L = L;
        Vec<R> x(x_in, x_in + n), t((size_t)n), u((size_t)n);
        for (int i = 0; i < 3; ++i) {
            adain_f(w.a1[i], x.data(), C, L, c.a1[i], t.data());
            c.s1[i].resize(n);
            snake_fwd(t.data(), B, C, L, P + w.al1[i], c.s1[i].data());
            cfwd(w.c1[i], c.s1[i].data(), L, u.data());
            adain_f(w.a2[i], u.data(), C, L, c.a2[i], t.data());
            c.s2[i].resize(n);
            snake_fwd(t.data(), B, C, L, P + w.al2[i], c.s2[i].data());
            cfwd(w.c2[i], c.s2[i].data(), L, u.data());
            for (int64_t j = 0; j < n; ++j) x[j] = u[j] + x[j];
        }
        x_out.swap(x);
    }
    void rb1_b(const RB1& w, RB1Cache& c, const R* dX_out, Vec<R>* dX_in) {
        const int C = w.C, L = c.L;
        const int64_t n = (int64_t)B * C * L;
        Vec<R> dx(dX_out, dX_out + n), t((size_t)n), u((size_t)n), pre((size_t)n);
        for (int i = 2; i >= 0; --i) {
            // convs2 -> snake2 -> adain2
            cbwd(w.c2[i], c.s2[i].data(), L, dx.data(), t.data());
            adain_fwd(c.a2[i].x.data(), B, C, L, aff_ptr(w.a2[i]), 2 * C, c.a2[i].mean.data(), c.a2[i].rstd.data(),
                      pre.data());
            snake_bwd(pre.data(), B, C, L, P + w.al2[i], t.data(), u.data(), g(w.al2[i]));
            adain_b(w.a2[i], c.a2[i], C, L, u.data(), t.data());
            // convs1 -> snake1 -> adain1
            cbwd(w.c1[i], c.s1[i].data(), L, t.data(), u.data());
            adain_fwd(c.a1[i].x.data(), B, C, L, aff_ptr(w.a1[i]), 2 * C, c.a1[i].mean.data(), c.a1[i].rstd.data(),
                      pre.data());
            snake_bwd(pre.data(), B, C, L, P + w.al1[i], u.data(), t.data(), g(w.al1[i]));
            adain_b(w.a1[i], c.a1[i], C, L, t.data(), u.data());
            for (int64_t j = 0; j < n; ++j) dx[j] += u[j];
        }
        if (dX_in) dX_in->swap(dx);
    }

    // ── full forward / backward state
    Vec<R> F0dn, Ndn, asrres, enc_in;
    BlkCache encc;
    std::vector<BlkCache> decc;
    std::vector<char> res_applied;
    std::vector<int> x_ch;
    std::vector<Vec<R>> dec_in;
    struct Stage { Vec<R> x_in, xsrc; RB1Cache noise; std::vector<RB1Cache> res; int Cin, Lin, Cout, Lout, Lu; };
    std::vector<Stage> st;
    Vec<R> head_x, post, audio;
    int L_last = 0, frames = 0;
    const R* har = nullptr;
    const R* asr = nullptr;

    void forward(const R* asr_, const R* F0, const R* Np, const R* har_, int frames_) {
        asr = asr_; har = har_; frames = frames_;
        const auto& cf = lay.cfg;
        resolve_affines();
        // backbone (kokoro_decoder_backward.cpp:482-537)
        F0dn.resize((size_t)B * T); Ndn.resize((size_t)B * T);
        cfwd(lay.F0c, F0, 2 * T, F0dn.data());
        cfwd(lay.Nc, Np, 2 * T, Ndn.data());
        asrres.resize((size_t)B * cf.asr_res_dim * T);
        cfwd(lay.asr_res, asr, T, asrres.data());
        const int Ce = cf.asr_dim + 2;
        enc_in.resize((size_t)B * Ce * T);
        for (int b = 0; b < B; ++b) {
            std::memcpy(&enc_in[(size_t)b * Ce * T], asr + (int64_t)b * cf.asr_dim * T, sizeof(R) * cf.asr_dim * T);
            std::memcpy(&enc_in[((size_t)b * Ce + cf.asr_dim) * T], &F0dn[(size_t)b * T], sizeof(R) * T);
            std::memcpy(&enc_in[((size_t)b * Ce + cf.asr_dim + 1) * T], &Ndn[(size_t)b * T], sizeof(R) * T);
        }
        Vec<R> x;
        blk_f(lay.enc, enc_in.data(), T, encc, x);
        int L = T;
        bool res = true;
        const int nd = (int)lay.dec.size();
        decc.resize(nd); res_applied.assign(nd, 0); x_ch.assign(nd, 0); dec_in.resize(nd);
        for (int i = 0; i < nd; ++i) {
            const Blk& w = lay.dec[i];
            const int Cx = (int)(x.size() / ((size_t)B * L));
            x_ch[i] = Cx;
            if (res) {
                res_applied[i] = 1;
                const int Cc = Cx + cf.asr_res_dim + 2;
                Vec<R>& bi = dec_in[i];
                bi.resize((size_t)B * Cc * L);
                for (int b = 0; b < B; ++b) {
                    R* o = &bi[(size_t)b * Cc * L];
                    std::memcpy(o, &x[(size_t)b * Cx * L], sizeof(R) * Cx * L);
                    std::memcpy(o + (size_t)Cx * L, &asrres[(size_t)b * cf.asr_res_dim * L],
                                sizeof(R) * cf.asr_res_dim * L);
                    std::memcpy(o + (size_t)(Cx + cf.asr_res_dim) * L, &F0dn[(size_t)b * L], sizeof(R) * L);
                    std::memcpy(o + (size_t)(Cx + cf.asr_res_dim + 1) * L, &Ndn[(size_t)b * L], sizeof(R) * L);
                }
            } else {
                dec_in[i] = x;
            }
            Vec<R> y;
            blk_f(w, dec_in[i].data(), L, decc[i], y);
            L = decc[i].Lout;
            x.swap(y);
            if (w.up) res = false;
        }
        // generator (kokoro_decoder_backward.cpp:592-667)
        const int U = cf.n_ups, K = cf.n_kernels;
        st.resize(U);
        for (int i = 0; i < U; ++i) {
            Stage& s = st[i];
            const Up& up = lay.ups[i];
            s.Cin = up.cin; s.Lin = L; s.Cout = up.cout;
            s.x_in = x;
            const int64_t nin = (int64_t)B * up.cin * L;
            Vec<R> a((size_t)nin);
            leaky_fwd(x.data(), nin, R(0.1), a.data());
            const Conv& nc = lay.noise[i];
            const int Lsrc = out_len(nc, frames);
            s.xsrc.resize((size_t)B * up.cout * Lsrc);
            cfwd(nc, har, frames, s.xsrc.data());
            Vec<R> src;
            rb1_f(lay.nres[i], s.xsrc.data(), Lsrc, s.noise, src);
            const int Lu = (L - 1) * up.s - 2 * up.p + (up.k - 1) + 1;
            s.Lu = Lu;
            Vec<R> u((size_t)B * up.cout * Lu);
            convT_fwd(a.data(), B, up.cin, L, P + up.w, P + up.b, up.cout, up.k, up.s, up.p, u.data(), Lu);
            int Lx = Lu;
            if (i == U - 1) {   // reflect pad left 1 (pad1d mode 1)
                Vec<R> pd((size_t)B * up.cout * (Lu + 1));
                for (int64_t r = 0; r < (int64_t)B * up.cout; ++r) {
                    pd[r * (Lu + 1)] = u[r * Lu + 1];
                    for (int l = 0; l < Lu; ++l) pd[r * (Lu + 1) + 1 + l] = u[r * Lu + l];
                }
                u.swap(pd);
                Lx = Lu + 1;
            }
            if (Lx != Lsrc) {
                std::fprintf(stderr, "oracle: noise source length %d != upsampled length %d at stage %d\n", Lsrc, Lx, i);
                std::abort();
            }
            s.Lout = Lx;
            for (size_t j = 0; j < u.size(); ++j) u[j] += src[j];
            s.res.resize(K);
            Vec<R> xs((size_t)B * up.cout * Lx, R(0));
            for (int j = 0; j < K; ++j) {
                Vec<R> xj;
                rb1_f(lay.rbs[i * K + j], u.data(), Lx, s.res[j], xj);
                for (size_t q = 0; q < xs.size(); ++q) xs[q] += xj[q];
            }
            const R invK = R(1) / (R)K;
            for (auto& v : xs) v *= invK;
            x.swap(xs);
            L = Lx;
        }
        // spectral head (kokoro_decoder_backward.cpp:378-410)
        L_last = L;
        const int Cl = lay.post.cin;
        head_x = x;
        const int64_t nl = (int64_t)B * Cl * L;
        Vec<R> xl((size_t)nl);
        leaky_fwd(x.data(), nl, R(0.01), xl.data());
        post.resize((size_t)B * lay.post.cout * L);
        cfwd(lay.post, xl.data(), L, post.data());
        head_xl = xl;
        const int nf = cf.n_fft / 2 + 1;
        Vec<R> re((size_t)B * nf * L), im((size_t)B * nf * L);
        for (int b = 0; b < B; ++b)
            for (int k = 0; k < nf; ++k)
                for (int l = 0; l < L; ++l) {
                    const R pm = post[((size_t)b * 2 * nf + k) * L + l];
                    const R pp = post[((size_t)b * 2 * nf + nf + k) * L + l];
                    const R mag = std::exp(pm), ang = std::sin(pp);
                    re[((size_t)b * nf + k) * L + l] = mag * std::cos(ang);
                    im[((size_t)b * nf + k) * L + l] = mag * std::sin(ang);
                }
        const Vec<R> win = hann<R>(cf.n_fft);
        audio.resize((size_t)B * cf.hop * (L - 1));
        istft_fwd(re.data(), im.data(), B, cf.n_fft, cf.hop, L, win.data(), audio.data());
    }
    Vec<R> head_xl;

    void backward(const R* daudio, R* d_asr, R* d_style) {
        const auto& cf = lay.cfg;
        const int L = L_last, nf = cf.n_fft / 2 + 1;
        // spectral head backward (kokoro_decoder_backward.cpp:412-458)
        const Vec<R> win = hann<R>(cf.n_fft);
        Vec<R> dre((size_t)B * nf * L), dim((size_t)B * nf * L);
        istft_bwd(daudio, B, cf.n_fft, cf.hop, L, win.data(), dre.data(), dim.data());
        Vec<R> dpost((size_t)B * 2 * nf * L);
        for (int b = 0; b < B; ++b)
            for (int k = 0; k < nf; ++k)
                for (int l = 0; l < L; ++l) {
                    const R pm = post[((size_t)b * 2 * nf + k) * L + l];
                    const R pp = post[((size_t)b * 2 * nf + nf + k) * L + l];
                    const R mag = std::exp(pm), ang = std::sin(pp);
                    const R ca = std::cos(ang), sa = std::sin(ang);
                    const R dR = dre[((size_t)b * nf + k) * L + l], dI = dim[((size_t)b * nf + k) * L + l];
                    const R dmag = dR * ca + dI * sa;
                    const R dang = mag * (-dR * sa + dI * ca);
                    dpost[((size_t)b * 2 * nf + k) * L + l] = dmag * mag;
                    dpost[((size_t)b * 2 * nf + nf + k) * L + l] = dang * std::cos(pp);
                }
        const int Cl = lay.post.cin;
        Vec<R> dxl((size_t)B * Cl * L), dX((size_t)B * Cl * L);
        cbwd(lay.post, head_xl.data(), L, dpost.data(), dxl.data());
        leaky_bwd(head_x.data(), dxl.data(), (int64_t)dX.size(), R(0.01), dX.data());
        // generator backward (kokoro_decoder_backward.cpp:669-737)
        const int U = cf.n_ups, K = cf.n_kernels;
        for (int i = U - 1; i >= 0; --i) {
            Stage& s = st[i];
            const Up& up = lay.ups[i];
            const int Lx = s.Lout;
            const int64_t n = (int64_t)B * up.cout * Lx;
            Vec<R> dsc((size_t)n);
            const R invK = R(1) / (R)K;
            for (int64_t j = 0; j < n; ++j) dsc[j] = dX[j] * invK;
            Vec<R> dm((size_t)n, R(0));
            for (int j = 0; j < K; ++j) {
                Vec<R> dj;
                rb1_b(lay.rbs[i * K + j], s.res[j], dsc.data(), &dj);
                for (int64_t q = 0; q < n; ++q) dm[q] += dj[q];
            }
            {   // noise branch: affine / conv grads kept; dX into har dropped
                Vec<R> dsrc;
                rb1_b(lay.nres[i], s.noise, dm.data(), &dsrc);
                if (G) {
                    const Conv& nc = lay.noise[i];
                    conv_wgrad(dsrc.data(), har, B, nc.cin, frames, nc.cout, nc.k, nc.s, nc.p, nc.d, Lx, G + nc.w,
                               g(nc.b));
                }
            }
            Vec<R> du;
            if (i == U - 1) {   // reflect-pad adjoint
                du.assign((size_t)B * up.cout * s.Lu, R(0));
                for (int64_t r = 0; r < (int64_t)B * up.cout; ++r) {
                    for (int l = 0; l < s.Lu; ++l) du[r * s.Lu + l] = dm[r * Lx + 1 + l];
                    du[r * s.Lu + 1] += dm[r * Lx];
                }
            } else {
                du.swap(dm);
            }
            const int64_t nin = (int64_t)B * up.cin * s.Lin;
            Vec<R> a((size_t)nin), da((size_t)nin);
            leaky_fwd(s.x_in.data(), nin, R(0.1), a.data());
            convT_dgrad(du.data(), B, up.cin, s.Lin, P + up.w, up.cout, up.k, up.s, up.p, da.data(), s.Lu);
            if (G) convT_wgrad(du.data(), a.data(), B, up.cin, s.Lin, up.cout, up.k, up.s, up.p, s.Lu, G + up.w, G + up.b);
            dX.resize((size_t)nin);
            leaky_bwd(s.x_in.data(), da.data(), nin, R(0.1), dX.data());
        }
        // backbone backward (kokoro_decoder_backward.cpp:539-574), extended with
        // the cat-channel grads (asr_res, F0_dn, N_dn) that the reference drops.
        const int nd = (int)lay.dec.size();
        const int Ar = cf.asr_res_dim;
        Vec<R> dasrres((size_t)B * Ar * T, R(0)), dF0((size_t)B * T, R(0)), dN((size_t)B * T, R(0));
        for (int i = nd - 1; i >= 0; --i) {
            Vec<R> bdx;
            blk_b(lay.dec[i], decc[i], dX.data(), bdx);
            const int Lin = decc[i].Lin;
            if (res_applied[i]) {
                const int Cx = x_ch[i], Cc = Cx + Ar + 2;
                dX.assign((size_t)B * Cx * Lin, R(0));
                for (int b = 0; b < B; ++b) {
                    const R* s0 = &bdx[(size_t)b * Cc * Lin];
                    std::memcpy(&dX[(size_t)b * Cx * Lin], s0, sizeof(R) * Cx * Lin);
                    for (int64_t q = 0; q < (int64_t)Ar * Lin; ++q) dasrres[(size_t)b * Ar * Lin + q] += s0[(size_t)Cx * Lin + q];
                    for (int l = 0; l < Lin; ++l) {
                        dF0[(size_t)b * Lin + l] += s0[(size_t)(Cx + Ar) * Lin + l];
                        dN[(size_t)b * Lin + l] += s0[(size_t)(Cx + Ar + 1) * Lin + l];
                    }
                }
            } else {
                dX.swap(bdx);
            }
        }
        Vec<R> denc;
        blk_b(lay.enc, encc, dX.data(), denc);
        const int Ce = cf.asr_dim + 2;
        for (int b = 0; b < B; ++b)
            for (int l = 0; l < T; ++l) {
                dF0[(size_t)b * T + l] += denc[((size_t)b * Ce + cf.asr_dim) * T + l];
                dN[(size_t)b * T + l] += denc[((size_t)b * Ce + cf.asr_dim + 1) * T + l];
            }
        // frozen-input convs: weight grads only (F0/N have no input grad)
        if (G) {
            conv_wgrad(dF0.data(), F0_in, B, 1, 2 * T, 1, 3, 2, 1, 1, T, G + lay.F0c.w, G + lay.F0c.b);
            conv_wgrad(dN.data(), N_in, B, 1, 2 * T, 1, 3, 2, 1, 1, T, G + lay.Nc.w, G + lay.Nc.b);
        }
        Vec<R> dasr_res((size_t)B * cf.asr_dim * T);
        cbwd(lay.asr_res, asr, T, dasrres.data(), dasr_res.data());
        if (d_asr)
            for (int b = 0; b < B; ++b)
                for (int64_t q = 0; q < (int64_t)cf.asr_dim * T; ++q)
                    d_asr[(size_t)b * cf.asr_dim * T + q] = denc[(size_t)b * Ce * T + q] + dasr_res[(size_t)b * cf.asr_dim * T + q];
        affine_backward(d_style);
    }
    const R* F0_in = nullptr;
    const R* N_in = nullptr;
};

}  // namespace orc

// ─── C API ──────────────────────────────────────────────────────────────────

namespace {

template <class R>
int run(const orc_cfg* cfg, int B, int T, const R* params, const R* asr, const R* F0, const R* N, const R* style,
        const R* har, int frames, const R* aff_in, const R* daudio, R* audio_out, R* grads, R* d_asr, R* d_style,
        R* d_aff, R* aff_out) {
    orc::Layout lay(*cfg);
    orc::Decoder<R> d(lay, params, grads, B, T);
    d.style = style;
    d.aff_in = aff_in;
    d.F0_in = F0;
    d.N_in = N;
    std::vector<R> har_local;
    if (!har) {
        // the harmonic source makes n_fft + 2 channels (|X| and angle X per bin)
        if (cfg->har_ch != cfg->n_fft + 2) return -2;
        const int S = 2 * T * cfg->upsample_scale;
        frames = S / cfg->hop + 1;
        har_local.resize((size_t)B * cfg->har_ch * frames);
        orc::harmonic_source(F0, B, 2 * T, params + lay.llin_w, params + lay.llin_b, *cfg, har_local.data());
        har = har_local.data();
    }
    d.forward(asr, F0, N, har, frames);
    if (audio_out) std::memcpy(audio_out, d.audio.data(), sizeof(R) * d.audio.size());
    if (aff_out) std::memcpy(aff_out, d.aff.data(), sizeof(R) * d.aff.size());
    if (daudio) {
        d.backward(daudio, d_asr, d_style);
        if (d_aff) std::memcpy(d_aff, d.daff.data(), sizeof(R) * d.daff.size());
    }
    return 0;
}

// One block forward (+ backward when dy != NULL); x, y, dy, dx in NCL.
template <class R>
int run_block(const orc_block_spec* spec, int B, int L, const R* params, const R* x, const R* style, const R* aff_in,
              const R* dy, R* y, R* grads, R* dx, R* d_style, R* d_aff, R* aff_out) {
    if (spec->kind != 1 && spec->kind != 2) return -1;
    orc::Layout lay(*spec);
    orc::Decoder<R> d(lay, params, grads, B, L);
    d.style = style;
    d.aff_in = aff_in;
    d.resolve_affines();
    if (aff_out) std::memcpy(aff_out, d.aff.data(), sizeof(R) * d.aff.size());
    if (grads) std::fill(grads, grads + lay.total, R(0));
    if (d_style) std::fill(d_style, d_style + (int64_t)B * spec->style_dim, R(0));
    std::vector<R> out, din;
    if (spec->kind == 1) {
        typename orc::Decoder<R>::BlkCache c;
        d.blk_f(lay.enc, x, L, c, out);
        if (dy) d.blk_b(lay.enc, c, dy, din);
    } else {
        typename orc::Decoder<R>::RB1Cache c;
        d.rb1_f(lay.rbs[0], x, L, c, out);
        if (dy) d.rb1_b(lay.rbs[0], c, dy, &din);
    }
    if (y) std::memcpy(y, out.data(), sizeof(R) * out.size());
    if (dy) {
        if (dx) std::memcpy(dx, din.data(), sizeof(R) * din.size());
        d.affine_backward(d_style);
        if (d_aff) std::memcpy(d_aff, d.daff.data(), sizeof(R) * d.daff.size());
    }
    return 0;
}

}  // namespace

extern "C" {

int orc_block_param_count(const orc_block_spec* spec, int64_t* total, int* n_entries, int* n_affine,
                          int64_t* aff_per_clip) {
    orc::Layout lay(*spec);
    if (total) *total = lay.total;
    if (n_entries) *n_entries = (int)lay.table.size();
    if (n_affine) *n_affine = (int)lay.aff_C.size();
    if (aff_per_clip) *aff_per_clip = lay.aff_per_clip;
    return 0;
}

int orc_block_param_table(const orc_block_spec* spec, orc_param* out, int max_entries, int* aff_C) {
    orc::Layout lay(*spec);
    const int n = std::min<int>(max_entries, (int)lay.table.size());
    for (int i = 0; i < n; ++i) out[i] = lay.table[i];
    if (aff_C)
        for (size_t i = 0; i < lay.aff_C.size(); ++i) aff_C[i] = lay.aff_C[i];
    return n;
}

int orc_block_run_f32(const orc_block_spec* spec, int B, int L, const float* params, const float* x,
                      const float* style, const float* aff_in, const float* dy, float* y, float* grads, float* dx,
                      float* d_style, float* d_aff, float* aff_out) {
    return run_block<float>(spec, B, L, params, x, style, aff_in, dy, y, grads, dx, d_style, d_aff, aff_out);
}
int orc_block_run_f64(const orc_block_spec* spec, int B, int L, const double* params, const double* x,
                      const double* style, const double* aff_in, const double* dy, double* y, double* grads,
                      double* dx, double* d_style, double* d_aff, double* aff_out) {
    return run_block<double>(spec, B, L, params, x, style, aff_in, dy, y, grads, dx, d_style, d_aff, aff_out);
}

int orc_param_count(const orc_cfg* cfg, int64_t* total, int* n_entries, int* n_affine, int64_t* aff_per_clip) {
    orc::Layout lay(*cfg);
    if (total) *total = lay.total;
    if (n_entries) *n_entries = (int)lay.table.size();
    if (n_affine) *n_affine = (int)lay.aff_C.size();
    if (aff_per_clip) *aff_per_clip = lay.aff_per_clip;
    return 0;
}

int orc_param_table(const orc_cfg* cfg, orc_param* out, int max_entries, int* aff_C) {
    orc::Layout lay(*cfg);
    const int n = std::min<int>(max_entries, (int)lay.table.size());
    for (int i = 0; i < n; ++i) out[i] = lay.table[i];
    if (aff_C)
        for (size_t i = 0; i < lay.aff_C.size(); ++i) aff_C[i] = lay.aff_C[i];
    return n;
}

int orc_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

// Full decoder forward (+ backward when daudio != NULL). See run() above.
int orc_decoder_run_f32(const orc_cfg* cfg, int B, int T, const float* params, const float* asr, const float* F0,
                        const float* N, const float* style, const float* har, int frames, const float* aff_in,
                        const float* daudio, float* audio, float* grads, float* d_asr, float* d_style, float* d_aff,
                        float* aff_out) {
    return run<float>(cfg, B, T, params, asr, F0, N, style, har, frames, aff_in, daudio, audio, grads, d_asr,
                      d_style, d_aff, aff_out);
}
int orc_decoder_run_f64(const orc_cfg* cfg, int B, int T, const double* params, const double* asr,
                        const double* F0, const double* N, const double* style, const double* har, int frames,
                        const double* aff_in, const double* daudio, double* audio, double* grads, double* d_asr,
                        double* d_style, double* d_aff, double* aff_out) {
    return run<double>(cfg, B, T, params, asr, F0, N, style, har, frames, aff_in, daudio, audio, grads, d_asr,
                       d_style, d_aff, aff_out);
}

int orc_harmonic_source_f32(const orc_cfg* cfg, const float* F0, int B, int F, const float* lw, const float* lb,
                            float* har) {
    orc::harmonic_source<float>(F0, B, F, lw, lb, *cfg, har);
    return 0;
}

// ── atom-level entry points (per-op parity and finite-difference tests)

#define ORC_ATOMS(R, SFX)                                                                                          \
    void orc_conv_fwd_##SFX(const R* x, int B, int Ci, int L, const R* W, const R* b, int Co, int k, int s, int p,  \
                            int d, R* y) {                                                                         \
        orc::conv_fwd<R>(x, B, Ci, L, W, b, Co, k, s, p, d, y, orc::conv_out_len(L, k, s, p, d));                  \
    }                                                                                                              \
    void orc_conv_dgrad_##SFX(const R* dy, int B, int Ci, int L, const R* W, int Co, int k, int s, int p, int d,   \
                              R* dx) {                                                                             \
        orc::conv_dgrad<R>(dy, B, Ci, L, W, Co, k, s, p, d, dx, orc::conv_out_len(L, k, s, p, d));                 \
    }                                                                                                              \
    void orc_conv_wgrad_##SFX(const R* dy, const R* x, int B, int Ci, int L, int Co, int k, int s, int p, int d,   \
                              R* dW, R* db) {                                                                      \
        orc::conv_wgrad<R>(dy, x, B, Ci, L, Co, k, s, p, d, orc::conv_out_len(L, k, s, p, d), dW, db);             \
    }                                                                                                              \
    void orc_convT_fwd_##SFX(const R* x, int B, int Ci, int L, const R* W, const R* b, int Co, int k, int s,       \
                             int p, R* y) {                                                                        \
        orc::convT_fwd<R>(x, B, Ci, L, W, b, Co, k, s, p, y, (L - 1) * s - 2 * p + k);                             \
    }                                                                                                              \
    void orc_convT_dgrad_##SFX(const R* dy, int B, int Ci, int L, const R* W, int Co, int k, int s, int p, R* dx) { \
        orc::convT_dgrad<R>(dy, B, Ci, L, W, Co, k, s, p, dx, (L - 1) * s - 2 * p + k);                            \
    }                                                                                                              \
    void orc_convT_wgrad_##SFX(const R* dy, const R* x, int B, int Ci, int L, int Co, int k, int s, int p, R* dW,  \
                               R* db) {                                                                            \
        orc::convT_wgrad<R>(dy, x, B, Ci, L, Co, k, s, p, (L - 1) * s - 2 * p + k, dW, db);                        \
    }                                                                                                              \
    void orc_adain_fwd_##SFX(const R* x, int B, int C, int L, const R* gb, R eps, R* y) {                          \
        std::vector<R> m((size_t)B * C), r((size_t)B * C);                                                         \
        orc::in_stats<R>(x, B, C, L, eps, m.data(), r.data());                                                     \
        orc::adain_fwd<R>(x, B, C, L, gb, 2 * C, m.data(), r.data(), y);                                           \
    }                                                                                                              \
    void orc_adain_bwd_##SFX(const R* x, int B, int C, int L, const R* gb, R eps, const R* dy, R* dx, R* dgb) {    \
        std::vector<R> m((size_t)B * C), r((size_t)B * C);                                                         \
        orc::in_stats<R>(x, B, C, L, eps, m.data(), r.data());                                                     \
        orc::adain_bwd<R>(x, B, C, L, gb, 2 * C, m.data(), r.data(), dy, dx, dgb);                                 \
    }                                                                                                              \
    void orc_snake_fwd_##SFX(const R* x, int B, int C, int L, const R* alpha, R* y) {                              \
        orc::snake_fwd<R>(x, B, C, L, alpha, y);                                                                   \
    }                                                                                                              \
    void orc_snake_bwd_##SFX(const R* x, int B, int C, int L, const R* alpha, const R* dy, R* dx, R* dalpha) {     \
        orc::snake_bwd<R>(x, B, C, L, alpha, dy, dx, dalpha);                                                      \
    }                                                                                                              \
    void orc_istft_fwd_##SFX(const R* re, const R* im, int B, int n_fft, int hop, int L, R* audio) {               \
        const std::vector<R> w = orc::hann<R>(n_fft);                                                              \
        orc::istft_fwd<R>(re, im, B, n_fft, hop, L, w.data(), audio);                                              \
    }                                                                                                              \
    void orc_istft_bwd_##SFX(const R* da, int B, int n_fft, int hop, int L, R* dre, R* dim) {                      \
        const std::vector<R> w = orc::hann<R>(n_fft);                                                              \
        orc::istft_bwd<R>(da, B, n_fft, hop, L, w.data(), dre, dim);                                               \
    }

ORC_ATOMS(float, f32)
ORC_ATOMS(double, f64)

}  // extern "C"
