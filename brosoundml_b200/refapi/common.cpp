// brotensor::Tensor (managed storage), the runtime and copy ops, the generic
// modules' forwards, and the helpers that map the reference's weight structs onto
// this build's flat parameter layout.
#include <brotensor/ops/concat.h>
#include <brotensor/runtime.h>
#include <brotensor/tensor.h>

#include <algorithm>
#include <cstring>
#include <utility>

#include "brosoundml/modules.h"
#include "internal.h"

namespace brotensor {

using brosoundml::refapi::check;

void Tensor::alloc(std::int64_t n) {
    release();
    if (n <= 0) return;
    void* p = nullptr;
    check(bsml_managed_alloc(n * (std::int64_t)sizeof(float), &p));
    data = p;
    cap_ = (std::size_t)n;
}

void Tensor::release() {
    if (data) bsml_managed_free(data);
    data = nullptr;
    cap_ = 0;
}

Tensor::~Tensor() { release(); }

Tensor::Tensor(const Tensor& o) : rows(o.rows), cols(o.cols), device(o.device), dtype(o.dtype) {
    alloc(o.size());
    if (o.size() > 0) {
        brosoundml::refapi::copy_floats(f32(), o.f32(), o.size());
        brosoundml::refapi::sync();
    }
}

Tensor::Tensor(Tensor&& o) noexcept
    : rows(o.rows), cols(o.cols), device(o.device), dtype(o.dtype), data(o.data), cap_(o.cap_) {
    o.data = nullptr;
    o.cap_ = 0;
    o.rows = o.cols = 0;
}

Tensor& Tensor::operator=(const Tensor& o) {
    if (this == &o) return *this;
    if ((std::int64_t)cap_ < o.size() || o.size() == 0) alloc(o.size());
    rows = o.rows;
    cols = o.cols;
    device = o.device;
    dtype = o.dtype;
    if (o.size() > 0) {
        brosoundml::refapi::copy_floats(f32(), o.f32(), o.size());
        brosoundml::refapi::sync();
    }
    return *this;
}

Tensor& Tensor::operator=(Tensor&& o) noexcept {
    if (this == &o) return *this;
    release();
    rows = o.rows;
    cols = o.cols;
    device = o.device;
    dtype = o.dtype;
    data = o.data;
    cap_ = o.cap_;
    o.data = nullptr;
    o.cap_ = 0;
    o.rows = o.cols = 0;
    return *this;
}

Tensor Tensor::zeros_on(Device dev, int r, int c, Dtype dt) {
    if (r < 0 || c < 0) brosoundml::refapi::fail("Tensor", "negative shape");
    Tensor t;
    t.rows = r;
    t.cols = c;
    t.device = dev;
    t.dtype = dt;
    t.alloc((std::int64_t)r * c);   // zero-filled
    return t;
}

Tensor Tensor::empty_on(Device dev, int r, int c, Dtype dt) { return zeros_on(dev, r, c, dt); }

Tensor Tensor::from_host_on(Device dev, const float* src, int r, int c) {
    Tensor t = zeros_on(dev, r, c);
    if (t.size() > 0) {
        check(bsml_memcpy(t.data, src, t.size() * (std::int64_t)sizeof(float), nullptr));
        brosoundml::refapi::sync();
    }
    return t;
}

Tensor Tensor::mat(int r, int c) { return zeros_on(Device::CPU, r, c); }

std::vector<float> Tensor::to_host_vector() const {
    std::vector<float> v((std::size_t)size());
    if (size() > 0) {
        check(bsml_memcpy(v.data(), data, size() * (std::int64_t)sizeof(float), nullptr));
        brosoundml::refapi::sync();
    }
    return v;
}

Tensor Tensor::to(Device dev) const {
    Tensor t(*this);
    t.device = dev;
    return t;
}

void Tensor::resize(int r, int c) {
    if (r < 0 || c < 0) brosoundml::refapi::fail("Tensor::resize", "negative shape");
    const std::int64_t n = (std::int64_t)r * c;
    if (n != size() || (n > 0 && !data)) alloc(n);
    rows = r;
    cols = c;
}

void init() {
    // creates the context of device 0 (the first C-ABI call would otherwise)
    check(bsml_synchronize());
}

void synchronize() { check(bsml_synchronize()); }

void copy_d2d(const Tensor& src, int src_off, Tensor& dst, int dst_off, int n) {
    if (n < 0 || src_off < 0 || dst_off < 0 || src_off + (std::int64_t)n > src.size() ||
        dst_off + (std::int64_t)n > dst.size())
        brosoundml::refapi::fail("copy_d2d", "range out of bounds");
    brosoundml::refapi::copy_floats(dst.f32() + dst_off, src.f32() + src_off, n);
    brosoundml::refapi::sync();
}

}  // namespace brotensor

namespace brosoundml {

namespace bt = brotensor;
using refapi::check;
using refapi::check_count;
using refapi::need;

void Linear::forward(const bt::Tensor& x, bt::Tensor& y) const {
    need(x.size() == in_features && W.size() == (std::int64_t)out_features * in_features, "Linear::forward",
         "shape mismatch");
    need(b.empty() || b.size() == out_features, "Linear::forward", "bias shape mismatch");
    refapi::shape_out(y, out_features, 1, x);
    // a 1x1 convolution over one position
    check(bsml_conv1d_forward(x.f32(), 1, in_features, 1, W.f32(), b.empty() ? nullptr : b.f32(), out_features, 1,
                              1, 0, 1, y.f32(), nullptr));
    refapi::sync();
}

void Linear::forward_batched(const bt::Tensor& X, bt::Tensor& Y) const {
    need(X.cols == in_features && W.size() == (std::int64_t)out_features * in_features, "Linear::forward_batched",
         "shape mismatch");
    need(b.empty() || b.size() == out_features, "Linear::forward_batched", "bias shape mismatch");
    refapi::shape_out(Y, X.rows, out_features, X);
    check(bsml_conv1d_forward(X.f32(), X.rows, in_features, 1, W.f32(), b.empty() ? nullptr : b.f32(), out_features,
                              1, 1, 0, 1, Y.f32(), nullptr));
    refapi::sync();
}

void Conv1d::forward(const bt::Tensor& X, int N, int L, bt::Tensor& Y) const {
    const char* where = "Conv1d::forward";
    need(groups == 1, where, "groups other than 1 are not supported by this build");
    need(N > 0 && L > 0 && X.size() == (std::int64_t)N * in_channels * L, where, "input shape mismatch");
    need(W.size() == (std::int64_t)out_channels * in_channels * kernel_size, where, "weight shape mismatch");
    need(b.empty() || b.size() == out_channels, where, "bias shape mismatch");
    const int Lo = out_len(L);
    need(Lo > 0, where, "input shorter than the kernel");
    refapi::shape_out(Y, N, out_channels * Lo, X);
    check(bsml_conv1d_forward(X.f32(), N, in_channels, L, W.f32(), b.empty() ? nullptr : b.f32(), out_channels,
                              kernel_size, stride, padding, dilation, Y.f32(), nullptr));
    refapi::sync();
}

namespace refapi {

void shape_out(bt::Tensor& out, int r, int c, const bt::Tensor& like) {
    out.resize(r, c);
    out.device = like.device;
}

void need_size(const bt::Tensor& t, std::int64_t n, const char* where, const char* what) {
    if (t.size() != n)
        fail(where, std::string(what) + " has " + std::to_string(t.size()) + " elements, expected " +
                        std::to_string(n));
}

// ── ParamBuf
ParamBuf::~ParamBuf() {
    if (p_) bsml_managed_free(p_);
    if (zeros_) bsml_managed_free(zeros_);
}

void ParamBuf::init(const bsml_decoder* h) {
    std::int64_t n = 0, apc = 0;
    int ne = 0, na = 0;
    check(bsml_decoder_param_count(h, &n, &ne, &na, &apc));
    table_.resize((std::size_t)ne);
    check_count(bsml_decoder_param_table(h, table_.data(), ne, nullptr));
    n_ = n;
    max_entry_ = 0;
    for (const auto& e : table_) max_entry_ = std::max(max_entry_, e.numel);
    void* p = nullptr;
    check(bsml_managed_alloc(std::max<std::int64_t>(n, 1) * 4, &p));
    p_ = (float*)p;
    check(bsml_managed_alloc(std::max<std::int64_t>(max_entry_, 1) * 4, &p));
    zeros_ = (float*)p;
}

const bsml_param_entry* ParamBuf::find(const std::string& name) const {
    for (const auto& e : table_)
        if (name == e.name) return &e;
    return nullptr;
}

void ParamBuf::set(const std::string& name, const bt::Tensor& t, const char* where) {
    const bsml_param_entry* e = find(name);
    if (!e) fail(where, "no parameter named " + name);
    if (t.empty()) {
        copy_floats(p_ + e->offset, zeros_, e->numel);
        return;
    }
    if (t.size() != e->numel)
        fail(where, name + " has " + std::to_string(t.size()) + " elements, the architecture wants " +
                        std::to_string(e->numel));
    copy_floats(p_ + e->offset, t.f32(), e->numel);
}

// ── EngineState
EngineState::~EngineState() {
    if (aff) bsml_managed_free(aff);
    if (daff) bsml_managed_free(daff);
    if (h) bsml_decoder_destroy(h);
}

namespace {

template <class K>
std::vector<unsigned char> key_of(int tag, const K& k) {
    std::vector<unsigned char> v(sizeof(int) + sizeof(K));
    std::memcpy(v.data(), &tag, sizeof(int));
    std::memcpy(v.data() + sizeof(int), &k, sizeof(K));
    return v;
}

std::shared_ptr<EngineState> finish_state(std::shared_ptr<EngineState> s) {
    s->params.init(s->h);
    std::int64_t n = 0, apc = 0;
    int ne = 0, na = 0;
    check(bsml_decoder_param_count(s->h, &n, &ne, &na, &apc));
    s->aff_C.resize((std::size_t)na);
    std::vector<bsml_param_entry> tab((std::size_t)ne);
    check_count(bsml_decoder_param_table(s->h, tab.data(), ne, s->aff_C.data()));
    s->aff_per_clip = apc;
    void* p = nullptr;
    check(bsml_managed_alloc(std::max<std::int64_t>(apc, 1) * 4, &p));
    s->aff = (float*)p;
    check(bsml_managed_alloc(std::max<std::int64_t>(apc, 1) * 4, &p));
    s->daff = (float*)p;
    // fp32-grade tensor-core arithmetic; narrow channel counts fall back to the
    // fp32 CUDA-core kernels inside the engine
    check(bsml_decoder_set_math(s->h, BSML_MATH_TF32X3));
    return s;
}

}  // namespace

std::shared_ptr<EngineState> decoder_state(const bsml_decoder_config& cfg, std::shared_ptr<void> cur) {
    auto key = key_of(0, cfg);
    if (cur) {
        auto s = std::static_pointer_cast<EngineState>(cur);
        if (s->key == key) return s;
    }
    auto s = std::make_shared<EngineState>();
    s->key = key;
    check(bsml_decoder_create(&cfg, 0, &s->h));
    return finish_state(s);
}

std::shared_ptr<EngineState> block_state(const bsml_block_spec& spec, std::shared_ptr<void> cur) {
    auto key = key_of(1, spec);
    if (cur) {
        auto s = std::static_pointer_cast<EngineState>(cur);
        if (s->key == key) return s;
    }
    auto s = std::make_shared<EngineState>();
    s->key = key;
    check(bsml_block_create(&spec, 0, &s->h));
    return finish_state(s);
}

// ── architecture of the reference's structs
namespace {

int style_dim_of(const AdaIN1dWeights& a) {
    if (a.fc.in_features > 0) return a.fc.in_features;
    if (a.style_dim > 0) return a.style_dim;
    return 128;   // Kokoro; only the fc shapes depend on it, and an empty fc is not read
}

void check_conv(const Conv1d& c, int cin, int cout, int k, int s, int p, int d, const char* where,
                const std::string& what) {
    if (c.in_channels != cin || c.out_channels != cout || c.kernel_size != k || c.stride != s || c.padding != p ||
        c.dilation != d || c.groups != 1)
        fail(where, what + ": expected Conv1d(" + std::to_string(cin) + " -> " + std::to_string(cout) + ", k" +
                        std::to_string(k) + " s" + std::to_string(s) + " p" + std::to_string(p) + " d" +
                        std::to_string(d) + ")");
}

}  // namespace

bsml_block_spec spec_of(const AdainResBlk1dWeights& w) {
    const char* where = "adain_resblk_1d";
    need(w.channels_in > 0 && w.channels_out > 0, where, "channel counts must be positive");
    need(w.learned_sc == (w.channels_in != w.channels_out), where,
         "a learned 1x1 shortcut exactly when channels_in != channels_out is supported");
    check_conv(w.conv1, w.channels_in, w.channels_out, 3, 1, 1, 1, where, "conv1");
    check_conv(w.conv2, w.channels_out, w.channels_out, 3, 1, 1, 1, where, "conv2");
    if (w.learned_sc) check_conv(w.conv1x1, w.channels_in, w.channels_out, 1, 1, 0, 1, where, "conv1x1");
    bsml_block_spec s{};
    s.kind = BSML_BLOCK_RESBLK1D;
    s.style_dim = style_dim_of(w.norm1);
    s.cin = w.channels_in;
    s.cout = w.channels_out;
    s.upsample = w.upsample ? 1 : 0;
    return s;
}

bsml_block_spec spec_of(const AdaINResBlock1Weights& w) {
    const char* where = "adain_resblock1";
    need(w.channels > 0 && w.kernel_size > 0 && (w.kernel_size & 1), where, "channels and an odd kernel are needed");
    need(w.dilations.size() == 3, where, "three dilations are needed");
    for (int i = 0; i < 3; ++i) {
        const int d = w.dilations[i];
        check_conv(w.convs1[i], w.channels, w.channels, w.kernel_size, 1, d * (w.kernel_size - 1) / 2, d, where,
                   "convs1[" + std::to_string(i) + "]");
        check_conv(w.convs2[i], w.channels, w.channels, w.kernel_size, 1, (w.kernel_size - 1) / 2, 1, where,
                   "convs2[" + std::to_string(i) + "]");
    }
    bsml_block_spec s{};
    s.kind = BSML_BLOCK_RESBLOCK1;
    s.style_dim = style_dim_of(w.adain1[0]);
    s.cin = s.cout = w.channels;
    s.kernel = w.kernel_size;
    for (int i = 0; i < 3; ++i) s.dil[i] = w.dilations[i];
    return s;
}

bsml_decoder_config config_of(const DecoderBackbone* bb, const Generator* gen) {
    const char* where = "decoder config";
    bsml_decoder_config c{};
    c.harmonic_num = 8;
    c.sample_rate = 24000;
    if (bb) {
        need(!bb->decode.empty() && bb->decode.size() <= 8, where, "1 to 8 decode blocks are supported");
        c.asr_dim = bb->asr_res.in_channels;
        c.asr_res_dim = bb->asr_res.out_channels;
        c.enc_dim = bb->encode.channels_out;
        c.style_dim = style_dim_of(bb->encode.norm1);
        c.n_decode = (int)bb->decode.size();
        c.upsample_block = -1;
        for (int i = 0; i < c.n_decode; ++i) {
            c.dec_out[i] = bb->decode[i].channels_out;
            if (bb->decode[i].upsample) {
                need(c.upsample_block < 0, where, "one upsampling decode block is supported");
                c.upsample_block = i;
            }
        }
        check_conv(bb->F0_conv, 1, 1, 3, 2, 1, 1, where, "F0_conv");
        check_conv(bb->N_conv, 1, 1, 3, 2, 1, 1, where, "N_conv");
        check_conv(bb->asr_res, c.asr_dim, c.asr_res_dim, 1, 1, 0, 1, where, "asr_res");
        need(bb->encode.channels_in == c.asr_dim + 2, where, "encode takes [asr, F0, N]");
    }
    if (gen) {
        const int U = gen->num_upsamples, K = gen->num_kernels;
        need(U >= 1 && U <= 4 && K >= 1 && K <= 4, where, "1-4 upsamples and 1-4 kernels are supported");
        need((int)gen->ups_W.size() == U && (int)gen->ups_C_in.size() == U && (int)gen->ups_C_out.size() == U &&
                 (int)gen->ups_k.size() == U && (int)gen->ups_stride.size() == U && (int)gen->ups_pad.size() == U &&
                 (int)gen->noise_convs.size() == U && (int)gen->noise_res.size() == U &&
                 (int)gen->resblocks.size() == U * K,
             where, "generator lists do not match num_upsamples / num_kernels");
        c.n_ups = U;
        c.n_kernels = K;
        c.init_ch = gen->ups_C_in[0];
        for (int i = 0; i < U; ++i) {
            need(gen->ups_C_in[i] == (c.init_ch >> i) && gen->ups_C_out[i] == (c.init_ch >> (i + 1)), where,
                 "upsamplers must halve the channel count");
            need(gen->ups_pad[i] == (gen->ups_k[i] - gen->ups_stride[i]) / 2, where,
                 "upsampler padding must be (k - stride) / 2");
            c.ups_rate[i] = gen->ups_stride[i];
            c.ups_kernel[i] = gen->ups_k[i];
            const Conv1d& nc = gen->noise_convs[i];
            c.noise_kernel[i] = nc.kernel_size;
            c.noise_stride[i] = nc.stride;
            c.noise_pad[i] = nc.padding;
            need(nc.dilation == 1 && nc.groups == 1 && nc.out_channels == (c.init_ch >> (i + 1)), where,
                 "noise_convs shape");
            const AdaINResBlock1Weights& nr = gen->noise_res[i];
            spec_of(nr);
            c.nr_kernel[i] = nr.kernel_size;
            for (int j = 0; j < 3; ++j) c.nr_dil[i][j] = nr.dilations[j];
        }
        c.har_ch = gen->noise_convs[0].in_channels;
        for (int j = 0; j < K; ++j) {
            const AdaINResBlock1Weights& r = gen->resblocks[j];
            spec_of(r);
            c.rb_kernel[j] = r.kernel_size;
            for (int d = 0; d < 3; ++d) c.rb_dil[j][d] = r.dilations[d];
            for (int i = 1; i < U; ++i) {
                const AdaINResBlock1Weights& q = gen->resblocks[i * K + j];
                need(q.kernel_size == r.kernel_size && q.dilations == r.dilations, where,
                     "resblock kernels / dilations must repeat across stages");
            }
        }
        c.n_fft = gen->n_fft;
        c.hop = gen->hop_size;
        need(gen->win_size == gen->n_fft, where, "win_size must equal n_fft");
        c.post_kernel = gen->conv_post.kernel_size;
        check_conv(gen->conv_post, c.init_ch >> U, c.n_fft + 2, c.post_kernel, 1, (c.post_kernel - 1) / 2, 1, where,
                   "conv_post");
        int up = c.hop;
        for (int i = 0; i < U; ++i) up *= c.ups_rate[i];
        c.upsample_scale = up;
        if (!bb) {
            // stand-in backbone (never run): one decode block that outputs init_ch
            c.asr_dim = 1; c.asr_res_dim = 1; c.enc_dim = 1;
            c.style_dim = style_dim_of(gen->noise_res[0].adain1[0]);
            c.n_decode = 1; c.dec_out[0] = c.init_ch; c.upsample_block = -1;
        }
    } else {
        // stand-in generator (never run) after the backbone's last block
        const int C = c.dec_out[c.n_decode - 1];
        need(C >= 2, where, "the backbone's last block needs at least 2 channels");
        c.n_ups = 1; c.n_kernels = 1; c.init_ch = C;
        c.ups_rate[0] = 1; c.ups_kernel[0] = 1;
        c.noise_kernel[0] = 1; c.noise_stride[0] = 1; c.noise_pad[0] = 0;
        c.nr_kernel[0] = 1; c.rb_kernel[0] = 1;
        for (int j = 0; j < 3; ++j) { c.nr_dil[0][j] = 1; c.rb_dil[0][j] = 1; }
        c.har_ch = 1; c.n_fft = 2; c.hop = 1; c.post_kernel = 1; c.harmonic_num = 0; c.upsample_scale = 1;
    }
    if (bb && gen) need(c.dec_out[c.n_decode - 1] == c.init_ch, where, "the backbone must output init_ch channels");
    return c;
}

// ── parameter filling (keys: the upstream state-dict names the layout uses)
namespace {
std::string sub(const std::string& p, const std::string& n) { return p.empty() ? n : p + "." + n; }
}  // namespace

void fill_block(ParamBuf& P, const std::string& pre, const AdainResBlk1dWeights& w, const char* where) {
    P.set(sub(pre, "norm1.fc.weight"), w.norm1.fc.W, where);
    P.set(sub(pre, "norm1.fc.bias"), w.norm1.fc.b, where);
    P.set(sub(pre, "norm2.fc.weight"), w.norm2.fc.W, where);
    P.set(sub(pre, "norm2.fc.bias"), w.norm2.fc.b, where);
    P.set(sub(pre, "conv1.weight"), w.conv1.W, where);
    P.set(sub(pre, "conv1.bias"), w.conv1.b, where);
    P.set(sub(pre, "conv2.weight"), w.conv2.W, where);
    P.set(sub(pre, "conv2.bias"), w.conv2.b, where);
    if (w.learned_sc) P.set(sub(pre, "conv1x1.weight"), w.conv1x1.W, where);
    if (w.upsample) {
        P.set(sub(pre, "pool.weight"), w.pool_W, where);
        P.set(sub(pre, "pool.bias"), w.pool_b, where);
    }
}

void fill_rb1(ParamBuf& P, const std::string& pre, const AdaINResBlock1Weights& w, const char* where) {
    for (int i = 0; i < 3; ++i) {
        const std::string s = std::to_string(i);
        P.set(sub(pre, "convs1." + s + ".weight"), w.convs1[i].W, where);
        P.set(sub(pre, "convs1." + s + ".bias"), w.convs1[i].b, where);
        P.set(sub(pre, "convs2." + s + ".weight"), w.convs2[i].W, where);
        P.set(sub(pre, "convs2." + s + ".bias"), w.convs2[i].b, where);
        P.set(sub(pre, "adain1." + s + ".fc.weight"), w.adain1[i].fc.W, where);
        P.set(sub(pre, "adain1." + s + ".fc.bias"), w.adain1[i].fc.b, where);
        P.set(sub(pre, "adain2." + s + ".fc.weight"), w.adain2[i].fc.W, where);
        P.set(sub(pre, "adain2." + s + ".fc.bias"), w.adain2[i].fc.b, where);
        need(!w.alpha1[i].empty() && !w.alpha2[i].empty(), where, "Snake alphas are required");
        P.set(sub(pre, "alpha1." + s), w.alpha1[i], where);
        P.set(sub(pre, "alpha2." + s), w.alpha2[i], where);
    }
}

void fill_backbone(ParamBuf& P, const DecoderBackbone& bb, const char* where) {
    P.set("F0_conv.weight", bb.F0_conv.W, where);
    P.set("F0_conv.bias", bb.F0_conv.b, where);
    P.set("N_conv.weight", bb.N_conv.W, where);
    P.set("N_conv.bias", bb.N_conv.b, where);
    P.set("asr_res.0.weight", bb.asr_res.W, where);
    P.set("asr_res.0.bias", bb.asr_res.b, where);
    fill_block(P, "encode", bb.encode, where);
    for (size_t i = 0; i < bb.decode.size(); ++i) fill_block(P, "decode." + std::to_string(i), bb.decode[i], where);
}

void fill_generator(ParamBuf& P, const Generator& gen, const char* where) {
    for (int i = 0; i < gen.num_upsamples; ++i) {
        const std::string s = std::to_string(i);
        P.set("generator.ups." + s + ".weight", gen.ups_W[i], where);
        P.set("generator.ups." + s + ".bias", gen.ups_b[i], where);
        P.set("generator.noise_convs." + s + ".weight", gen.noise_convs[i].W, where);
        P.set("generator.noise_convs." + s + ".bias", gen.noise_convs[i].b, where);
        fill_rb1(P, "generator.noise_res." + s, gen.noise_res[i], where);
    }
    for (size_t k = 0; k < gen.resblocks.size(); ++k)
        fill_rb1(P, "generator.resblocks." + std::to_string(k), gen.resblocks[k], where);
    P.set("generator.conv_post.weight", gen.conv_post.W, where);
    P.set("generator.conv_post.bias", gen.conv_post.b, where);
}

}  // namespace refapi
}  // namespace brosoundml
