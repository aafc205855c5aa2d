// Conv-weight LoRA kernels and host side (see convlora.h).
#include "convlora.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "kernels.h"

namespace bsml {

namespace {

// eff[w + i*cols + c] = base[...] + scale * sum_r B[i][r] A[r][c]   (blockIdx.y = weight)
__global__ void fold_kernel(const ConvLoraW* ws, int rank, float scale, const float* P, const float* base,
                            float* eff) {
    const ConvLoraW W = ws[blockIdx.y];
    const int64_t n = (int64_t)W.rows * W.cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / W.cols), col = (int)(i - (int64_t)row * W.cols);
        float d = 0.f;
        for (int r = 0; r < rank; ++r)
            d = fmaf(P[W.offB + (int64_t)row * rank + r], P[W.offA + (int64_t)r * W.cols + col], d);
        eff[W.w + i] = fmaf(scale, d, base[W.w + i]);
    }
}

// dB[i][r] += scale * dW[i][:] . A[r][:]   (one warp per (weight, row, r); blockIdx.y = weight)
__global__ void dB_kernel(const ConvLoraW* ws, int rank, float scale, const float* P, const float* dW, float* G) {
    const ConvLoraW W = ws[blockIdx.y];
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= W.rows * rank) return;
    const int row = warp / rank, r = warp - row * rank;
    const float* g = dW + W.w + (int64_t)row * W.cols;
    const float* a = P + W.offA + (int64_t)r * W.cols;
    double s = 0.0;
    for (int c = lane; c < W.cols; c += 32) s += (double)g[c] * a[c];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) G[W.offB + (int64_t)row * rank + r] += (float)(scale * s);
}

// dA[r][c] += scale * sum_i B[i][r] dW[i][c]   (one thread per (r, c); blockIdx.y = weight)
__global__ void dA_kernel(const ConvLoraW* ws, int rank, float scale, const float* P, const float* dW, float* G) {
    const ConvLoraW W = ws[blockIdx.y];
    const int64_t n = (int64_t)rank * W.cols;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int r = (int)(i / W.cols), c = (int)(i - (int64_t)r * W.cols);
        double s = 0.0;
        for (int row = 0; row < W.rows; ++row)
            s += (double)P[W.offB + (int64_t)row * rank + r] * dW[W.w + (int64_t)row * W.cols + c];
        G[W.offA + i] += (float)(scale * s);
    }
}

}  // namespace

ConvLora::ConvLora(Engine& eng, int rank, float scale, uint64_t seed) : eng_(eng), rank_(rank), scale_(scale) {
    if (rank < 1 || rank > 64) fail("bsml_convlora_create", "rank must be in 1..64");
    BSML_CUDA(cudaGetDevice(&device_));
    const Layout& L = eng.layout();
    n_dec_ = L.total;
    int64_t off = 0;
    for (const bsml_param_entry& e : L.table) {
        const std::string name(e.name);
        if (e.ndim != 3 || name.size() < 7 || name.compare(name.size() - 7, 7, ".weight") != 0) continue;
        ConvLoraW w{};
        w.w = e.offset;
        w.rows = e.shape[0];
        w.cols = e.shape[1] * e.shape[2];
        w.offA = off; off += (int64_t)rank * w.cols;
        w.offB = off; off += (int64_t)w.rows * rank;
        ws_.push_back(w);
    }
    n_params_ = off;
    // A ~ N(0, 0.01) from a seeded splitmix64 stream (Box-Muller), B = 0: the adapted
    // decoder starts as the base decoder
    std::vector<float> h(n_params_, 0.f);
    uint64_t s = seed ? seed : 0x5EEDC0DEull;
    auto next = [&]() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    auto unif = [&]() { return ((next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); };   // (0, 1)
    for (const ConvLoraW& w : ws_)
        for (int64_t i = 0; i < (int64_t)rank * w.cols; ++i)
            h[w.offA + i] = (float)(0.01 * std::sqrt(-2.0 * std::log(unif())) * std::cos(6.283185307179586 * unif()));
    auto dalloc = [](int64_t n) {
        float* p = nullptr;
        BSML_CUDA(cudaMalloc(&p, sizeof(float) * std::max<int64_t>(n, 1)));
        return p;
    };
    P_ = dalloc(n_params_);
    G_ = dalloc(n_params_);
    M_ = dalloc(n_params_);
    V_ = dalloc(n_params_);
    eff_ = dalloc(n_dec_);
    dgrad_ = dalloc(n_dec_);
    BSML_CUDA(cudaMemcpy(P_, h.data(), sizeof(float) * n_params_, cudaMemcpyHostToDevice));
    BSML_CUDA(cudaMemset(G_, 0, sizeof(float) * n_params_));
    BSML_CUDA(cudaMemset(M_, 0, sizeof(float) * n_params_));
    BSML_CUDA(cudaMemset(V_, 0, sizeof(float) * n_params_));
    BSML_CUDA(cudaMalloc(&d_ws_, sizeof(ConvLoraW) * std::max<size_t>(ws_.size(), 1)));
    BSML_CUDA(cudaMemcpy(d_ws_, ws_.data(), sizeof(ConvLoraW) * ws_.size(), cudaMemcpyHostToDevice));
}

ConvLora::~ConvLora() {
    cudaSetDevice(device_);
    for (void* p : {(void*)P_, (void*)G_, (void*)M_, (void*)V_, (void*)eff_, (void*)dgrad_, (void*)d_ws_}) cudaFree(p);
}

void ConvLora::forward(int B, int T, const float* base, const float* asr, const float* F0, const float* N,
                       const float* style, const float* har, int frames, float* audio, cudaStream_t st) {
    if (!base) fail("bsml_convlora_forward", "null parameters");
    BSML_CUDA(cudaSetDevice(device_));
    fwd_done_ = false;
    BSML_CUDA(cudaMemcpyAsync(eff_, base, sizeof(float) * n_dec_, cudaMemcpyDeviceToDevice, st));
    ::bsml::count_launch();
    fold_kernel<<<dim3(256, (unsigned)ws_.size()), 256, 0, st>>>(d_ws_, rank_, scale_, P_, base, eff_);
    BSML_LAUNCH("convlora_fold");
    eng_.forward(B, T, eff_, asr, F0, N, style, har, frames, nullptr, audio, nullptr, st);
    fwd_done_ = true;
}

void ConvLora::backward(const float* daudio, cudaStream_t st) {
    if (!fwd_done_) fail("bsml_convlora_backward", "no matching forward");
    BSML_CUDA(cudaSetDevice(device_));
    eng_.backward(daudio, dgrad_, nullptr, nullptr, nullptr, st);
    int max_rows = 0;
    for (const ConvLoraW& w : ws_) max_rows = std::max(max_rows, w.rows);
    ::bsml::count_launch();
    dB_kernel<<<dim3((unsigned)ceil_div((int64_t)max_rows * rank_ * 32, 256), (unsigned)ws_.size()), 256, 0, st>>>(
        d_ws_, rank_, scale_, P_, dgrad_, G_);
    BSML_LAUNCH("convlora_dB");
    ::bsml::count_launch();
    dA_kernel<<<dim3(64, (unsigned)ws_.size()), 256, 0, st>>>(d_ws_, rank_, scale_, P_, dgrad_, G_);
    BSML_LAUNCH("convlora_dA");
}

void ConvLora::zero_grad(cudaStream_t st) {
    BSML_CUDA(cudaSetDevice(device_));
    BSML_CUDA(cudaMemsetAsync(G_, 0, sizeof(float) * n_params_, st));
}

void ConvLora::adam_step(float lr, float b1, float b2, float eps, cudaStream_t st) {
    BSML_CUDA(cudaSetDevice(device_));
    ++step_;
    adam(P_, G_, M_, V_, n_params_, lr, b1, b2, eps, step_, st);
}

namespace {
constexpr char kConvMagic[8] = {'E', 'C', 'L', 'R', '1', 0, 0, 0};
struct CFile {
    std::FILE* f;
    ~CFile() {
        if (f) std::fclose(f);
    }
};
template <class T>
void put(std::FILE* f, T v) { std::fwrite(&v, sizeof(T), 1, f); }
template <class T>
T get(std::FILE* f) {
    T v{};
    if (std::fread(&v, sizeof(T), 1, f) != 1) fail("ConvLora::load", "truncated file");
    return v;
}
}  // namespace

void ConvLora::save(const std::string& path) const {
    BSML_CUDA(cudaSetDevice(device_));
    BSML_CUDA(cudaDeviceSynchronize());
    std::vector<float> p(n_params_), m(n_params_), v(n_params_);
    BSML_CUDA(cudaMemcpy(p.data(), P_, sizeof(float) * n_params_, cudaMemcpyDeviceToHost));
    BSML_CUDA(cudaMemcpy(m.data(), M_, sizeof(float) * n_params_, cudaMemcpyDeviceToHost));
    BSML_CUDA(cudaMemcpy(v.data(), V_, sizeof(float) * n_params_, cudaMemcpyDeviceToHost));
    CFile fh{std::fopen(path.c_str(), "wb")};
    if (!fh.f) fail("ConvLora::save", "cannot open " + path);
    std::fwrite(kConvMagic, 1, 8, fh.f);
    put<int32_t>(fh.f, rank_);
    put<float>(fh.f, scale_);
    put<int32_t>(fh.f, (int32_t)ws_.size());
    for (const ConvLoraW& w : ws_) {
        put<int64_t>(fh.f, w.w);
        put<int32_t>(fh.f, w.rows);
        put<int32_t>(fh.f, w.cols);
    }
    put<int32_t>(fh.f, step_);
    put<int64_t>(fh.f, n_params_);
    for (const auto* a : {&p, &m, &v}) std::fwrite(a->data(), sizeof(float), a->size(), fh.f);
    if (std::ferror(fh.f)) fail("ConvLora::save", "write error on " + path);
}

void ConvLora::load(const std::string& path) {
    BSML_CUDA(cudaSetDevice(device_));
    CFile fh{std::fopen(path.c_str(), "rb")};
    if (!fh.f) fail("ConvLora::load", "cannot open " + path);
    char magic[8];
    if (std::fread(magic, 1, 8, fh.f) != 8 || std::memcmp(magic, kConvMagic, 8) != 0)
        fail("ConvLora::load", "bad magic in " + path);
    const int32_t rank = get<int32_t>(fh.f);
    const float scale = get<float>(fh.f);
    const int32_t nw = get<int32_t>(fh.f);
    if (rank != rank_ || nw != (int32_t)ws_.size()) fail("ConvLora::load", "architecture mismatch");
    for (const ConvLoraW& w : ws_) {
        const int64_t off = get<int64_t>(fh.f);
        const int32_t r = get<int32_t>(fh.f), c = get<int32_t>(fh.f);
        if (off != w.w || r != w.rows || c != w.cols) fail("ConvLora::load", "architecture mismatch");
    }
    const int32_t step = get<int32_t>(fh.f);
    const int64_t n = get<int64_t>(fh.f);
    if (n != n_params_ || step < 0) fail("ConvLora::load", "architecture mismatch");
    std::vector<float> p(n_params_), m(n_params_), v(n_params_);
    for (auto* a : {&p, &m, &v})
        if (std::fread(a->data(), sizeof(float), a->size(), fh.f) != a->size())
            fail("ConvLora::load", "truncated data");
    BSML_CUDA(cudaDeviceSynchronize());
    BSML_CUDA(cudaMemcpy(P_, p.data(), sizeof(float) * n_params_, cudaMemcpyHostToDevice));
    BSML_CUDA(cudaMemcpy(M_, m.data(), sizeof(float) * n_params_, cudaMemcpyHostToDevice));
    BSML_CUDA(cudaMemcpy(V_, v.data(), sizeof(float) * n_params_, cudaMemcpyHostToDevice));
    step_ = step;
    scale_ = scale;
}

}  // namespace bsml
