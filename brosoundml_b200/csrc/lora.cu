// DecoderLora kernels and host side (see lora.h). The reference runs one clip
// at a time through brotensor's lora_forward / lora_backward; here every adapter
// of every clip is one row of a few batched kernels:
//   h_ab  = A_a s_b                       (rank)
//   y_ab  = W_a s_b + bias_a + scale * B_a (g_b * h_ab)   -> the AdaIN's (gamma ; beta)
// and, from the engine's dY_ab = d(gamma ; beta):
//   dB_a += scale * sum_b dY_ab (g_b * h_ab)^T
//   dhg_ab = scale * B_a^T dY_ab ;  dA_a += sum_b (dhg_ab * g_b) s_b^T ;  dG_b = sum_a dhg_ab * h_ab
// and the gate g_b = W2 tanh(W1 v_b) with its backward (decoder_lora.cpp:30-78).
#include "lora.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "kernels.h"

namespace bsml {

namespace {

constexpr int kMaxRank = 32;   // one warp lane per LoRA rank

__device__ __forceinline__ float warp_sum(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// g_b = W2 tanh(W1 v_b); act_b kept for the backward. One CTA per clip.
__global__ void gate_fwd_kernel(const float* W1, const float* W2, const float* cond, int in_dim, int hidden,
                                int rank, float* act, float* g) {
    __shared__ float a[64];
    const int b = blockIdx.x, t = threadIdx.x;
    if (t < hidden) {
        float s = 0.f;
        for (int i = 0; i < in_dim; ++i) s = fmaf(W1[t * in_dim + i], cond[b * in_dim + i], s);
        a[t] = tanhf(s);
        act[b * hidden + t] = a[t];
    }
    __syncthreads();
    if (t < rank) {
        float s = 0.f;
        for (int j = 0; j < hidden; ++j) s = fmaf(W2[t * hidden + j], a[j], s);
        g[b * rank + t] = s;
    }
}

// h[a][b][r] = A_a[r] . s_b  (one warp per (a, b, r))
__global__ void lora_h_kernel(const LoraAd* ads, int n_ad, int B, int rank, int S, const float* P,
                              const float* style, float* h) {
    const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (w >= n_ad * B * rank) return;
    const int r = w % rank, b = (w / rank) % B, a = w / (rank * B);
    const float* A = P + ads[a].offA + (int64_t)r * S;
    float s = 0.f;
    for (int i = lane; i < S; i += 32) s = fmaf(A[i], style[(int64_t)b * S + i], s);
    s = warp_sum(s);
    if (lane == 0) h[w] = s;
}

// aff[B*aff_base + b*2C + o] = W[o] . s_b + bias[o] + scale * sum_r B[o][r] g_b[r] h_ab[r]  (warp per row)
__global__ void lora_aff_kernel(const LoraAd* ads, const int* row_ad, int total_rows, int B, int rank, int S,
                                float scale, const float* base, const float* P, const float* style, const float* g,
                                const float* h, float* aff) {
    const int q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (q >= total_rows) return;
    const int a = row_ad[q];
    const LoraAd ad = ads[a];
    const int o = q - (int)(ad.aff_base);   // rows of adapter a start at its per-clip offset
    const float* W = base + ad.fw + (int64_t)o * S;
    const float bo = base[ad.fb + o];
    const float Bv = lane < rank ? P[ad.offB + (int64_t)o * rank + lane] : 0.f;
    for (int b = 0; b < B; ++b) {
        float s = 0.f;
        for (int i = lane; i < S; i += 32) s = fmaf(W[i], style[(int64_t)b * S + i], s);
        float d = lane < rank ? Bv * g[b * rank + lane] * h[((int64_t)a * B + b) * rank + lane] : 0.f;
        s = warp_sum(s);
        d = warp_sum(d);
        if (lane == 0) aff[(int64_t)B * ad.aff_base + (int64_t)b * 2 * ad.C + o] = s + bo + scale * d;
    }
}

// dB (+)= scale * dY (g*h)^T per row; dhg[a][b][r] += scale * B[o][r] dY_b[o]. One CTA per
// (adapter, chunk of its rows); dhg partials combined in shared memory, one global atomic each.
__global__ void lora_bwd_rows_kernel(const LoraAd* ads, int B, int rank, float scale, const float* P, float* G,
                                     const float* g, const float* h, const float* daff, int rows_per, double* dhg) {
    extern __shared__ double sh[];   // [B][rank]
    const int a = blockIdx.x;
    const LoraAd ad = ads[a];
    for (int i = threadIdx.x; i < B * rank; i += blockDim.x) sh[i] = 0.0;
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int o0 = blockIdx.y * rows_per, o1 = min(2 * ad.C, o0 + rows_per);
    for (int o = o0 + warp; o < o1; o += nw) {
        const float Bv = lane < rank ? P[ad.offB + (int64_t)o * rank + lane] : 0.f;
        double dBacc = 0.0;
        for (int b = 0; b < B; ++b) {
            const float dy = daff[(int64_t)B * ad.aff_base + (int64_t)b * 2 * ad.C + o];
            if (lane < rank) {
                const float hg = g[b * rank + lane] * h[((int64_t)a * B + b) * rank + lane];
                dBacc += (double)dy * hg;
                atomicAdd(&sh[b * rank + lane], (double)scale * Bv * dy);
            }
        }
        if (lane < rank) G[ad.offB + (int64_t)o * rank + lane] += (float)(scale * dBacc);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < B * rank; i += blockDim.x) atomicAdd(&dhg[(int64_t)a * B * rank + i], sh[i]);
}

// dA[a][r][s] += sum_b dhg[a][b][r] g_b[r] s_b[s]
__global__ void lora_bwd_A_kernel(const LoraAd* ads, int n_ad, int B, int rank, int S, float* G, const float* g,
                                  const float* style, const double* dhg) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (i >= (int64_t)n_ad * rank * S) return;
    const int s = (int)(i % S), r = (int)((i / S) % rank), a = (int)(i / ((int64_t)S * rank));
    double acc = 0.0;
    for (int b = 0; b < B; ++b)
        acc += dhg[((int64_t)a * B + b) * rank + r] * g[b * rank + r] * style[(int64_t)b * S + s];
    G[ads[a].offA + (int64_t)r * S + s] += (float)acc;
}

// dG[b][r] = sum_a dhg[a][b][r] h[a][b][r]
__global__ void lora_dG_kernel(int n_ad, int B, int rank, const float* h, const double* dhg, float* dG) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * rank) return;
    double acc = 0.0;
    for (int a = 0; a < n_ad; ++a) acc += dhg[(int64_t)a * B * rank + i] * h[(int64_t)a * B * rank + i];
    dG[i] = (float)acc;
}

// Gate backward over all clips: dW2 += dG act^T ; dPre1 = (W2^T dG) (1 - act^2) ; dW1 += dPre1 v^T.
__global__ void gate_bwd_kernel(const float* W2, float* dW1, float* dW2, const float* cond, const float* act,
                                const float* dG, int B, int in_dim, int hidden, int rank) {
    const int t = threadIdx.x;
    if (t < rank * hidden) {
        const int r = t / hidden, j = t % hidden;
        double acc = 0.0;
        for (int b = 0; b < B; ++b) acc += (double)dG[b * rank + r] * act[b * hidden + j];
        dW2[t] += (float)acc;
    }
    if (t < hidden * in_dim) {
        const int j = t / in_dim, i = t % in_dim;
        double acc = 0.0;
        for (int b = 0; b < B; ++b) {
            float da = 0.f;
            for (int r = 0; r < rank; ++r) da = fmaf(W2[r * hidden + j], dG[b * rank + r], da);
            const float ab = act[b * hidden + j];
            acc += (double)(da * (1.f - ab * ab)) * cond[b * in_dim + i];
        }
        dW1[t] += (float)acc;
    }
}

// splitmix64 stream -> xavier-uniform U(-a, a), a = sqrt(6 / (fan_in + fan_out))
struct Rng {
    uint64_t s;
    uint64_t next() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    float uniform() { return (float)((next() >> 40) * (1.0 / 16777216.0)); }   // [0, 1)
};
void xavier(std::vector<float>& h, int64_t off, int rows, int cols, Rng& rng) {
    const float a = std::sqrt(6.f / (float)(rows + cols));
    for (int64_t i = 0; i < (int64_t)rows * cols; ++i) h[off + i] = (2.f * rng.uniform() - 1.f) * a;
}

template <class T>
T* dalloc(int64_t n) {
    T* p = nullptr;
    BSML_CUDA(cudaMalloc(&p, sizeof(T) * std::max<int64_t>(n, 1)));
    return p;
}

}  // namespace

void gate_forward(const float* W1, const float* W2, const float* v, int B, int in_dim, int hidden, int gate_dim,
                  float* act, float* g, cudaStream_t st) {
    if (hidden > 64 || gate_dim > 64) fail("bsml_gate_forward", "hidden and gate widths above 64 are not supported");
    ::bsml::count_launch();
    gate_fwd_kernel<<<B, 64, 0, st>>>(W1, W2, v, in_dim, hidden, gate_dim, act, g);
    BSML_LAUNCH("gate_fwd");
}

void gate_backward(const float* W2, const float* v, const float* act, const float* dG, int B, int in_dim,
                   int hidden, int gate_dim, float* dW1, float* dW2, cudaStream_t st) {
    if (gate_dim * hidden > 512 || hidden * in_dim > 512)
        fail("bsml_gate_backward", "gate weights above 512 elements are not supported");
    ::bsml::count_launch();
    gate_bwd_kernel<<<1, 512, 0, st>>>(W2, dW1, dW2, v, act, dG, B, in_dim, hidden, gate_dim);
    BSML_LAUNCH("gate_bwd");
}

Lora::Lora(Engine& eng, int rank, float scale, uint64_t seed) : eng_(eng), rank_(rank), scale_(scale) {
    if (rank < 1 || rank > kMaxRank) fail("bsml_lora_create", "rank must be in 1..32");
    BSML_CUDA(cudaGetDevice(&device_));
    const Layout& L = eng.layout();
    S_ = L.cfg.style_dim;
    aff_per_clip_ = L.aff_per_clip;
    int64_t off = off_W2() + (int64_t)rank * kHidden;
    for (const AdaP* p : L.adains) {
        LoraAd a{};
        a.fw = p->fw; a.fb = p->fb; a.C = p->C;
        a.aff_base = L.aff_base[p->idx];
        a.offA = off; off += (int64_t)rank * S_;
        a.offB = off; off += (int64_t)2 * p->C * rank;
        ads_.push_back(a);
    }
    n_params_ = off;
    total_rows_ = (int)aff_per_clip_;
    // initial values (DecoderLora::make, decoder_lora.cpp:115-147): gate W1 and every A, B
    // xavier-uniform from the seeded stream, gate W2 zero (g(v) = 0: the base decoder)
    std::vector<float> h(n_params_, 0.f);
    Rng rng{seed ? seed : 0xD1B54A32D192ED03ull};
    for (const LoraAd& a : ads_) {
        xavier(h, a.offA, rank, S_, rng);
        xavier(h, a.offB, 2 * a.C, rank, rng);
    }
    Rng grng{(seed ? seed : 0xD1B54A32D192ED03ull) ^ 0xABCDEFull};
    xavier(h, off_W1(), kHidden, kInDim, grng);
    P_ = dalloc<float>(n_params_);
    G_ = dalloc<float>(n_params_);
    M_ = dalloc<float>(n_params_);
    V_ = dalloc<float>(n_params_);
    BSML_CUDA(cudaMemcpy(P_, h.data(), sizeof(float) * n_params_, cudaMemcpyHostToDevice));
    BSML_CUDA(cudaMemset(G_, 0, sizeof(float) * n_params_));
    BSML_CUDA(cudaMemset(M_, 0, sizeof(float) * n_params_));
    BSML_CUDA(cudaMemset(V_, 0, sizeof(float) * n_params_));
    d_ads_ = dalloc<LoraAd>((int64_t)ads_.size());
    BSML_CUDA(cudaMemcpy(d_ads_, ads_.data(), sizeof(LoraAd) * ads_.size(), cudaMemcpyHostToDevice));
    std::vector<int> ra(total_rows_);
    for (size_t a = 0; a < ads_.size(); ++a)
        for (int o = 0; o < 2 * ads_[a].C; ++o) ra[ads_[a].aff_base + o] = (int)a;
    d_row_ad_ = dalloc<int>(total_rows_);
    BSML_CUDA(cudaMemcpy(d_row_ad_, ra.data(), sizeof(int) * total_rows_, cudaMemcpyHostToDevice));
}

Lora::~Lora() {
    cudaSetDevice(device_);
    for (void* p : {(void*)P_, (void*)G_, (void*)M_, (void*)V_, (void*)d_ads_, (void*)d_row_ad_, (void*)style_,
                    (void*)cond_, (void*)act_, (void*)g_, (void*)h_, (void*)dG_, (void*)aff_, (void*)daff_,
                    (void*)dhg_})
        cudaFree(p);
}

void Lora::ensure_batch(int B) {
    if (B <= B_cap_) return;
    for (void* p : {(void*)style_, (void*)cond_, (void*)act_, (void*)g_, (void*)h_, (void*)dG_, (void*)aff_,
                    (void*)daff_, (void*)dhg_})
        if (p) BSML_CUDA(cudaFree(p));
    const int64_t n_ad = (int64_t)ads_.size();
    style_ = dalloc<float>((int64_t)B * S_);
    cond_ = dalloc<float>((int64_t)B * kInDim);
    act_ = dalloc<float>((int64_t)B * kHidden);
    g_ = dalloc<float>((int64_t)B * rank_);
    h_ = dalloc<float>(n_ad * B * rank_);
    dG_ = dalloc<float>((int64_t)B * rank_);
    aff_ = dalloc<float>((int64_t)B * aff_per_clip_);
    daff_ = dalloc<float>((int64_t)B * aff_per_clip_);
    dhg_ = dalloc<double>(n_ad * B * rank_);
    B_cap_ = B;
}

void Lora::forward(int B, int T, const float* params, const float* asr, const float* F0, const float* N,
                   const float* ref_s, int ref_stride, const float* har, int frames, const float* cond, float* audio,
                   cudaStream_t st) {
    if (B < 1 || T < 1) fail("bsml_lora_forward", "B and T must be positive");
    if (!params || !ref_s || !cond) fail("bsml_lora_forward", "null input");
    if (ref_stride < S_) fail("bsml_lora_forward", "ref_s row stride below the style width");
    BSML_CUDA(cudaSetDevice(device_));
    ensure_batch(B);
    B_ = B;
    fwd_done_ = false;
    // style = ref_s[:, :S] (decoder_lora.cpp:214-215), condition kept for the backward
    BSML_CUDA(cudaMemcpy2DAsync(style_, sizeof(float) * S_, ref_s, sizeof(float) * ref_stride, sizeof(float) * S_,
                                B, cudaMemcpyDeviceToDevice, st));
    BSML_CUDA(cudaMemcpyAsync(cond_, cond, sizeof(float) * B * kInDim, cudaMemcpyDeviceToDevice, st));
    const int n_ad = (int)ads_.size();
    ::bsml::count_launch();
    gate_fwd_kernel<<<B, 64, 0, st>>>(P_ + off_W1(), P_ + off_W2(), cond_, kInDim, kHidden, rank_, act_, g_);
    BSML_LAUNCH("lora_gate_fwd");
    const int64_t hw = (int64_t)n_ad * B * rank_ * 32;
    ::bsml::count_launch();
    lora_h_kernel<<<(unsigned)ceil_div(hw, 256), 256, 0, st>>>(d_ads_, n_ad, B, rank_, S_, P_, style_, h_);
    BSML_LAUNCH("lora_h");
    ::bsml::count_launch();
    lora_aff_kernel<<<(unsigned)ceil_div((int64_t)total_rows_ * 32, 256), 256, 0, st>>>(
        d_ads_, d_row_ad_, total_rows_, B, rank_, S_, scale_, params, P_, style_, g_, h_, aff_);
    BSML_LAUNCH("lora_aff");
    eng_.forward(B, T, params, asr, F0, N, /*style=*/nullptr, har, frames, aff_, audio, nullptr, st);
    fwd_done_ = true;
}

void Lora::backward(const float* daudio, cudaStream_t st) {
    if (!fwd_done_) fail("bsml_lora_backward", "no matching forward");
    BSML_CUDA(cudaSetDevice(device_));
    const int B = B_, n_ad = (int)ads_.size();
    // decoder backward with frozen weights: only the affine gradients
    eng_.backward(daudio, /*grads=*/nullptr, nullptr, nullptr, daff_, st);
    BSML_CUDA(cudaMemsetAsync(dhg_, 0, sizeof(double) * n_ad * B * rank_, st));
    const int rows_per = 256;
    int max_rows = 0;
    for (const LoraAd& a : ads_) max_rows = std::max(max_rows, 2 * a.C);
    dim3 grid((unsigned)n_ad, (unsigned)ceil_div(max_rows, rows_per));
    ::bsml::count_launch();
    lora_bwd_rows_kernel<<<grid, 256, sizeof(double) * B * rank_, st>>>(d_ads_, B, rank_, scale_, P_, G_, g_, h_,
                                                                        daff_, rows_per, dhg_);
    BSML_LAUNCH("lora_bwd_rows");
    ::bsml::count_launch();
    lora_bwd_A_kernel<<<(unsigned)ceil_div((int64_t)n_ad * rank_ * S_, 256), 256, 0, st>>>(d_ads_, n_ad, B, rank_,
                                                                                             S_, G_, g_, style_, dhg_);
    BSML_LAUNCH("lora_bwd_A");
    ::bsml::count_launch();
    lora_dG_kernel<<<(unsigned)ceil_div(B * rank_, 128), 128, 0, st>>>(n_ad, B, rank_, h_, dhg_, dG_);
    BSML_LAUNCH("lora_dG");
    ::bsml::count_launch();
    gate_bwd_kernel<<<1, 512, 0, st>>>(P_ + off_W2(), G_ + off_W1(), G_ + off_W2(), cond_, act_, dG_, B, kInDim,
                                       kHidden, rank_);
    BSML_LAUNCH("lora_gate_bwd");
}

void Lora::zero_grad(cudaStream_t st) {
    BSML_CUDA(cudaSetDevice(device_));
    BSML_CUDA(cudaMemsetAsync(G_, 0, sizeof(float) * n_params_, st));
}

void Lora::adam_step(float lr, float b1, float b2, float eps, cudaStream_t st) {
    BSML_CUDA(cudaSetDevice(device_));
    ++step_;   // one shared step for every tensor (decoder_lora.cpp:306-314)
    adam(P_, G_, M_, V_, n_params_, lr, b1, b2, eps, step_, st);
}

// ── ELRA1: "ELRA1\0\0\0", int32 rank, int32 style_dim, float scale, int32 gate hidden,
// tensor W1, tensor W2, then per adapter: int32 C, tensor A, tensor B; a tensor is
// int32 rows, int32 cols, rows*cols float32 row-major; all little-endian.
namespace {
constexpr char kMagic[8] = {'E', 'L', 'R', 'A', '1', 0, 0, 0};

struct File {
    std::FILE* f;
    ~File() { if (f) std::fclose(f); }
};
void put_i32(std::FILE* f, int32_t v) { std::fwrite(&v, 4, 1, f); }
void put_tensor(std::FILE* f, const float* h, int rows, int cols) {
    put_i32(f, rows);
    put_i32(f, cols);
    std::fwrite(h, sizeof(float), (size_t)rows * cols, f);
}
int32_t get_i32(std::FILE* f, const char* what) {
    int32_t v = 0;
    if (std::fread(&v, 4, 1, f) != 1) fail("DecoderLora::load", std::string("truncated ") + what);
    return v;
}
void get_tensor(std::FILE* f, float* h, int rows, int cols) {
    const int32_t r = get_i32(f, "tensor header"), c = get_i32(f, "tensor header");
    if (r != rows || c != cols)
        fail("DecoderLora::load", "tensor shape " + std::to_string(r) + "x" + std::to_string(c) + " where " +
                                      std::to_string(rows) + "x" + std::to_string(cols) + " is expected");
    if (std::fread(h, sizeof(float), (size_t)rows * cols, f) != (size_t)rows * cols)
        fail("DecoderLora::load", "truncated tensor data");
}
}  // namespace

namespace {
constexpr char kStateMagic[8] = {'E', 'L', 'R', 'S', 'T', 'A', 'T', 'E'};
}

void Lora::save(const std::string& path, bool full_state) const {
    BSML_CUDA(cudaSetDevice(device_));
    std::vector<float> h(n_params_);
    BSML_CUDA(cudaDeviceSynchronize());
    BSML_CUDA(cudaMemcpy(h.data(), P_, sizeof(float) * n_params_, cudaMemcpyDeviceToHost));
    File fh{std::fopen(path.c_str(), "wb")};
    if (!fh.f) fail("DecoderLora::save", "cannot open " + path);
    std::fwrite(kMagic, 1, 8, fh.f);
    put_i32(fh.f, rank_);
    put_i32(fh.f, S_);
    std::fwrite(&scale_, sizeof(float), 1, fh.f);
    put_i32(fh.f, kHidden);
    put_tensor(fh.f, h.data() + off_W1(), kHidden, kInDim);
    put_tensor(fh.f, h.data() + off_W2(), rank_, kHidden);
    for (const LoraAd& a : ads_) {
        put_i32(fh.f, a.C);
        put_tensor(fh.f, h.data() + a.offA, rank_, S_);
        put_tensor(fh.f, h.data() + a.offB, 2 * a.C, rank_);
    }
    if (full_state) {
        // optimiser state after the ELRA1 body (a reader of the plain format stops
        // before it): magic, step, n, then Adam's first and second moments in the
        // same order as the parameters above
        std::vector<float> m(n_params_), v(n_params_);
        BSML_CUDA(cudaMemcpy(m.data(), M_, sizeof(float) * n_params_, cudaMemcpyDeviceToHost));
        BSML_CUDA(cudaMemcpy(v.data(), V_, sizeof(float) * n_params_, cudaMemcpyDeviceToHost));
        std::fwrite(kStateMagic, 1, 8, fh.f);
        put_i32(fh.f, step_);
        const int64_t n = n_params_;
        std::fwrite(&n, sizeof(n), 1, fh.f);
        std::fwrite(m.data(), sizeof(float), m.size(), fh.f);
        std::fwrite(v.data(), sizeof(float), v.size(), fh.f);
    }
    if (std::ferror(fh.f)) fail("DecoderLora::save", "write error on " + path);
}

void Lora::load(const std::string& path, bool full_state) {
    BSML_CUDA(cudaSetDevice(device_));
    File fh{std::fopen(path.c_str(), "rb")};
    if (!fh.f) fail("DecoderLora::load", "cannot open " + path);
    char magic[8];
    if (std::fread(magic, 1, 8, fh.f) != 8 || std::memcmp(magic, kMagic, 8) != 0)
        fail("DecoderLora::load", "bad magic in " + path);
    const int32_t rank = get_i32(fh.f, "header"), sd = get_i32(fh.f, "header");
    float scale = 0.f;
    if (std::fread(&scale, sizeof(float), 1, fh.f) != 1) fail("DecoderLora::load", "truncated header");
    const int32_t gh = get_i32(fh.f, "header");
    if (rank != rank_ || sd != S_ || gh != kHidden) fail("DecoderLora::load", "architecture mismatch");
    std::vector<float> h(n_params_);
    get_tensor(fh.f, h.data() + off_W1(), kHidden, kInDim);
    get_tensor(fh.f, h.data() + off_W2(), rank_, kHidden);
    for (const LoraAd& a : ads_) {
        if (get_i32(fh.f, "adapter header") != a.C) fail("DecoderLora::load", "architecture mismatch");
        get_tensor(fh.f, h.data() + a.offA, rank_, S_);
        get_tensor(fh.f, h.data() + a.offB, 2 * a.C, rank_);
    }
    std::vector<float> m, v;
    int32_t step = 0;
    if (full_state) {
        char sm[8];
        if (std::fread(sm, 1, 8, fh.f) != 8 || std::memcmp(sm, kStateMagic, 8) != 0)
            fail("DecoderLora::load", "no optimiser state in " + path);
        step = get_i32(fh.f, "state header");
        int64_t n = 0;
        if (std::fread(&n, sizeof(n), 1, fh.f) != 1) fail("DecoderLora::load", "truncated state header");
        if (n != n_params_ || step < 0) fail("DecoderLora::load", "architecture mismatch");
        m.resize(n_params_);
        v.resize(n_params_);
        if (std::fread(m.data(), sizeof(float), m.size(), fh.f) != m.size() ||
            std::fread(v.data(), sizeof(float), v.size(), fh.f) != v.size())
            fail("DecoderLora::load", "truncated optimiser state");
    }
    BSML_CUDA(cudaDeviceSynchronize());
    BSML_CUDA(cudaMemcpy(P_, h.data(), sizeof(float) * n_params_, cudaMemcpyHostToDevice));
    if (full_state) {
        BSML_CUDA(cudaMemcpy(M_, m.data(), sizeof(float) * n_params_, cudaMemcpyHostToDevice));
        BSML_CUDA(cudaMemcpy(V_, v.data(), sizeof(float) * n_params_, cudaMemcpyHostToDevice));
        step_ = step;
    }
    scale_ = scale;
}

}  // namespace bsml
