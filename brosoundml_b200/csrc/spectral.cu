// Spectral head (polar exp/sin + iSTFT and their adjoints), the harmonic
// source (phase scan + sines + STFT), the L1 loss and Adam.
#include <cmath>

#include "kernels.h"

namespace bsml {

namespace {

inline int grid_for(int64_t n, int threads = 256) {
    int64_t g = ceil_div(n, threads);
    if (g > 148 * 32) g = 148 * 32;
    return (int)(g < 1 ? 1 : g);
}

constexpr int MAX_NFFT = 64;

// Per-block tables: irfft basis (c_k/N cos, -c_k/N sin), analysis basis (cos, sin),
// periodic Hann window in the reference's float arithmetic
// (kokoro_decoder_backward.cpp:581-588).
struct Tables {
    float cb[MAX_NFFT / 2 + 1][MAX_NFFT];
    float sb[MAX_NFFT / 2 + 1][MAX_NFFT];
    float w[MAX_NFFT];
};

__device__ void build_tables(Tables& T, int N, bool synthesis) {
    const int nf = N / 2 + 1;
    for (int i = threadIdx.x; i < nf * N; i += blockDim.x) {
        const int k = i / N, m = i % N;
        double s, c;
        sincospi(2.0 * (double)((k * m) % N) / (double)N, &s, &c);
        if (synthesis) {
            const double ck = (k == 0 || 2 * k == N) ? 1.0 : 2.0;
            T.cb[k][m] = (float)(ck / N * c);
            T.sb[k][m] = (float)(-ck / N * s);
        } else {
            T.cb[k][m] = (float)c;
            T.sb[k][m] = (float)s;
        }
    }
    for (int m = threadIdx.x; m < N; m += blockDim.x) T.w[m] = 0.5f - 0.5f * cosf(6.28318530717958647692f * (float)m / (float)N);
    __syncthreads();
}

__global__ void polar_fwd_kernel(Act post, int nf, float* spec) {
    const int64_t n = (int64_t)post.B * post.L * nf;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int k = (int)(i % nf);
        const int64_t r = i / nf;
        const int l = (int)(r % post.L), b = (int)(r / post.L);
        const float* pr = post.row(b, l);
        const float mag = expf(pr[k]), ang = sinf(pr[nf + k]);
        float sa, ca;
        sincosf(ang, &sa, &ca);
        spec[r * 2 * nf + 2 * k] = mag * ca;
        spec[r * 2 * nf + 2 * k + 1] = mag * sa;
    }
}

// one thread per output sample: overlap-add of <= ceil(N/hop) windowed frames,
// divided by the window envelope (torch.istft, center=True, normalized=False).
__global__ void istft_fwd_kernel(const float* spec, int B, int L, int N, int hop, float* audio) {
    __shared__ Tables T;
    build_tables(T, N, true);
    const int nf = N / 2 + 1, pad = N / 2;
    const int S = hop * (L - 1);
    const int64_t n = (int64_t)B * S;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int s = (int)(i % S), b = (int)(i / S);
        const int f = s + pad;
        int t0 = f - (N - 1);
        t0 = t0 <= 0 ? 0 : (t0 + hop - 1) / hop;
        const int t1 = min(L - 1, f / hop);
        float v = 0.f, env = 0.f;
        for (int t = t0; t <= t1; ++t) {
            const int m = f - t * hop;
            const float* sp = spec + ((int64_t)b * L + t) * 2 * nf;
            float fr = 0.f;
            for (int k = 0; k < nf; ++k) fr += sp[2 * k] * T.cb[k][m] + sp[2 * k + 1] * T.sb[k][m];
            v += fr * T.w[m];
            env += T.w[m] * T.w[m];
        }
        audio[i] = v / env;
    }
}

// one thread per (b, frame): adjoint of istft_fwd_kernel. mode 0: writes dre/dim
// (B, nf, L) NCL. mode 1: applies the polar / exp / sin adjoint
// (kokoro_decoder_backward.cpp:428-449) and writes dpost (channels-last).
__global__ void istft_bwd_kernel(const float* daudio, int B, int L, int N, int hop, int mode, float* dre, float* dim,
                                 Act post, Act dpost) {
    __shared__ Tables T;
    build_tables(T, N, true);
    const int nf = N / 2 + 1, pad = N / 2;
    const int S = hop * (L - 1);
    const int64_t n = (int64_t)B * L;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i % L), b = (int)(i / L);
        float g[MAX_NFFT];
        for (int m = 0; m < N; ++m) {
            const int f = t * hop + m;
            const int s = f - pad;
            float gv = 0.f;
            if (s >= 0 && s < S) {
                int u0 = f - (N - 1);
                u0 = u0 <= 0 ? 0 : (u0 + hop - 1) / hop;
                const int u1 = min(L - 1, f / hop);
                float env = 0.f;
                for (int u = u0; u <= u1; ++u) {
                    const float wv = T.w[f - u * hop];
                    env += wv * wv;
                }
                gv = daudio[(int64_t)b * S + s] / env * T.w[m];
            }
            g[m] = gv;
        }
        for (int k = 0; k < nf; ++k) {
            float ar = 0.f, ai = 0.f;
            for (int m = 0; m < N; ++m) {
                ar += g[m] * T.cb[k][m];
                ai += g[m] * T.sb[k][m];
            }
            if (mode == 0) {
                dre[((int64_t)b * nf + k) * L + t] = ar;
                dim[((int64_t)b * nf + k) * L + t] = ai;
            } else {
                const float* pr = post.row(b, t);
                const float pm = pr[k], pp = pr[nf + k];
                const float mag = expf(pm), ang = sinf(pp);
                float sa, ca;
                sincosf(ang, &sa, &ca);
                const float dmag = ar * ca + ai * sa;
                const float dang = mag * (-ar * sa + ai * ca);
                float* dp = dpost.row(b, t);
                dp[k] = dmag * mag;
                dp[nf + k] = dang * cosf(pp);
            }
        }
    }
}

__global__ void ncl_pair_to_spec_kernel(const float* re, const float* im, int B, int nf, int L, float* spec) {
    const int64_t n = (int64_t)B * nf * L;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int l = (int)(i % L);
        const int64_t r = i / L;
        const int k = (int)(r % nf), b = (int)(r / nf);
        spec[((int64_t)b * L + l) * 2 * nf + 2 * k] = re[i];
        spec[((int64_t)b * L + l) * 2 * nf + 2 * k + 1] = im[i];
    }
}

// ── harmonic source (kokoro_modules.cpp:1574-1665)
//
// Two phase modes. PHASE_FP32_RUNNING (default) is the reference's own
// arithmetic (kokoro_modules.cpp:1601-1616): per harmonic an fp32 accumulator,
// per sample phase = fl(phase + omega) and, when it exceeds 2*pi (the float
// constant), one fp32 subtraction of it; omega = fl(fl(fl(2pi * (h+1)) * f0) / sr).
// Every rounding is pinned with the _rn intrinsics, so the phase sequence is the
// reference's bit for bit. The recurrence is serial: hs_phase32_kernel runs one
// thread per (clip, harmonic) through all samples and records the accumulator at
// each F0 frame start; hs_source32_kernel then replays one frame per thread from
// those starts (the same fp32 steps, so the same values) and forms the sines.
// PHASE_EXACT forms each frame's start phase exactly in double instead (an
// accurate sine source whose phase does not drift with clip length).
constexpr float kTwoPiF = 6.28318530717958647692f;
constexpr int MAX_HARM = 16;

__device__ __forceinline__ float hs_omega(int h, float f0, float sr) {
    return __fdiv_rn(__fmul_rn(__fmul_rn(kTwoPiF, (float)(h + 1)), f0), sr);
}
__device__ __forceinline__ float hs_step(float p, float om) {
    p = __fadd_rn(p, om);
    return p > kTwoPiF ? __fsub_rn(p, kTwoPiF) : p;
}

__global__ void hs_phase32_kernel(const float* F0, int B, int F, int scale, int H, float sr, float* start) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * H) return;
    const int b = i / H, h = i % H;
    float p = 0.f;
    for (int f = 0; f < F; ++f) {
        start[(int64_t)i * F + f] = p;
        const float om = hs_omega(h, F0[(int64_t)b * F + f], sr);
        int j = 0;
        for (; j + 4 <= scale; j += 4) {
            p = hs_step(p, om);
            p = hs_step(p, om);
            p = hs_step(p, om);
            p = hs_step(p, om);
        }
        for (; j < scale; ++j) p = hs_step(p, om);
    }
}

// one thread per (clip, frame): H running phases from the frame start, sine
// mixture -> l_linear -> tanh for the frame's samples
__global__ void hs_source32_kernel(const float* F0, int B, int F, int scale, int H, float sr, const float* start,
                                   const float* lw, const float* lb, float* src) {
    const int64_t n = (int64_t)B * F;
    const int64_t S = (int64_t)F * scale;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int b = (int)(i / F), f = (int)(i % F);
        const float f0 = F0[i];
        const float uv = f0 > 0.f ? 1.f : 0.f;
        float p[MAX_HARM], om[MAX_HARM], w[MAX_HARM];
#pragma unroll
        for (int h = 0; h < MAX_HARM; ++h) {
            p[h] = h < H ? start[((int64_t)b * H + h) * F + f] : 0.f;
            om[h] = h < H ? hs_omega(h, f0, sr) : 0.f;
            w[h] = h < H ? lw[h] : 0.f;
        }
        const float bias = lb[0];
        float* out = src + (int64_t)b * S + (int64_t)f * scale;
        for (int j = 0; j < scale; ++j) {
            float mf = 0.f;
#pragma unroll
            for (int h = 0; h < MAX_HARM; ++h)
                if (h < H) {
                    p[h] = hs_step(p[h], om[h]);
                    mf += w[h] * (sinf(p[h]) * 0.1f * uv);
                }
            out[j] = tanhf(mf + bias);
        }
    }
}

// PHASE_EXACT: phase at the start of every F0 frame, per (clip, harmonic), as the
// exact running sum of the per-sample float increments, reduced mod 2*pi in double.
__global__ void hs_phase_kernel(const float* F0, int B, int F, int scale, int H, float sr, double* start) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * H) return;
    const int b = i / H, h = i % H;
    const double two_pi = 6.283185307179586476925286766559;
    double acc = 0.0;
    for (int f = 0; f < F; ++f) {
        start[(int64_t)i * F + f] = acc;
        const float omega = hs_omega(h, F0[(int64_t)b * F + f], sr);
        acc = fmod(acc + (double)scale * (double)omega, two_pi);
    }
}

// PHASE_EXACT: sine mixture -> l_linear -> tanh, one thread per sample
__global__ void hs_source_kernel(const float* F0, int B, int F, int scale, int H, float sr, const double* start,
                                 const float* lw, const float* lb, float* src) {
    const int64_t S = (int64_t)F * scale;
    const int64_t n = (int64_t)B * S;
    const double two_pi = 6.283185307179586476925286766559;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i % S;
        const int b = (int)(i / S);
        const int f = (int)(t / scale);
        const int j = (int)(t - (int64_t)f * scale);
        const float f0 = F0[(int64_t)b * F + f];
        const float uv = f0 > 0.f ? 1.f : 0.f;
        float mf = 0.f;
        for (int h = 0; h < H; ++h) {
            const float omega = hs_omega(h, f0, sr);
            const double ph = fmod(start[((int64_t)b * H + h) * F + f] + (double)(j + 1) * (double)omega, two_pi);
            mf += lw[h] * (sinf((float)ph) * 0.1f * uv);
        }
        src[i] = tanhf(mf + lb[0]);
    }
}

// STFT (center, reflect pad N/2, periodic Hann) -> [|X| ; angle X], one thread per (b, frame)
__global__ void hs_stft_kernel(const float* src, int B, int S, int N, int hop, Act har) {
    __shared__ Tables T;
    build_tables(T, N, false);
    const int nf = N / 2 + 1, pad = N / 2;
    const int frames = har.L;
    const int64_t n = (int64_t)B * frames;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i % frames), b = (int)(i / frames);
        float v[MAX_NFFT];
        for (int m = 0; m < N; ++m) {
            int j = t * hop + m - pad;
            if (j < 0) j = -j;
            if (j >= S) j = 2 * (S - 1) - j;
            v[m] = T.w[m] * src[(int64_t)b * S + j];
        }
        float* hr = har.row(b, t);
        for (int k = 0; k < nf; ++k) {
            float xr = 0.f, xi = 0.f;
            for (int m = 0; m < N; ++m) {
                xr += v[m] * T.cb[k][m];
                xi -= v[m] * T.sb[k][m];
            }
            hr[k] = sqrtf(xr * xr + xi * xi);
            hr[nf + k] = atan2f(xi, xr);
        }
    }
}

__global__ void l1_kernel(const float* a, const float* t, int64_t n, float* da, double* acc) {
    __shared__ double red[256];
    double s = 0;
    const float inv = 1.f / (float)n;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float d = a[i] - t[i];
        s += fabsf(d);
        da[i] = d > 0.f ? inv : (d < 0.f ? -inv : 0.f);
    }
    red[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) atomicAdd(acc, red[0]);
}
__global__ void l1_final_kernel(const double* acc, int64_t n, float* loss) { *loss = (float)(*acc / (double)n); }
__global__ void zero1(double* p) { *p = 0.0; }

__global__ void adam_kernel(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2,
                            float eps, float bc1, float bc2) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float gi = g[i];
        const float mi = b1 * m[i] + (1.f - b1) * gi;
        const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
        m[i] = mi;
        v[i] = vi;
        p[i] -= lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    }
}

}  // namespace

void polar_fwd(const Act& post, int nf, float* spec, cudaStream_t st) {
    ::bsml::count_launch();
    polar_fwd_kernel<<<grid_for((int64_t)post.B * post.L * nf), 256, 0, st>>>(post, nf, spec);
    BSML_LAUNCH("polar_fwd");
}

void istft_fwd(const float* spec, int B, int L, int n_fft, int hop, float* audio, cudaStream_t st) {
    if (n_fft > MAX_NFFT) fail("istft", "n_fft above 64 is not supported");
    ::bsml::count_launch();
    istft_fwd_kernel<<<grid_for((int64_t)B * hop * (L - 1)), 256, 0, st>>>(spec, B, L, n_fft, hop, audio);
    BSML_LAUNCH("istft_fwd");
}

void istft_polar_bwd(const float* daudio, const Act& post, int n_fft, int hop, const Act& dpost, cudaStream_t st) {
    if (n_fft > MAX_NFFT) fail("istft", "n_fft above 64 is not supported");
    ::bsml::count_launch();
    istft_bwd_kernel<<<grid_for((int64_t)post.B * post.L, 128), 128, 0, st>>>(daudio, post.B, post.L, n_fft, hop, 1,
                                                                            nullptr, nullptr, post, dpost);
    BSML_LAUNCH("istft_polar_bwd");
}

void istft_bwd_ncl(const float* daudio, int B, int L, int n_fft, int hop, float* dre, float* dim, cudaStream_t st) {
    if (n_fft > MAX_NFFT) fail("istft", "n_fft above 64 is not supported");
    ::bsml::count_launch();
    istft_bwd_kernel<<<grid_for((int64_t)B * L, 128), 128, 0, st>>>(daudio, B, L, n_fft, hop, 0, dre, dim, Act{},
                                                                  Act{});
    BSML_LAUNCH("istft_bwd");
}

void istft_fwd_ncl(const float* re, const float* im, int B, int L, int n_fft, int hop, float* audio,
                   float* spec_scratch, cudaStream_t st) {
    const int nf = n_fft / 2 + 1;
    ::bsml::count_launch();
    ncl_pair_to_spec_kernel<<<grid_for((int64_t)B * nf * L), 256, 0, st>>>(re, im, B, nf, L, spec_scratch);
    istft_fwd(spec_scratch, B, L, n_fft, hop, audio, st);
}

void harmonic_source(const float* F0, int B, int F, int scale, int harmonic_num, int sample_rate, int n_fft, int hop,
                     const float* lw, const float* lb, double* phase_start, float* src, const Act& har,
                     cudaStream_t st, int phase_mode) {
    if (n_fft > MAX_NFFT) fail("harmonic_source", "n_fft above 64 is not supported");
    const int H = harmonic_num + 1;
    if (H > MAX_HARM) fail("harmonic_source", "harmonic_num above 15 is not supported");
    const int64_t S = (int64_t)F * scale;
    if (phase_mode == PHASE_EXACT) {
        ::bsml::count_launch();
        hs_phase_kernel<<<(unsigned)ceil_div(B * H, 64), 64, 0, st>>>(F0, B, F, scale, H, (float)sample_rate,
                                                                      phase_start);
        ::bsml::count_launch();
        hs_source_kernel<<<grid_for(B * S), 256, 0, st>>>(F0, B, F, scale, H, (float)sample_rate, phase_start, lw,
                                                          lb, src);
    } else {
        // the fp32 starts fit in the B*H*F doubles reserved for them
        float* start = reinterpret_cast<float*>(phase_start);
        ::bsml::count_launch();
        hs_phase32_kernel<<<(unsigned)ceil_div(B * H, 32), 32, 0, st>>>(F0, B, F, scale, H, (float)sample_rate,
                                                                        start);
        ::bsml::count_launch();
        hs_source32_kernel<<<grid_for((int64_t)B * F, 64), 64, 0, st>>>(F0, B, F, scale, H, (float)sample_rate,
                                                                        start, lw, lb, src);
    }
    ::bsml::count_launch();
    hs_stft_kernel<<<grid_for((int64_t)B * har.L, 128), 128, 0, st>>>(src, B, (int)S, n_fft, hop, har);
    BSML_LAUNCH("harmonic_source");
}

void l1_loss(const float* a, const float* t, int64_t n, float* loss, float* da, double* acc, cudaStream_t st) {
    ::bsml::count_launch();
    zero1<<<1, 1, 0, st>>>(acc);
    ::bsml::count_launch();
    l1_kernel<<<grid_for(n), 256, 0, st>>>(a, t, n, da, acc);
    ::bsml::count_launch();
    l1_final_kernel<<<1, 1, 0, st>>>(acc, n, loss);
    BSML_LAUNCH("l1_loss");
}

void adam(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2, float eps, int step,
          cudaStream_t st) {
    const float bc1 = 1.f - powf(b1, (float)step), bc2 = 1.f - powf(b2, (float)step);
    ::bsml::count_launch();
    adam_kernel<<<grid_for(n), 256, 0, st>>>(p, g, m, v, n, lr, b1, b2, eps, bc1, bc2);
    BSML_LAUNCH("adam");
}

}  // namespace bsml
