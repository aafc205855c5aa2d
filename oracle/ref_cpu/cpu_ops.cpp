// CPU stand-ins for the brotensor ops (declarations and conventions in
// brotensor/cpu_ops.h) and for the one module method the reference's decoder
// sources call, Conv1d::forward (the reference's modules.h, defined in its
// src/modules.cpp, which is not compiled here). Checker only.
#include <brotensor/cpu_ops.h>

#include <cmath>
#include <stdexcept>
#include <string>

#include "brosoundml/modules.h"

namespace brotensor {

namespace {

[[noreturn]] void bad(const char* op, const std::string& why) {
    throw std::runtime_error(std::string("brotensor(cpu checker): ") + op + ": " + why);
}
void need_n(const Tensor& t, std::int64_t n, const char* op, const char* what) {
    if (t.size() != n) bad(op, std::string(what) + " has " + std::to_string(t.size()) + " elements, expected " +
                                   std::to_string(n));
}
constexpr double kPi = 3.14159265358979323846;

}  // namespace

// ── activation
void leaky_relu_forward(const Tensor& x, float slope, Tensor& y) {
    Tensor o = Tensor::zeros_on(x.device, x.rows, x.cols);
    for (std::int64_t i = 0; i < x.size(); ++i) o[i] = x[i] > 0.f ? x[i] : slope * x[i];
    y = std::move(o);
}

void leaky_relu_backward(const Tensor& x, const Tensor& dy, float slope, Tensor& dx) {
    need_n(dy, x.size(), "leaky_relu_backward", "dy");
    Tensor o = Tensor::zeros_on(x.device, x.rows, x.cols);
    for (std::int64_t i = 0; i < x.size(); ++i) o[i] = x[i] > 0.f ? dy[i] : slope * dy[i];
    dx = std::move(o);
}

void snake_forward(const Tensor& x, const Tensor& alpha, const Tensor* beta, int N, int C, int L, Tensor& y) {
    if (beta) bad("snake_forward", "beta is not supported");
    need_n(x, (std::int64_t)N * C * L, "snake_forward", "x");
    need_n(alpha, C, "snake_forward", "alpha");
    Tensor o = Tensor::zeros_on(x.device, x.rows, x.cols);
    for (int n = 0; n < N; ++n)
        for (int c = 0; c < C; ++c) {
            const double a = alpha[c];
            for (int l = 0; l < L; ++l) {
                const std::int64_t i = ((std::int64_t)n * C + c) * L + l;
                const double s = std::sin(a * x[i]);
                o[i] = (float)(x[i] + s * s / a);
            }
        }
    y = std::move(o);
}

void snake_backward(const Tensor& x, const Tensor& alpha, const Tensor* beta, const Tensor& dy, int N, int C, int L,
                    Tensor& dx, Tensor& dalpha, Tensor* dbeta) {
    if (beta || dbeta) bad("snake_backward", "beta is not supported");
    need_n(dy, (std::int64_t)N * C * L, "snake_backward", "dy");
    Tensor o = Tensor::zeros_on(x.device, x.rows, x.cols);
    Tensor da = Tensor::zeros_on(x.device, C, 1);
    for (int c = 0; c < C; ++c) {
        const double a = alpha[c];
        double acc = 0;
        for (int n = 0; n < N; ++n)
            for (int l = 0; l < L; ++l) {
                const std::int64_t i = ((std::int64_t)n * C + c) * L + l;
                const double s = std::sin(a * x[i]), s2 = std::sin(2 * a * x[i]);
                o[i] = (float)(dy[i] * (1.0 + s2));
                acc += dy[i] * (x[i] * s2 / a - s * s / (a * a));
            }
        da[c] = (float)acc;
    }
    dx = std::move(o);
    dalpha = std::move(da);
}

void tanh_forward(const Tensor& x, Tensor& y) {
    Tensor o = Tensor::zeros_on(x.device, x.rows, x.cols);
    for (std::int64_t i = 0; i < x.size(); ++i) o[i] = std::tanh(x[i]);
    y = std::move(o);
}

void tanh_backward(const Tensor& y, const Tensor& dy, Tensor& dx) {
    need_n(dy, y.size(), "tanh_backward", "dy");
    Tensor o = Tensor::zeros_on(y.device, y.rows, y.cols);
    for (std::int64_t i = 0; i < y.size(); ++i) o[i] = dy[i] * (1.f - y[i] * y[i]);
    dx = std::move(o);
}

// ── copies
void copy_d2d(const Tensor& src, std::size_t so, Tensor& dst, std::size_t d, std::size_t n) {
    if ((std::int64_t)(so + n) > src.size() || (std::int64_t)(d + n) > dst.size()) bad("copy_d2d", "out of range");
    for (std::size_t i = 0; i < n; ++i) dst[(std::int64_t)(d + i)] = src[(std::int64_t)(so + i)];
}

// ── convolutions
namespace {
int conv_len(int L, int k, int s, int p, int d) { return (L + 2 * p - d * (k - 1) - 1) / s + 1; }
int convT_len(int L, int k, int s, int p, int op, int d) { return (L - 1) * s - 2 * p + d * (k - 1) + op + 1; }
}  // namespace

void conv1d_forward(const Tensor& x, const Tensor& W, const Tensor* b, int N, int Ci, int L, int Co, int k, int s,
                    int p, int d, int groups, Tensor& y) {
    const int cig = Ci / groups, cog = Co / groups, Lo = conv_len(L, k, s, p, d);
    need_n(x, (std::int64_t)N * Ci * L, "conv1d_forward", "x");
    need_n(W, (std::int64_t)Co * cig * k, "conv1d_forward", "W");
    Tensor o = Tensor::zeros_on(x.device, N, Co * Lo);
    for (int n = 0; n < N; ++n)
        for (int co = 0; co < Co; ++co) {
            const int g = co / cog;
            for (int t = 0; t < Lo; ++t) {
                double acc = (b && b->size()) ? (*b)[co] : 0.0;
                for (int cl = 0; cl < cig; ++cl) {
                    const int ci = g * cig + cl;
                    for (int j = 0; j < k; ++j) {
                        const int l = t * s + j * d - p;
                        if (l < 0 || l >= L) continue;
                        acc += (double)W[((std::int64_t)co * cig + cl) * k + j] * x[((std::int64_t)n * Ci + ci) * L + l];
                    }
                }
                o[((std::int64_t)n * Co + co) * Lo + t] = (float)acc;
            }
        }
    y = std::move(o);
}

void conv1d_backward_input(const Tensor& W, const Tensor& dY, int N, int Ci, int L, int Co, int k, int s, int p,
                           int d, int groups, Tensor& dX) {
    const int cig = Ci / groups, cog = Co / groups, Lo = conv_len(L, k, s, p, d);
    need_n(dY, (std::int64_t)N * Co * Lo, "conv1d_backward_input", "dY");
    std::vector<double> acc((size_t)N * Ci * L, 0.0);
    for (int n = 0; n < N; ++n)
        for (int co = 0; co < Co; ++co) {
            const int g = co / cog;
            for (int t = 0; t < Lo; ++t) {
                const double gy = dY[((std::int64_t)n * Co + co) * Lo + t];
                for (int cl = 0; cl < cig; ++cl)
                    for (int j = 0; j < k; ++j) {
                        const int l = t * s + j * d - p;
                        if (l < 0 || l >= L) continue;
                        acc[((size_t)n * Ci + g * cig + cl) * L + l] += gy * W[((std::int64_t)co * cig + cl) * k + j];
                    }
            }
        }
    Tensor o = Tensor::zeros_on(dY.device, N, Ci * L);
    for (size_t i = 0; i < acc.size(); ++i) o[(std::int64_t)i] = (float)acc[i];
    dX = std::move(o);
}

void conv_transpose1d_forward(const Tensor& x, const Tensor& W, const Tensor* b, int N, int Ci, int L, int Co, int k,
                              int s, int p, int op, int d, int groups, Tensor& y) {
    const int cig = Ci / groups, cog = Co / groups, Lo = convT_len(L, k, s, p, op, d);
    need_n(x, (std::int64_t)N * Ci * L, "conv_transpose1d_forward", "x");
    need_n(W, (std::int64_t)Ci * cog * k, "conv_transpose1d_forward", "W");
    std::vector<double> acc((size_t)N * Co * Lo, 0.0);
    for (int n = 0; n < N; ++n)
        for (int ci = 0; ci < Ci; ++ci) {
            const int g = ci / cig;
            for (int l = 0; l < L; ++l) {
                const double xv = x[((std::int64_t)n * Ci + ci) * L + l];
                for (int cl = 0; cl < cog; ++cl)
                    for (int j = 0; j < k; ++j) {
                        const int o = l * s + j * d - p;
                        if (o < 0 || o >= Lo) continue;
                        acc[((size_t)n * Co + g * cog + cl) * Lo + o] += xv * W[((std::int64_t)ci * cog + cl) * k + j];
                    }
            }
        }
    Tensor out = Tensor::zeros_on(x.device, N, Co * Lo);
    for (int n = 0; n < N; ++n)
        for (int co = 0; co < Co; ++co)
            for (int o = 0; o < Lo; ++o) {
                const size_t i = ((size_t)n * Co + co) * Lo + o;
                out[(std::int64_t)i] = (float)(acc[i] + ((b && b->size()) ? (*b)[co] : 0.0));
            }
    y = std::move(out);
}

void conv_transpose1d_forward(const Tensor& x, const Tensor& W, const Tensor* b, int N, int Ci, int L, int Co, int k,
                              int s, int p, int op, int d, Tensor& y) {
    conv_transpose1d_forward(x, W, b, N, Ci, L, Co, k, s, p, op, d, 1, y);
}

void conv_transpose1d_backward_input(const Tensor& W, const Tensor& dY, int N, int Ci, int L, int Co, int k, int s,
                                     int p, int op, int d, int groups, Tensor& dX) {
    const int cig = Ci / groups, cog = Co / groups, Lo = convT_len(L, k, s, p, op, d);
    need_n(dY, (std::int64_t)N * Co * Lo, "conv_transpose1d_backward_input", "dY");
    Tensor o = Tensor::zeros_on(dY.device, N, Ci * L);
    for (int n = 0; n < N; ++n)
        for (int ci = 0; ci < Ci; ++ci) {
            const int g = ci / cig;
            for (int l = 0; l < L; ++l) {
                double acc = 0;
                for (int cl = 0; cl < cog; ++cl)
                    for (int j = 0; j < k; ++j) {
                        const int t = l * s + j * d - p;
                        if (t < 0 || t >= Lo) continue;
                        acc += (double)W[((std::int64_t)ci * cog + cl) * k + j] *
                               dY[((std::int64_t)n * Co + g * cog + cl) * Lo + t];
                    }
                o[((std::int64_t)n * Ci + ci) * L + l] = (float)acc;
            }
        }
    dX = std::move(o);
}

void conv_transpose1d_backward_input(const Tensor& W, const Tensor& dY, int N, int Ci, int L, int Co, int k, int s,
                                     int p, int op, int d, Tensor& dX) {
    conv_transpose1d_backward_input(W, dY, N, Ci, L, Co, k, s, p, op, d, 1, dX);
}

// ── modulate / elementwise / reductions / layouts
void modulate(const Tensor& X, const Tensor& gamma, const Tensor& beta, Tensor& Y) {
    const int M = X.rows, C = X.cols;
    need_n(gamma, C, "modulate", "gamma");
    need_n(beta, C, "modulate", "beta");
    Tensor o = Tensor::zeros_on(X.device, M, C);
    for (int m = 0; m < M; ++m)
        for (int c = 0; c < C; ++c) {
            const std::int64_t i = (std::int64_t)m * C + c;
            o[i] = X[i] * (1.f + gamma[c]) + beta[c];
        }
    Y = std::move(o);
}

void mul_inplace(Tensor& a, const Tensor& b) {
    need_n(b, a.size(), "mul_inplace", "b");
    for (std::int64_t i = 0; i < a.size(); ++i) a[i] *= b[i];
}
void add_inplace(Tensor& a, const Tensor& b) {
    need_n(b, a.size(), "add_inplace", "b");
    for (std::int64_t i = 0; i < a.size(); ++i) a[i] += b[i];
}
void scale_inplace(Tensor& a, float s) {
    for (std::int64_t i = 0; i < a.size(); ++i) a[i] *= s;
}

void sum_cols(const Tensor& t, Tensor& out) {
    Tensor o = Tensor::zeros_on(t.device, 1, t.cols);
    for (int c = 0; c < t.cols; ++c) {
        double acc = 0;
        for (int m = 0; m < t.rows; ++m) acc += t[(std::int64_t)m * t.cols + c];
        o[c] = (float)acc;
    }
    out = std::move(o);
}

void nchw_to_sequence(const Tensor& x, int N, int C, int H, int W, Tensor& y) {
    const int S = H * W;
    need_n(x, (std::int64_t)N * C * S, "nchw_to_sequence", "x");
    Tensor o = Tensor::zeros_on(x.device, N * S, C);
    for (int n = 0; n < N; ++n)
        for (int c = 0; c < C; ++c)
            for (int q = 0; q < S; ++q) o[((std::int64_t)n * S + q) * C + c] = x[((std::int64_t)n * C + c) * S + q];
    y = std::move(o);
}

void sequence_to_nchw(const Tensor& x, int N, int C, int H, int W, Tensor& y) {
    const int S = H * W;
    need_n(x, (std::int64_t)N * C * S, "sequence_to_nchw", "x");
    Tensor o = Tensor::zeros_on(x.device, N, C * S);
    for (int n = 0; n < N; ++n)
        for (int c = 0; c < C; ++c)
            for (int q = 0; q < S; ++q) o[((std::int64_t)n * C + c) * S + q] = x[((std::int64_t)n * S + q) * C + c];
    y = std::move(o);
}

// ── GroupNorm
void group_norm_forward(const Tensor& x, const Tensor& gamma, const Tensor& beta, int N, int C, int H, int W,
                        int G, float eps, Tensor& y) {
    const int cg = C / G, S = H * W;
    need_n(x, (std::int64_t)N * C * S, "group_norm_forward", "x");
    Tensor o = Tensor::zeros_on(x.device, x.rows, x.cols);
    for (int n = 0; n < N; ++n)
        for (int g = 0; g < G; ++g) {
            const std::int64_t base = ((std::int64_t)n * C + g * cg) * S, cnt = (std::int64_t)cg * S;
            double m = 0, v = 0;
            for (std::int64_t i = 0; i < cnt; ++i) m += x[base + i];
            m /= cnt;
            for (std::int64_t i = 0; i < cnt; ++i) v += (x[base + i] - m) * (x[base + i] - m);
            v /= cnt;
            const double rs = 1.0 / std::sqrt(v + eps);
            for (int cl = 0; cl < cg; ++cl) {
                const int c = g * cg + cl;
                for (int q = 0; q < S; ++q) {
                    const std::int64_t i = base + (std::int64_t)cl * S + q;
                    o[i] = (float)((x[i] - m) * rs * gamma[c] + beta[c]);
                }
            }
        }
    y = std::move(o);
}

void group_norm_backward(const Tensor& x, const Tensor& gamma, const Tensor& dy, int N, int C, int H, int W, int G,
                         float eps, Tensor& dx, Tensor& dgamma, Tensor& dbeta) {
    const int cg = C / G, S = H * W;
    need_n(dy, x.size(), "group_norm_backward", "dy");
    if (dgamma.size() != C) dgamma = Tensor::zeros_on(x.device, C, 1);
    if (dbeta.size() != C) dbeta = Tensor::zeros_on(x.device, C, 1);
    Tensor o = Tensor::zeros_on(x.device, x.rows, x.cols);
    for (int n = 0; n < N; ++n)
        for (int g = 0; g < G; ++g) {
            const std::int64_t base = ((std::int64_t)n * C + g * cg) * S, cnt = (std::int64_t)cg * S;
            double m = 0, v = 0;
            for (std::int64_t i = 0; i < cnt; ++i) m += x[base + i];
            m /= cnt;
            for (std::int64_t i = 0; i < cnt; ++i) v += (x[base + i] - m) * (x[base + i] - m);
            v /= cnt;
            const double rs = 1.0 / std::sqrt(v + eps);
            // with dxh = dy * gamma: dx = rs * (dxh - mean(dxh) - xh * mean(dxh * xh))
            double s1 = 0, s2 = 0;
            for (int cl = 0; cl < cg; ++cl) {
                const int c = g * cg + cl;
                for (int q = 0; q < S; ++q) {
                    const std::int64_t i = base + (std::int64_t)cl * S + q;
                    const double xh = (x[i] - m) * rs, dxh = (double)dy[i] * gamma[c];
                    s1 += dxh;
                    s2 += dxh * xh;
                    dgamma[c] += (float)(dy[i] * xh);
                    dbeta[c] += dy[i];
                }
            }
            s1 /= cnt;
            s2 /= cnt;
            for (int cl = 0; cl < cg; ++cl) {
                const int c = g * cg + cl;
                for (int q = 0; q < S; ++q) {
                    const std::int64_t i = base + (std::int64_t)cl * S + q;
                    const double xh = (x[i] - m) * rs, dxh = (double)dy[i] * gamma[c];
                    o[i] = (float)(rs * (dxh - s1 - xh * s2));
                }
            }
        }
    dx = std::move(o);
}

// ── spectral
void complex_from_polar(const Tensor& mag, const Tensor& pha, Tensor& spec) {
    need_n(pha, mag.size(), "complex_from_polar", "pha");
    Tensor o = Tensor::zeros_on(mag.device, mag.rows, 2 * mag.cols);
    for (std::int64_t i = 0; i < mag.size(); ++i) {
        o[2 * i] = (float)((double)mag[i] * std::cos((double)pha[i]));
        o[2 * i + 1] = (float)((double)mag[i] * std::sin((double)pha[i]));
    }
    spec = std::move(o);
}

namespace {
// torch.istft(onesided, center, normalized=False) as a linear map of the frames:
// frame t's samples x_t[m] = w[m] * irfft(X_t)[m] land at t*hop + m - pad (pad =
// n_fft/2 with center), divided by the overlapped window-square envelope.
struct Istft {
    int n_fft, hop, L, S, nf, pad;
    std::vector<double> w, env;
    Istft(const Tensor& window, int n, int h, int frames, int signal_len, bool center)
        : n_fft(n), hop(h), L(frames), S(signal_len), nf(n / 2 + 1), pad(center ? n / 2 : 0) {
        if (window.size() != n_fft) bad("istft", "window length must equal n_fft");
        w.resize(n_fft);
        for (int m = 0; m < n_fft; ++m) w[m] = window[m];
        env.assign((size_t)(L - 1) * hop + n_fft, 0.0);
        for (int t = 0; t < L; ++t)
            for (int m = 0; m < n_fft; ++m) env[(size_t)t * hop + m] += w[m] * w[m];
    }
    // coefficient of Re X_k / Im X_k in sample m of the inverse real DFT
    double cre(int k, int m) const {
        const double c = (k == 0 || 2 * k == n_fft) ? 1.0 : 2.0;
        return c / n_fft * std::cos(2 * kPi * (double)k * m / n_fft);
    }
    double cim(int k, int m) const {
        if (k == 0 || 2 * k == n_fft) return 0.0;
        return -2.0 / n_fft * std::sin(2 * kPi * (double)k * m / n_fft);
    }
};
}  // namespace

void istft(const Tensor& spec, const Tensor& window, int N, int signal_len, int n_fft, int hop, int /*win*/,
           bool center, bool normalized, Tensor& audio) {
    if (N != 1 || normalized) bad("istft", "N = 1, normalized = false only");
    const int nf = n_fft / 2 + 1, L = spec.rows;
    if (spec.cols != 2 * nf) bad("istft", "spec must be (frames, 2 * n_freq)");
    Istft I(window, n_fft, hop, L, signal_len, center);
    std::vector<double> y(I.env.size(), 0.0);
    for (int t = 0; t < L; ++t)
        for (int m = 0; m < n_fft; ++m) {
            double v = 0;
            for (int k = 0; k < nf; ++k)
                v += I.cre(k, m) * spec[(std::int64_t)t * 2 * nf + 2 * k] + I.cim(k, m) * spec[(std::int64_t)t * 2 * nf + 2 * k + 1];
            y[(size_t)t * hop + m] += I.w[m] * v;
        }
    Tensor o = Tensor::zeros_on(spec.device, 1, signal_len);
    for (int j = 0; j < signal_len; ++j) {
        const size_t q = (size_t)j + I.pad;
        o[j] = (float)(y[q] / I.env[q]);
    }
    audio = std::move(o);
}

void istft_backward(const Tensor& daudio, const Tensor& window, int N, int signal_len, int n_fft, int hop, int /*win*/,
                    bool center, bool normalized, Tensor& dspec) {
    if (N != 1 || normalized) bad("istft_backward", "N = 1, normalized = false only");
    need_n(daudio, signal_len, "istft_backward", "daudio");
    const int nf = n_fft / 2 + 1, L = signal_len / hop + 1;
    Istft I(window, n_fft, hop, L, signal_len, center);
    std::vector<double> dy(I.env.size(), 0.0);
    for (int j = 0; j < signal_len; ++j) dy[(size_t)j + I.pad] = daudio[j] / I.env[(size_t)j + I.pad];
    Tensor o = Tensor::zeros_on(daudio.device, L, 2 * nf);
    for (int t = 0; t < L; ++t)
        for (int k = 0; k < nf; ++k) {
            double gr = 0, gi = 0;
            for (int m = 0; m < n_fft; ++m) {
                const double g = I.w[m] * dy[(size_t)t * hop + m];
                gr += I.cre(k, m) * g;
                gi += I.cim(k, m) * g;
            }
            o[(std::int64_t)t * 2 * nf + 2 * k] = (float)gr;
            o[(std::int64_t)t * 2 * nf + 2 * k + 1] = (float)gi;
        }
    dspec = std::move(o);
}

void pad1d_forward(const Tensor& x, int N, int C, int L, int pl, int pr, int mode, Tensor& y) {
    if (mode != 1) bad("pad1d_forward", "reflect mode (1) only");
    need_n(x, (std::int64_t)N * C * L, "pad1d_forward", "x");
    const int Lo = pl + L + pr;
    Tensor o = Tensor::zeros_on(x.device, N, C * Lo);
    for (int nc = 0; nc < N * C; ++nc)
        for (int j = 0; j < Lo; ++j) {
            int l = j - pl;
            if (l < 0) l = -l;
            if (l >= L) l = 2 * (L - 1) - l;
            o[(std::int64_t)nc * Lo + j] = x[(std::int64_t)nc * L + l];
        }
    y = std::move(o);
}

void pad1d_backward(const Tensor& dy, int N, int C, int L, int pl, int pr, int mode, Tensor& dx) {
    if (mode != 1) bad("pad1d_backward", "reflect mode (1) only");
    const int Lo = pl + L + pr;
    need_n(dy, (std::int64_t)N * C * Lo, "pad1d_backward", "dy");
    Tensor o = Tensor::zeros_on(dy.device, N, C * L);
    for (int nc = 0; nc < N * C; ++nc)
        for (int j = 0; j < Lo; ++j) {
            int l = j - pl;
            if (l < 0) l = -l;
            if (l >= L) l = 2 * (L - 1) - l;
            o[(std::int64_t)nc * L + l] += dy[(std::int64_t)nc * Lo + j];
        }
    dx = std::move(o);
}

// ── linear / LoRA / optimiser
void linear_forward(const Tensor& W, const Tensor& b, const Tensor& x, Tensor& y) {
    const int out = W.rows, in = W.cols;
    need_n(x, in, "linear_forward", "x");
    Tensor o = Tensor::zeros_on(x.device, out, 1);
    for (int r = 0; r < out; ++r) {
        double acc = b.size() ? b[r] : 0.0;
        for (int c = 0; c < in; ++c) acc += (double)W[(std::int64_t)r * in + c] * x[c];
        o[r] = (float)acc;
    }
    y = std::move(o);
}

void linear_backward(const Tensor& W, const Tensor& x, const Tensor& dY, Tensor& dX, Tensor& dW, Tensor& dB) {
    const int out = W.rows, in = W.cols;
    need_n(dY, out, "linear_backward", "dY");
    need_n(x, in, "linear_backward", "x");
    if (dW.size() != W.size()) dW = Tensor::zeros_on(W.device, out, in);
    if (dB.size() != out) dB = Tensor::zeros_on(W.device, out, 1);
    Tensor o = Tensor::zeros_on(W.device, in, 1);
    for (int c = 0; c < in; ++c) {
        double acc = 0;
        for (int r = 0; r < out; ++r) acc += (double)W[(std::int64_t)r * in + c] * dY[r];
        o[c] = (float)acc;
    }
    for (int r = 0; r < out; ++r) {
        for (int c = 0; c < in; ++c) dW[(std::int64_t)r * in + c] += dY[r] * x[c];
        dB[r] += dY[r];
    }
    dX = std::move(o);
}

void lora_forward(const Tensor& W, const Tensor& b, const Tensor& x, const Tensor& A, const Tensor& B, float scale,
                  const Tensor* g, Tensor& y, Tensor& h, Tensor& hg) {
    const int out = W.rows, in = W.cols, r = A.rows;
    need_n(x, in, "lora_forward", "x");
    Tensor hh = Tensor::zeros_on(x.device, r, 1), hgg = Tensor::zeros_on(x.device, r, 1);
    for (int q = 0; q < r; ++q) {
        double acc = 0;
        for (int c = 0; c < in; ++c) acc += (double)A[(std::int64_t)q * in + c] * x[c];
        hh[q] = (float)acc;
        hgg[q] = (float)(acc * (g ? (*g)[q] : 1.0f));
    }
    Tensor o = Tensor::zeros_on(x.device, out, 1);
    for (int o_ = 0; o_ < out; ++o_) {
        double base = b.size() ? b[o_] : 0.0, d = 0;
        for (int c = 0; c < in; ++c) base += (double)W[(std::int64_t)o_ * in + c] * x[c];
        for (int q = 0; q < r; ++q) d += (double)B[(std::int64_t)o_ * r + q] * hgg[q];
        o[o_] = (float)(base + scale * d);
    }
    y = std::move(o);
    h = std::move(hh);
    hg = std::move(hgg);
}

void lora_backward(const Tensor& W, const Tensor& x, const Tensor& A, const Tensor& B, float scale, const Tensor* g,
                   const Tensor& h, const Tensor& hg, const Tensor& dY, Tensor& dA, Tensor& dB, Tensor* dG,
                   Tensor* dX) {
    const int out = W.rows, in = W.cols, r = A.rows;
    need_n(dY, out, "lora_backward", "dY");
    std::vector<double> dhg(r, 0.0);
    for (int q = 0; q < r; ++q)
        for (int o_ = 0; o_ < out; ++o_) dhg[q] += scale * (double)B[(std::int64_t)o_ * r + q] * dY[o_];
    for (int o_ = 0; o_ < out; ++o_)
        for (int q = 0; q < r; ++q) dB[(std::int64_t)o_ * r + q] += (float)(scale * (double)dY[o_] * hg[q]);
    std::vector<double> dh(r);
    for (int q = 0; q < r; ++q) dh[q] = dhg[q] * (g ? (*g)[q] : 1.0f);
    for (int q = 0; q < r; ++q)
        for (int c = 0; c < in; ++c) dA[(std::int64_t)q * in + c] += (float)(dh[q] * x[c]);
    if (dG)
        for (int q = 0; q < r; ++q) (*dG)[q] += (float)(dhg[q] * h[q]);
    if (dX) {
        Tensor o = Tensor::zeros_on(x.device, in, 1);
        for (int c = 0; c < in; ++c) {
            double acc = 0;
            for (int o_ = 0; o_ < out; ++o_) acc += (double)W[(std::int64_t)o_ * in + c] * dY[o_];
            for (int q = 0; q < r; ++q) acc += (double)A[(std::int64_t)q * in + c] * dh[q];
            o[c] = (float)acc;
        }
        *dX = std::move(o);
    }
}

void adam_step(Tensor& p, const Tensor& g, Tensor& m, Tensor& v, float lr, float b1, float b2, float eps, int step) {
    const double bc1 = 1.0 - std::pow((double)b1, step), bc2 = 1.0 - std::pow((double)b2, step);
    for (std::int64_t i = 0; i < p.size(); ++i) {
        m[i] = b1 * m[i] + (1.f - b1) * g[i];
        v[i] = b2 * v[i] + (1.f - b2) * g[i] * g[i];
        p[i] -= (float)(lr * (m[i] / bc1) / (std::sqrt(v[i] / bc2) + eps));
    }
}

void xavier_init(Tensor& W, std::uint64_t& s) {
    const double a = std::sqrt(6.0 / (double)(W.rows + W.cols));
    for (std::int64_t i = 0; i < W.size(); ++i) {
        std::uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        z ^= z >> 31;
        W[i] = (float)((((z >> 40) * (1.0 / 16777216.0)) * 2.0 - 1.0) * a);
    }
}

}  // namespace brotensor

namespace brosoundml {

// the reference's Conv1d::forward (declared in its include/brosoundml/modules.h)
void Conv1d::forward(const brotensor::Tensor& X, int N, int L, brotensor::Tensor& Y) const {
    brotensor::conv1d_forward(X, W, b.size() ? &b : nullptr, N, in_channels, L, out_channels, kernel_size, stride,
                              padding, dilation, groups, Y);
}

}  // namespace brosoundml
