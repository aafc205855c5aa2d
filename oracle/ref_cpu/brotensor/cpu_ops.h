// CPU stand-ins for the brotensor ops the reference's decoder sources call
// (src/kokoro_decoder_backward.cpp, src/decoder_lora.cpp). Checker only: these
// exist so the reference's own composition compiles and runs here, as the
// reference (whose op library, brotensor, is absent) would run it on its CPU
// backend. Each op is restated from the PyTorch definition the upstream Kokoro
// model uses; signatures follow the reference's call sites. fp32 storage.
#pragma once

#include <brotensor/tensor.h>

#include <cstddef>
#include <cstdint>

namespace brotensor {

// ── activation
void leaky_relu_forward(const Tensor& x, float slope, Tensor& y);
void leaky_relu_backward(const Tensor& x, const Tensor& dy, float slope, Tensor& dx);
// Snake1D y = x + sin^2(alpha x) / alpha, alpha (C, 1) per channel, x (N, C*L);
// beta must be null (the SnakeBeta variant is not used on this path)
void snake_forward(const Tensor& x, const Tensor& alpha, const Tensor* beta, int N, int C, int L, Tensor& y);
void snake_backward(const Tensor& x, const Tensor& alpha, const Tensor* beta, const Tensor& dy, int N, int C, int L,
                    Tensor& dx, Tensor& dalpha, Tensor* dbeta);
void tanh_forward(const Tensor& x, Tensor& y);
// dx = dy * (1 - y^2), y = tanh output
void tanh_backward(const Tensor& y, const Tensor& dy, Tensor& dx);

// ── copies
void copy_d2d(const Tensor& src, std::size_t src_off, Tensor& dst, std::size_t dst_off, std::size_t n);

// ── convolutions (NCL, W (C_out, (C_in/groups)*k) for conv1d, (C_in, (C_out/groups)*k) for convT)
void conv1d_forward(const Tensor& x, const Tensor& W, const Tensor* b, int N, int C_in, int L, int C_out, int k,
                    int stride, int pad, int dil, int groups, Tensor& y);
void conv1d_backward_input(const Tensor& W, const Tensor& dY, int N, int C_in, int L, int C_out, int k, int stride,
                           int pad, int dil, int groups, Tensor& dX);
void conv_transpose1d_forward(const Tensor& x, const Tensor& W, const Tensor* b, int N, int C_in, int L, int C_out,
                              int k, int stride, int pad, int out_pad, int dil, int groups, Tensor& y);
void conv_transpose1d_forward(const Tensor& x, const Tensor& W, const Tensor* b, int N, int C_in, int L, int C_out,
                              int k, int stride, int pad, int out_pad, int dil, Tensor& y);
void conv_transpose1d_backward_input(const Tensor& W, const Tensor& dY, int N, int C_in, int L_in, int C_out, int k,
                                     int stride, int pad, int out_pad, int dil, int groups, Tensor& dX);
void conv_transpose1d_backward_input(const Tensor& W, const Tensor& dY, int N, int C_in, int L_in, int C_out, int k,
                                     int stride, int pad, int out_pad, int dil, Tensor& dX);

// ── modulate: Y = X * (1 + gamma) + beta, X (M, C), gamma / beta (C, 1)
void modulate(const Tensor& X, const Tensor& gamma, const Tensor& beta, Tensor& Y);

// ── elementwise
void mul_inplace(Tensor& a, const Tensor& b);
void add_inplace(Tensor& a, const Tensor& b);
void scale_inplace(Tensor& a, float s);

// ── GroupNorm over x (N, C*H*W), biased variance; gamma / beta (C, 1)
void group_norm_forward(const Tensor& x, const Tensor& gamma, const Tensor& beta, int N, int C, int H, int W,
                        int groups, float eps, Tensor& y);
// dgamma / dbeta accumulate (+=)
void group_norm_backward(const Tensor& x, const Tensor& gamma, const Tensor& dy, int N, int C, int H, int W,
                         int groups, float eps, Tensor& dx, Tensor& dgamma, Tensor& dbeta);

// ── reductions: column sums of (M, C) -> (1, C)
void sum_cols(const Tensor& t, Tensor& out);

// ── layouts: (N, C*H*W) <-> (N*H*W, C)
void nchw_to_sequence(const Tensor& x, int N, int C, int H, int W, Tensor& y);
void sequence_to_nchw(const Tensor& x, int N, int C, int H, int W, Tensor& y);

// ── spectral (torch.istft semantics: onesided, window envelope, center trim)
// mag / pha (L, nf) -> spec (L, 2*nf), interleaved (re, im)
void complex_from_polar(const Tensor& mag, const Tensor& pha, Tensor& spec);
void istft(const Tensor& spec, const Tensor& window, int N, int signal_len, int n_fft, int hop, int win, bool center,
           bool normalized, Tensor& audio);
void istft_backward(const Tensor& daudio, const Tensor& window, int N, int signal_len, int n_fft, int hop, int win,
                    bool center, bool normalized, Tensor& dspec);
// mode 1 = reflect; x (N, C*L) -> y (N, C*(pl + L + pr))
void pad1d_forward(const Tensor& x, int N, int C, int L, int pl, int pr, int mode, Tensor& y);
void pad1d_backward(const Tensor& dy, int N, int C, int L, int pl, int pr, int mode, Tensor& dx);

// ── linear / LoRA / optimiser
// y = W x + b, x (in, 1)
void linear_forward(const Tensor& W, const Tensor& b, const Tensor& x, Tensor& y);
// dX = W^T dY (overwritten); dW += dY x^T; dB += dY
void linear_backward(const Tensor& W, const Tensor& x, const Tensor& dY, Tensor& dX, Tensor& dW, Tensor& dB);
// y = W x + b + scale * B (g * h), h = A x, hg = g * h (g null: ones)
void lora_forward(const Tensor& W, const Tensor& b, const Tensor& x, const Tensor& A, const Tensor& B, float scale,
                  const Tensor* g, Tensor& y, Tensor& h, Tensor& hg);
// accumulates dA, dB, dG (+=); dX (nullable) overwritten
void lora_backward(const Tensor& W, const Tensor& x, const Tensor& A, const Tensor& B, float scale, const Tensor* g,
                   const Tensor& h, const Tensor& hg, const Tensor& dY, Tensor& dA, Tensor& dB, Tensor* dG,
                   Tensor* dX);
void adam_step(Tensor& p, const Tensor& g, Tensor& m, Tensor& v, float lr, float beta1, float beta2, float eps,
               int step);
// xavier-uniform from a splitmix64 stream advanced in place
void xavier_init(Tensor& W, std::uint64_t& rng);

}  // namespace brotensor
