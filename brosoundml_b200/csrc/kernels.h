// Host-side launchers for the sm_100a kernels (channels-last activations).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"

namespace bsml {

// ── forward-like convolution ─────────────────────────────────────────────────
// y[b, orow(o), co] = alpha * (sum_{t,ci} Wp[t][ci][co] * x[b, (o+o_base)*s + t*d - p, ci]
//                              + bias[co] + r[b, orow >> r_shift, co]) + (accum ? y : 0)
// with orow(o) = (o + o_base) * orow_mul + orow_off, skipped outside [0, y.L).
// Covers conv fwd, conv dgrad (flipped, transposed weights), convT fwd (one
// call per stride phase) and convT dgrad.
struct ConvFwd {
    Act x;                 // input  (B, L_in, Ci)
    Act y;                 // output (B, rows, Co)
    const float* wp = nullptr;   // packed weights [k][Ci][Cop]  (Cop = round_up(Co, 4))
    const float* bias = nullptr;
    const Act* r = nullptr;      // optional residual
    int r_shift = 0;
    int k = 1, s = 1, p = 0, d = 1;
    int No = 0, o_base = 0, orow_mul = 1, orow_off = 0;
    float alpha = 1.0f;
    bool accum = false;
};
void conv_fwd_simt(const ConvFwd& a, cudaStream_t st);

// ── weight gradient ──────────────────────────────────────────────────────────
// dW[(co*Ci + ci)*k + t] (+)= sum_{b,o} dy[b, o, co] * x[b, o*s + t*d - p, ci]
// db[co] (+)= sum_{b,o} dy[b, o, co]. `part` needs wgrad_partial_floats() floats.
struct ConvWgrad {
    Act dy;                // (B, Lo, Co)
    Act x;                 // (B, L_in, Ci)
    int k = 1, s = 1, p = 0, d = 1;
    float* dW = nullptr;
    float* db = nullptr;
    bool accum = false;
};
int64_t wgrad_partial_floats(const ConvWgrad& a);
void conv_wgrad_simt(const ConvWgrad& a, float* part, cudaStream_t st);
void colsum(const Act& dy, float* db, bool accum, float* part, cudaStream_t st);
int64_t colsum_partial_floats(const Act& dy);

// ── weight packing ───────────────────────────────────────────────────────────
// conv weight W (Co, Ci, k) -> Wp[t][ci][co] (fwd) ; for dgrad: Wd[t'][co][ci] = W[co][ci][k-1-t'] ;
// convT weight W (Ci, Co, k), phase r of stride s: Wr[m'][ci][co] = W[ci][co][r + (kr-1-m')*s].
void pack_conv_fwd(const float* W, int Co, int Ci, int k, float* wp, cudaStream_t st);
void pack_conv_dgrad(const float* W, int Co, int Ci, int k, float* wp, cudaStream_t st);
void pack_convT_phase(const float* W, int Ci, int Co, int k, int s, int r, float* wp, cudaStream_t st);
void pack_convT_dgrad(const float* W, int Ci, int Co, int k, float* wp, cudaStream_t st);

// ── normalisation and activations ────────────────────────────────────────────
enum Activation { ACT_NONE = 0, ACT_LEAKY = 1, ACT_SNAKE = 2 };

// Operand-plane output of an elementwise kernel, for the tensor-core convs:
// planes share the (B, L) geometry of the fp32 tensor with row pitch `ld`
// (mode 1: tf32 hi + fp32 lo planes, mode 0: one bf16 plane).
struct PlaneOut { void* hi = nullptr; void* lo = nullptr; int ld = 0; int mode = 1; };

// sums[(b*C + c)*2 + {0,1}] += sum_l x, sum_l x^2 (double; the caller zeroes sums)
void norm_sums(const Act& x, double* sums, cudaStream_t st);
// acc: (B*C*2) doubles, zeroed inside. mean/rstd: (B*C) floats.
void in_stats(const Act& x, float eps, double* acc, float* mean, float* rstd, cudaStream_t st);
// AdaIN + activation forward. With sums (norm_sums layout) the statistics come
// from the sums and mean / rstd are written; with sums == nullptr they are read.
// Writes y (fp32, nullable) and / or operand planes (nullable).
void adain_act_fwd_v(const Act& x, const double* sums, float eps, float* mean, float* rstd, const float* gb, int act,
                     float slope, const float* alpha, const Act* y, const PlaneOut* planes, cudaStream_t st);
// Backward of adain_act_fwd_v. out = dx (+ skip_scale * skip; dx may alias skip)
// goes to dx (nullable) and / or planes (nullable); with dx_accum the prior dx is
// added as well (out = dx_old + ..., then stored to dx and the planes);
// colsum[c] += sum over (b, l) of out (double, nullable, not zeroed here). dgb,
// dalpha as in adain_act_bwd.
void adain_act_bwd_v(const Act& x, const float* mean, const float* rstd, const float* gb, int act, float slope,
                     const float* alpha, const Act& dy, const Act* dx, const Act* skip, const PlaneOut* planes,
                     double* colsum, float* dgb, float* dalpha, double* acc, cudaStream_t st,
                     bool acc_ready = false, float skip_scale = 1.f, bool dx_accum = false,
                     const PlaneOut* planes2 = nullptr);
// The backward's reduction pass fused with recomputing the forward output act(AdaIN(x))
// into y / planes (a weight gradient's operand): acc is zeroed and filled for a
// following adain_act_bwd_v(..., acc_ready = true) with the same x, dy and affine.
void adain_recompute_reduce(const Act& x, const float* mean, const float* rstd, const float* gb, int act,
                            float slope, const float* alpha, const Act* y, const PlaneOut* planes, const Act& dy,
                            double* acc, cudaStream_t st);
// out = alpha * src -> dst (nullable), planes (nullable), colsum (nullable, added to).
// planes2 (here and in adain_act_bwd_v): a second set of operand planes of the same
// output in another mode (the weight gradients' operand when their mode differs)
void scale_out_v(const Act& src, float alpha, const Act* dst, const PlaneOut* planes, double* colsum,
                 cudaStream_t st, const PlaneOut* planes2 = nullptr);
// dst[i] (+)= (float) src[i]
void d2f(const double* src, int n, float* dst, bool accum, cudaStream_t st);
// y = act((1 + gamma) * (x - mean) * rstd + beta); gb = [B][2C] (gamma ; beta)
void adain_act_fwd(const Act& x, const float* mean, const float* rstd, const float* gb, int act, float slope,
                   const float* alpha, const Act& y, cudaStream_t st);
// Backward of adain_act_fwd. dy: grad of the activation output. Writes
// dx (+= skip when skip != nullptr, dx may alias skip), dgb [B][2C] (dGamma ; dBeta),
// and dalpha[c] += sum_b (snake only). acc: (B*C*3) doubles scratch.
void adain_act_bwd(const Act& x, const float* mean, const float* rstd, const float* gb, int act, float slope,
                   const float* alpha, const Act& dy, const Act& dx, const Act* skip, float* dgb, float* dalpha,
                   double* acc, cudaStream_t st);

// plain Snake1D and its backward (alpha grad per channel, overwritten); acc: B*C doubles
void snake_fwd(const Act& x, const float* alpha, const Act& y, cudaStream_t st);
void snake_bwd(const Act& x, const float* alpha, const Act& dy, const Act& dx, float* dalpha, double* acc,
               cudaStream_t st);

void leaky_fwd(const Act& x, float slope, const Act& y, cudaStream_t st);
void leaky_bwd(const Act& x, float slope, const Act& dy, const Act& dx, cudaStream_t st);
void copy_act(const Act& src, const Act& dst, cudaStream_t st);                 // same B, L, C
void add_act(const Act& src, const Act& dst, float alpha, cudaStream_t st);     // dst += alpha*src
void scale_act(const Act& x, float alpha, cudaStream_t st);
void pair_sum_rows(const Act& src, const Act& dst, cudaStream_t st);            // dst[l] = src[2l] + src[2l+1]
void reflect_left1_fwd(const Act& y, cudaStream_t st);                          // y[0] = y[2]
void reflect_left1_bwd(const Act& dy, cudaStream_t st);                         // dy[2] += dy[0]
void ncl_to_cl(const float* src, const Act& dst, cudaStream_t st);               // (B, C, L) -> Act
void cl_to_ncl(const Act& src, float* dst, cudaStream_t st);
void fill(float* p, int64_t n, float v, cudaStream_t st);

// depthwise ConvTranspose1d (groups = C), weight (C, 1, k): the upsampling pool.
void dwconvT_fwd(const Act& x, const float* W, const float* bias, int k, int s, int p, const Act& y, cudaStream_t st);
void dwconvT_dgrad(const Act& dy, const float* W, int k, int s, int p, const Act& dx, cudaStream_t st);
// acc: C*k doubles of scratch; part: colsum_partial_floats(dy) floats (bias sums)
void dwconvT_wgrad(const Act& dy, const Act& x, int k, int s, int p, float* dW, float* db, double* acc,
                   float* part, cudaStream_t st);

// ── AdaIN fc (style -> gamma/beta) for many AdaINs at once ──────────────────
// One AdaIN fc: weight/bias offsets into the flat params, output offset into the
// packed [a][B][2C] affine buffer, 2C rows, and the entry's first global row.
struct FcRow { int64_t w_off, b_off, out_off; int n_out; int row0; };
// table: one entry per AdaIN (device memory); style (B, S); out packed [a][B][2C]
void affine_fc_fwd(const FcRow* table, int n_entries, int total_rows, const int* row_entry, const float* params,
                   const float* style, int B, int S, float* out, cudaStream_t st);
void affine_fc_bwd(const FcRow* table, int n_entries, int total_rows, const int* row_entry, const float* params,
                   const float* style, const float* daff, int B, int S, float* grads, float* d_style, float* part,
                   cudaStream_t st);

// ── spectral head, harmonic source ──────────────────────────────────────────
// post (B, L, n_fft+2) -> spec (B, L, 2*nf) interleaved (re_k, im_k)
void polar_fwd(const Act& post, int nf, float* spec, cudaStream_t st);
void istft_fwd(const float* spec, int B, int L, int n_fft, int hop, float* audio, cudaStream_t st);
// daudio -> dpost (through the polar adjoint; post read for exp/sin)
void istft_polar_bwd(const float* daudio, const Act& post, int n_fft, int hop, const Act& dpost, cudaStream_t st);
// plain istft adjoint (for the atom API): daudio -> dre, dim (B, nf, L) NCL
void istft_bwd_ncl(const float* daudio, int B, int L, int n_fft, int hop, float* dre, float* dim, cudaStream_t st);
void istft_fwd_ncl(const float* re, const float* im, int B, int L, int n_fft, int hop, float* audio,
                   float* spec_scratch, cudaStream_t st);
// F0 (B, F) -> har Act (B, frames, 2*nf); scratch: B*(harmonic_num+1)*F doubles + B*F*scale floats.
// phase_mode: PHASE_FP32_RUNNING (the reference's fp32 per-sample accumulator) or PHASE_EXACT.
enum { PHASE_FP32_RUNNING = 0, PHASE_EXACT = 1 };
void harmonic_source(const float* F0, int B, int F, int scale, int harmonic_num, int sample_rate, int n_fft, int hop,
                     const float* lw, const float* lb, double* phase_start, float* src, const Act& har,
                     cudaStream_t st, int phase_mode = PHASE_FP32_RUNNING);

// ── loss and optimiser ───────────────────────────────────────────────────────
void l1_loss(const float* a, const float* t, int64_t n, float* loss, float* da, double* acc, cudaStream_t st);
void adam(float* p, const float* g, float* m, float* v, int64_t n, float lr, float b1, float b2, float eps, int step,
          cudaStream_t st);

}  // namespace bsml

namespace bsml {
// Weight gradient with the split-K partials bounded by `part_cap` floats (fewer
// splits when the cap is small); the bias column sums use the same bound.
// Returns false, launching nothing, when even one split does not fit.
bool conv_wgrad_simt_capped(const ConvWgrad& a, float* part, int64_t part_cap, cudaStream_t st);
}  // namespace bsml
