// tcgen05 implicit-GEMM convolution (sm_100a): TMA-staged K-major tiles,
// TMEM accumulators, fused epilogue.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace bsml {

// Operand arithmetic of the tensor-core path.
//   TC_TF32X3: each fp32 operand is split hi + lo (hi = tf32-rounded value,
//              lo = exact fp32 remainder) and D += Ahi*Bhi + Ahi*Blo + Alo*Bhi.
//   TC_BF16:   bf16 operands, one product, fp32 accumulation.
//   TC_BF16X3: each fp32 operand split into bf16 hi + bf16 lo (lo = v - hi rounded),
//              three products as in TF32X3, at the bf16 rate.
enum TcMode { TC_BF16 = 0, TC_TF32X3 = 1, TC_BF16X3 = 2 };

// Operand planes in global memory: fp32 (tf32 hi/lo) or bf16, row pitch `ld`
// elements (16-byte multiple).
struct TcPlanes {
    const void* hi = nullptr;
    const void* lo = nullptr;   // TC_TF32X3 / TC_BF16X3 only
    int ld = 0;
};

inline int tc_pitch(int C, int mode) { return (int)round_up(C, mode == TC_TF32X3 ? 4 : 8); }
inline int tc_esize(int mode) { return mode == TC_TF32X3 ? 4 : 2; }

// Activation x (B, L, C) -> planes (same geometry, pitch tc_pitch(C)).
void make_act_planes(const Act& x, int mode, void* hi, void* lo, cudaStream_t st);
// Weight planes [taps][M][round_up(K, 8)] (K contiguous):
//   conv fwd:       M = Co, K = Ci, tap t   = W[co][ci][t]
//   conv dgrad:     M = Ci, K = Co, tap t'  = W[co][ci][k-1-t']
//   convT phase r:  M = Co, K = Ci, tap m'  = W[ci][co][r + (kr-1-m')*s]
//   convT dgrad:    M = Ci, K = s*Co (row-packed, see ConvTPack), r = the convT padding p
void pack_w_tc(const float* W, int kind, int Co, int Ci, int k, int s, int r, int mode, void* hi, void* lo,
               cudaStream_t st);
//   strided conv:   M = Co, K = s*ld (row-packed input, see the engine's strided noise conv),
//                   r = ld (the unpacked input's row pitch), taps = ceil(k / s):
//                   W2[u][co][j*ld + ci] = W[co][ci][u*s + j] (0 for ci >= Ci or u*s + j >= k)
enum { PACK_CONV_FWD = 0, PACK_CONV_DGRAD = 1, PACK_CONVT_PHASE = 2, PACK_CONVT_DGRAD = 3, PACK_CONV_STRIDED = 4 };

// One weight packing of a batch: the weight at params + w_off, packed as pack_w_tc
// would, into elements [start, start + n) of the batch's flat index space.
struct PackJob {
    // n: packed elements (taps x M x Kp); items: threads' work items (M x Kp, every
    // tap of one (m, kk) per item); start: prefix sum of items over the batch
    int64_t w_off = 0, n = 0, items = 0, start = 0;
    void* hi = nullptr;
    void* lo = nullptr;
    int kind = 0, Co = 0, Ci = 0, k = 0, s = 1, r = 0, taps = 0, M = 0, K = 0, Kp = 0;
};
PackJob make_pack_job(int64_t w_off, int kind, int Co, int Ci, int k, int s, int r, void* hi, void* lo);
// Every job of `jobs` (device array, starts as prefix sums of items, `total` items) in one launch.
constexpr int PACK_MAX_JOBS = 256;
void pack_w_tc_batch(const float* params, const PackJob* jobs, int n_jobs, int64_t total, int mode, cudaStream_t st);

// Weight gradient of a strided conv from its row-packed form: dW2 [Co][s*ld][U] (the
// tensor-core weight gradient's (co, channel, tap) order) -> dW [Co][Ci][k], element
// (co, ci, u*s + j) = dW2 (co, j*ld + ci, u).
void wgrad_unpack_strided(const float* dW2, int Co, int Ci, int k, int s, int ld, float* dW, cudaStream_t st);

// ConvTranspose1d (weight W[Ci][Co][k], stride s, padding p, output length Lu)
// input and weight gradients as stride-1 problems over dy viewed row-packed:
//   dy2[b, m, j*Co + co] = dy[b, m*s + j, co]      (Lu % s == 0, compact rows)
// With t - p = u*s + j (0 <= j < s), u in [u_min, u_max]:
//   dx[q, ci]       = sum_{u, j, co} W[ci, co, u*s + j + p] * dy2[q + u, j*Co + co]
//   dW[ci, co, t]   = sum_q x[q, ci] * dy2[q + u, j*Co + co]
// i.e. a conv with taps = u_max - u_min + 1, padding -u_min and K = s*Co.
struct ConvTPack {
    int taps, u_min;
};
inline int floor_div(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }
inline ConvTPack convT_pack(int k, int s, int p) {
    const int u_min = floor_div(-p, s), u_max = floor_div(k - 1 - p, s);
    return ConvTPack{u_max - u_min + 1, u_min};
}

struct TcConvFwd {
    // activations (B, L_in, Ci) as planes
    TcPlanes x;
    int B = 0, L_in = 0, Ci = 0;
    // weights [taps][Co][Kp]
    TcPlanes w;
    int taps = 0, Co = 0;
    // geometry (stride 1): input row = (o + o_base) + t*d - p
    int p = 0, d = 1, No = 0, o_base = 0;
    // epilogue (as ConvFwd): y[b, (o+o_base)*orow_mul + orow_off, co] =
    //   alpha*(acc + bias + r[row >> r_shift]) + (accum ? y : 0)
    Act y;
    const float* bias = nullptr;
    const Act* r = nullptr;
    int r_shift = 0, orow_mul = 1, orow_off = 0;
    float alpha = 1.f;
    bool accum = false;
    // optional: stats[(b*Co + co)*2 + {0,1}] += sum, sum of squares of the
    // stored outputs over the rows this call writes (accum must be false)
    double* stats = nullptr;
    // optional split-K scratch (floats): a call with fewer output tiles than half
    // the SMs splits its K loop (input-channel chunks) over otherwise idle SMs,
    // writes fp32 partial tiles here and applies the epilogue in a reduce pass
    float* part = nullptr;
    int64_t part_cap = 0;
};
void conv_fwd_tc(const TcConvFwd& a, int mode, cudaStream_t st);
// scratch floats conv_fwd_tc would use for a split-K launch of `a` (0: no split)
int64_t conv_fwd_tc_part_floats(const TcConvFwd& a, int mode);

// Weight gradient of a stride-1 conv: dW[(co*Ci + ci)*taps + t] (+)=
//   sum_{b,o} dY[b, o, co] * X[b, o + t*d - p, ci]
// over operand planes of dY (B, Lo, Co) and X (B, L_in, Ci). Split-K partials
// go to `part` (at most part_cap floats) and are reduced in double.
struct TcConvWgrad {
    TcPlanes dy, x;
    int B = 0, Lo = 0, Co = 0, L_in = 0, Ci = 0;
    int taps = 1, p = 0, d = 1;
    // ConvTranspose1d mode (ct_s > 0): x is dy2 of ConvTPack (Ci = ct_s * ct_Co
    // row-packed channels), dy is the convT input, and dW is the convT weight
    // [Co][ct_Co][ct_k] (Co = convT input channels)
    int ct_s = 0, ct_p = 0, ct_k = 0, ct_Co = 0;
    float* dW = nullptr;
    bool accum = false;
};
void conv_wgrad_tc(const TcConvWgrad& a, int mode, float* part, int64_t part_cap, cudaStream_t st);

// Reads and clears the device error word the tensor-core kernels set when a
// bounded wait gives up (0 = no error). Synchronises the device.
int tc_error_flag();
// a kernel whose bounded wait runs out (about 2 s): checks the error-word path
void tc_wait_selftest(cudaStream_t st);

}  // namespace bsml
