// fp32 CUDA-core convolution kernels (channels-last). Used for every conv in
// BSML_MATH_FP32_SIMT mode and, in the tensor-core modes, for the shapes the
// tcgen05 kernels do not take (tiny channel counts: F0/N convs, conv_post,
// noise_convs, asr_res).
#include <algorithm>

#include "kernels.h"

namespace bsml {

namespace {

constexpr int TO = 64;    // output positions per CTA
constexpr int TC = 64;    // output channels per CTA
constexpr int KC = 16;    // input channels per K step

struct FwdK {
    const float* x; int64_t x_bs; int x_ld; int L_in; int Ci;
    const float* wp; const float* bias; int Co; int Cop; int k, s, p, d;
    int No, o_base;
    float* y; int64_t y_bs; int y_ld; int orow_mul, orow_off, y_rows;
    const float* r; int64_t r_bs; int r_ld; int r_shift;
    float alpha; int accum;
};

__global__ void __launch_bounds__(256) conv_fwd_kernel(FwdK a) {
    __shared__ float xs[KC][TO + 4];
    __shared__ __align__(16) float ws[KC][TC];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int o0 = blockIdx.x * TO, co0 = blockIdx.y * TC, b = blockIdx.z;
    const float* xb = a.x + (int64_t)b * a.x_bs;
    float acc[4][4] = {};
    for (int t = 0; t < a.k; ++t) {
        const int off = t * a.d - a.p;
        for (int ci0 = 0; ci0 < a.Ci; ci0 += KC) {
            // x tile: 64 rows x 16 channels; thread -> (row = tid/4, 4 channels)
            {
                const int ro = tid >> 2, c4 = (tid & 3) * 4;
                const int o = o0 + ro;
                const int li = (o + a.o_base) * a.s + off;
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                if (o < a.No && li >= 0 && li < a.L_in) {
                    const float* src = xb + (int64_t)li * a.x_ld + ci0 + c4;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (ci0 + c4 + j < a.Ci) v[j] = src[j];
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) xs[c4 + j][ro] = v[j];
            }
            // w tile: 16 ci x 64 co from wp[(t*Ci + ci)*Cop + co]
            {
                const int rc = tid >> 4, c4 = (tid & 15) * 4;
                const int ci = ci0 + rc, co = co0 + c4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (ci < a.Ci && co < a.Cop)
                    v = *reinterpret_cast<const float4*>(a.wp + ((int64_t)t * a.Ci + ci) * a.Cop + co);
                *reinterpret_cast<float4*>(&ws[rc][c4]) = v;
            }
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < KC; ++kk) {
                float xv[4], wv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) xv[i] = xs[kk][ty * 4 + i];
                const float4 w4 = *reinterpret_cast<const float4*>(&ws[kk][tx * 4]);
                wv[0] = w4.x; wv[1] = w4.y; wv[2] = w4.z; wv[3] = w4.w;
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(xv[i], wv[j], acc[i][j]);
            }
            __syncthreads();
        }
    }
    // epilogue
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int o = o0 + ty * 4 + i;
        if (o >= a.No) continue;
        const int row = (o + a.o_base) * a.orow_mul + a.orow_off;
        if (row < 0 || row >= a.y_rows) continue;
        float* yr = a.y + (int64_t)b * a.y_bs + (int64_t)row * a.y_ld;
        const float* rr = a.r ? a.r + (int64_t)b * a.r_bs + (int64_t)(row >> a.r_shift) * a.r_ld : nullptr;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int co = co0 + tx * 4 + j;
            if (co >= a.Co) continue;
            float v = acc[i][j];
            if (a.bias) v += a.bias[co];
            if (rr) v += rr[co];
            v *= a.alpha;
            if (a.accum) v += yr[co];
            yr[co] = v;
        }
    }
}

// ── weight gradient: M = co (64), N = ci (64), K = (b, o) rows, split-K partials
constexpr int WR = 16;    // rows per K step

struct WgK {
    const float* dy; int64_t dy_bs; int dy_ld; int Lo; int Co;
    const float* x; int64_t x_bs; int x_ld; int L_in; int Ci;
    int k, s, p, d, B;
    int64_t rows_total; int rows_per_split;
    float* part;   // [split][Co][Ci][k]
};

__global__ void __launch_bounds__(256) conv_wgrad_kernel(WgK a) {
    __shared__ __align__(16) float gs[WR][TC];
    __shared__ __align__(16) float xs[WR][TC];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int co0 = blockIdx.x * TC;
    const int nci = (a.Ci + TC - 1) / TC;
    const int t = blockIdx.y / nci, ci0 = (blockIdx.y % nci) * TC;
    const int split = blockIdx.z;
    const int64_t r0 = (int64_t)split * a.rows_per_split;
    const int64_t r1 = min(a.rows_total, r0 + a.rows_per_split);
    const int off = t * a.d - a.p;
    float acc[4][4] = {};
    for (int64_t rb = r0; rb < r1; rb += WR) {
        // load 16 rows x 64 channels of dy and x
        {
            const int rr = tid >> 4, c4 = (tid & 15) * 4;
            const int64_t row = rb + rr;
            float gv[4] = {0.f, 0.f, 0.f, 0.f}, xv[4] = {0.f, 0.f, 0.f, 0.f};
            if (row < r1) {
                const int b = (int)(row / a.Lo), o = (int)(row % a.Lo);
                const float* g = a.dy + (int64_t)b * a.dy_bs + (int64_t)o * a.dy_ld + co0 + c4;
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (co0 + c4 + j < a.Co) gv[j] = g[j];
                const int li = o * a.s + off;
                if (li >= 0 && li < a.L_in) {
                    const float* xp = a.x + (int64_t)b * a.x_bs + (int64_t)li * a.x_ld + ci0 + c4;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (ci0 + c4 + j < a.Ci) xv[j] = xp[j];
                }
            }
            *reinterpret_cast<float4*>(&gs[rr][c4]) = make_float4(gv[0], gv[1], gv[2], gv[3]);
            *reinterpret_cast<float4*>(&xs[rr][c4]) = make_float4(xv[0], xv[1], xv[2], xv[3]);
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < WR; ++kk) {
            const float4 g4 = *reinterpret_cast<const float4*>(&gs[kk][ty * 4]);
            const float4 x4 = *reinterpret_cast<const float4*>(&xs[kk][tx * 4]);
            const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(gv[i], xv[j], acc[i][j]);
        }
        __syncthreads();
    }
    float* pp = a.part + (int64_t)split * a.Co * a.Ci * a.k;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int co = co0 + ty * 4 + i;
        if (co >= a.Co) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int ci = ci0 + tx * 4 + j;
            if (ci >= a.Ci) continue;
            pp[((int64_t)co * a.Ci + ci) * a.k + t] = acc[i][j];
        }
    }
}

__global__ void reduce_splits_kernel(const float* part, int splits, int64_t n, float* out, int accum) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const double s = sum_strided(part + i, n, splits);
        out[i] = (float)(accum ? out[i] + s : s);
    }
}

__global__ void colsum_kernel(const float* dy, int64_t bs, int ld, int L, int C, int B, int rows_per_split,
                              float* part) {
    const int split = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const int64_t total = (int64_t)B * L;
    const int64_t r0 = (int64_t)split * rows_per_split, r1 = min(total, r0 + rows_per_split);
    double s = 0;
    for (int64_t r = r0; r < r1; ++r) {
        const int b = (int)(r / L), l = (int)(r % L);
        s += dy[(int64_t)b * bs + (int64_t)l * ld + c];
    }
    part[(int64_t)split * C + c] = (float)s;
}

// ~512 rows per split, at most 256 splits, and at most 48M partial floats
int wgrad_splits(int64_t rows, int64_t wsize) {
    int64_t sp = ceil_div(rows, 512);
    if (sp > 256) sp = 256;
    const int64_t cap = (48ll << 20) / (wsize > 0 ? wsize : 1);
    if (sp > cap) sp = cap;
    return (int)(sp < 1 ? 1 : sp);
}

// ── packing
__global__ void pack_conv_fwd_kernel(const float* W, int Co, int Ci, int k, int Cop, float* wp) {
    const int64_t n = (int64_t)k * Ci * Cop;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int co = (int)(i % Cop);
        const int64_t r = i / Cop;
        const int ci = (int)(r % Ci), t = (int)(r / Ci);
        wp[i] = co < Co ? W[((int64_t)co * Ci + ci) * k + t] : 0.f;
    }
}
// dgrad as a forward conv over dy: out channel = ci, in channel = co, tap t' = k-1-t
__global__ void pack_conv_dgrad_kernel(const float* W, int Co, int Ci, int k, int Cip, float* wp) {
    const int64_t n = (int64_t)k * Co * Cip;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int ci = (int)(i % Cip);
        const int64_t r = i / Cip;
        const int co = (int)(r % Co), tp = (int)(r / Co);
        wp[i] = ci < Ci ? W[((int64_t)co * Ci + ci) * k + (k - 1 - tp)] : 0.f;
    }
}
// convT phase r: Wr[m'][ci][co] = W[ci][co][r + (kr-1-m')*s], kr = taps in this phase
__global__ void pack_convT_phase_kernel(const float* W, int Ci, int Co, int k, int s, int r, int kr, int Cop, float* wp) {
    const int64_t n = (int64_t)kr * Ci * Cop;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int co = (int)(i % Cop);
        const int64_t q = i / Cop;
        const int ci = (int)(q % Ci), mp = (int)(q / Ci);
        const int t = r + (kr - 1 - mp) * s;
        wp[i] = co < Co ? W[((int64_t)ci * Co + co) * k + t] : 0.f;
    }
}
// convT dgrad = forward conv over dy with weight (out = ci, in = co): Wp[t][co][ci] = W[ci][co][t]
__global__ void pack_convT_dgrad_kernel(const float* W, int Ci, int Co, int k, int Cip, float* wp) {
    const int64_t n = (int64_t)k * Co * Cip;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int ci = (int)(i % Cip);
        const int64_t q = i / Cip;
        const int co = (int)(q % Co), t = (int)(q / Co);
        wp[i] = ci < Ci ? W[((int64_t)ci * Co + co) * k + t] : 0.f;
    }
}

inline int grid_for(int64_t n, int threads = 256) {
    int64_t g = ceil_div(n, threads);
    if (g > 148 * 16) g = 148 * 16;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace

void conv_fwd_simt(const ConvFwd& c, cudaStream_t st) {
    if (c.No <= 0) return;
    FwdK a;
    a.x = c.x.p; a.x_bs = c.x.bstride; a.x_ld = c.x.ld; a.L_in = c.x.L; a.Ci = c.x.C;
    a.wp = c.wp; a.bias = c.bias; a.Co = c.y.C; a.Cop = (int)round_up(c.y.C, 4);
    a.k = c.k; a.s = c.s; a.p = c.p; a.d = c.d;
    a.No = c.No; a.o_base = c.o_base;
    a.y = c.y.p; a.y_bs = c.y.bstride; a.y_ld = c.y.ld; a.orow_mul = c.orow_mul; a.orow_off = c.orow_off;
    a.y_rows = c.y.L;
    a.r = c.r ? c.r->p : nullptr; a.r_bs = c.r ? c.r->bstride : 0; a.r_ld = c.r ? c.r->ld : 0; a.r_shift = c.r_shift;
    a.alpha = c.alpha; a.accum = c.accum ? 1 : 0;
    dim3 grid((unsigned)ceil_div(c.No, TO), (unsigned)ceil_div(c.y.C, TC), (unsigned)c.x.B);
    ::bsml::count_launch();
    conv_fwd_kernel<<<grid, 256, 0, st>>>(a);
    BSML_LAUNCH("conv_fwd_simt");
}

int64_t wgrad_partial_floats(const ConvWgrad& c) {
    const int64_t ws = (int64_t)c.dy.C * c.x.C * c.k;
    return (int64_t)wgrad_splits((int64_t)c.dy.B * c.dy.L, ws) * ws;
}

void conv_wgrad_simt(const ConvWgrad& c, float* part, cudaStream_t st) {
    WgK a;
    a.dy = c.dy.p; a.dy_bs = c.dy.bstride; a.dy_ld = c.dy.ld; a.Lo = c.dy.L; a.Co = c.dy.C;
    a.x = c.x.p; a.x_bs = c.x.bstride; a.x_ld = c.x.ld; a.L_in = c.x.L; a.Ci = c.x.C;
    a.k = c.k; a.s = c.s; a.p = c.p; a.d = c.d; a.B = c.dy.B;
    a.rows_total = (int64_t)c.dy.B * c.dy.L;
    const int sp = wgrad_splits(a.rows_total, (int64_t)a.Co * a.Ci * c.k);
    a.rows_per_split = (int)ceil_div(a.rows_total, sp);
    a.part = part;
    dim3 grid((unsigned)ceil_div(a.Co, TC), (unsigned)(ceil_div(a.Ci, TC) * c.k), (unsigned)sp);
    ::bsml::count_launch();
    conv_wgrad_kernel<<<grid, 256, 0, st>>>(a);
    BSML_LAUNCH("conv_wgrad_simt");
    const int64_t n = (int64_t)a.Co * a.Ci * c.k;
    ::bsml::count_launch();
    reduce_splits_kernel<<<grid_for(n), 256, 0, st>>>(part, sp, n, c.dW, c.accum ? 1 : 0);
    BSML_LAUNCH("reduce_splits");
    if (c.db) colsum(c.dy, c.db, c.accum, part, st);
}

// Column sums of a channels-last tensor: 256-row chunks, 4 warps per CTA, each
// lane owning 4 consecutive channels (float4 loads, coalesced 512-byte rows),
// fp32 within a chunk, double across chunks.
namespace {
constexpr int CS_ROWS = 256;
__global__ void __launch_bounds__(128) colsum_chunk_kernel(const float* dy, int64_t bs, int ld, int L, int C,
                                                          int64_t rows, float* part) {
    __shared__ float red[4][128];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c0 = blockIdx.y * 128 + lane * 4;
    const int64_t r0 = (int64_t)blockIdx.x * CS_ROWS;
    const int64_t r1 = min(rows, r0 + CS_ROWS);
    float s[4] = {0.f, 0.f, 0.f, 0.f};
    const bool vec = (c0 + 3 < C) && ((ld & 3) == 0);
    for (int64_t r = r0 + warp; r < r1; r += 4) {
        const int b = (int)(r / L), l = (int)(r - (int64_t)b * L);
        const float* p = dy + (int64_t)b * bs + (int64_t)l * ld + c0;
        if (vec) {
            const float4 v = *reinterpret_cast<const float4*>(p);
            s[0] += v.x; s[1] += v.y; s[2] += v.z; s[3] += v.w;
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (c0 + j < C) s[j] += p[j];
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[warp][lane * 4 + j] = s[j];
    __syncthreads();
    const int c = blockIdx.y * 128 + threadIdx.x;
    if (c < C) part[(int64_t)blockIdx.x * C + c] = red[0][threadIdx.x] + red[1][threadIdx.x] + red[2][threadIdx.x] +
                                                   red[3][threadIdx.x];
}
// out[c] (+)= sum over the chunk partials part[q][c]: 32 channels per CTA, 32 rows of
// threads taking every 32nd chunk (a fixed order), then a tree over the rows in
// shared memory; double throughout
__global__ void __launch_bounds__(1024) colsum_reduce_kernel(const float* part, int chunks, int C, float* out,
                                                            int accum) {
    __shared__ double red[32][33];
    const int c = blockIdx.x * 32 + threadIdx.x;
    double s = 0.0;
    if (c < C) {
        const int n = chunks > (int)threadIdx.y ? (chunks - (int)threadIdx.y + 31) / 32 : 0;
        s = sum_strided(part + (int64_t)threadIdx.y * C + c, 32ll * C, n);
    }
    red[threadIdx.y][threadIdx.x] = s;
    __syncthreads();
    for (int h = 16; h > 0; h >>= 1) {
        if ((int)threadIdx.y < h) red[threadIdx.y][threadIdx.x] += red[threadIdx.y + h][threadIdx.x];
        __syncthreads();
    }
    if (threadIdx.y == 0 && c < C) out[c] = (float)(accum ? out[c] + red[0][threadIdx.x] : red[0][threadIdx.x]);
}
}  // namespace

void colsum(const Act& dy, float* db, bool accum, float* part, cudaStream_t st) {
    const int64_t rows = (int64_t)dy.B * dy.L;
    const int chunks = (int)ceil_div(rows, CS_ROWS);
    dim3 grid((unsigned)chunks, (unsigned)ceil_div(dy.C, 128));
    ::bsml::count_launch();
    colsum_chunk_kernel<<<grid, 128, 0, st>>>(dy.p, dy.bstride, dy.ld, dy.L, dy.C, rows, part);
    BSML_LAUNCH("colsum");
    ::bsml::count_launch();
    colsum_reduce_kernel<<<(unsigned)ceil_div(dy.C, 32), dim3(32, 32), 0, st>>>(part, chunks, dy.C, db, accum ? 1 : 0);
    BSML_LAUNCH("colsum_reduce");
}

int64_t colsum_partial_floats(const Act& dy) { return ceil_div((int64_t)dy.B * dy.L, CS_ROWS) * dy.C; }

void pack_conv_fwd(const float* W, int Co, int Ci, int k, float* wp, cudaStream_t st) {
    const int Cop = (int)round_up(Co, 4);
    ::bsml::count_launch();
    pack_conv_fwd_kernel<<<grid_for((int64_t)k * Ci * Cop), 256, 0, st>>>(W, Co, Ci, k, Cop, wp);
    BSML_LAUNCH("pack_conv_fwd");
}
void pack_conv_dgrad(const float* W, int Co, int Ci, int k, float* wp, cudaStream_t st) {
    const int Cip = (int)round_up(Ci, 4);
    ::bsml::count_launch();
    pack_conv_dgrad_kernel<<<grid_for((int64_t)k * Co * Cip), 256, 0, st>>>(W, Co, Ci, k, Cip, wp);
    BSML_LAUNCH("pack_conv_dgrad");
}
void pack_convT_phase(const float* W, int Ci, int Co, int k, int s, int r, float* wp, cudaStream_t st) {
    const int kr = (k - r + s - 1) / s;
    const int Cop = (int)round_up(Co, 4);
    ::bsml::count_launch();
    pack_convT_phase_kernel<<<grid_for((int64_t)kr * Ci * Cop), 256, 0, st>>>(W, Ci, Co, k, s, r, kr, Cop, wp);
    BSML_LAUNCH("pack_convT_phase");
}
void pack_convT_dgrad(const float* W, int Ci, int Co, int k, float* wp, cudaStream_t st) {
    const int Cip = (int)round_up(Ci, 4);
    ::bsml::count_launch();
    pack_convT_dgrad_kernel<<<grid_for((int64_t)k * Co * Cip), 256, 0, st>>>(W, Ci, Co, k, Cip, wp);
    BSML_LAUNCH("pack_convT_dgrad");
}

}  // namespace bsml

namespace bsml {

bool conv_wgrad_simt_capped(const ConvWgrad& c, float* part, int64_t part_cap, cudaStream_t st) {
    const int64_t rows = (int64_t)c.dy.B * c.dy.L;
    const int64_t wsize = (int64_t)c.dy.C * c.x.C * c.k;
    int64_t sp = std::min<int64_t>(wgrad_splits(rows, wsize), part_cap / std::max<int64_t>(wsize, 1));
    int64_t sp_b = c.db ? std::min<int64_t>(wgrad_splits(rows, c.dy.C), part_cap / std::max(c.dy.C, 1)) : 1;
    if (sp < 1 || sp_b < 1) return false;
    WgK a;
    a.dy = c.dy.p; a.dy_bs = c.dy.bstride; a.dy_ld = c.dy.ld; a.Lo = c.dy.L; a.Co = c.dy.C;
    a.x = c.x.p; a.x_bs = c.x.bstride; a.x_ld = c.x.ld; a.L_in = c.x.L; a.Ci = c.x.C;
    a.k = c.k; a.s = c.s; a.p = c.p; a.d = c.d; a.B = c.dy.B;
    a.rows_total = rows;
    a.rows_per_split = (int)ceil_div(rows, sp);
    sp = ceil_div(rows, a.rows_per_split);
    a.part = part;
    dim3 grid((unsigned)ceil_div(a.Co, TC), (unsigned)(ceil_div(a.Ci, TC) * c.k), (unsigned)sp);
    ::bsml::count_launch();
    conv_wgrad_kernel<<<grid, 256, 0, st>>>(a);
    BSML_LAUNCH("conv_wgrad_simt_capped");
    ::bsml::count_launch();
    reduce_splits_kernel<<<grid_for(wsize), 256, 0, st>>>(part, (int)sp, wsize, c.dW, c.accum ? 1 : 0);
    BSML_LAUNCH("reduce_splits");
    if (c.db) {
        const int rps = (int)ceil_div(rows, sp_b);
        sp_b = ceil_div(rows, rps);
        dim3 g2((unsigned)ceil_div(c.dy.C, 128), (unsigned)sp_b);
        ::bsml::count_launch();
        colsum_kernel<<<g2, 128, 0, st>>>(c.dy.p, c.dy.bstride, c.dy.ld, c.dy.L, c.dy.C, c.dy.B, rps, part);
        ::bsml::count_launch();
        reduce_splits_kernel<<<grid_for(c.dy.C), 256, 0, st>>>(part, (int)sp_b, c.dy.C, c.db, c.accum ? 1 : 0);
        BSML_LAUNCH("colsum_capped");
    }
    return true;
}

}  // namespace bsml
