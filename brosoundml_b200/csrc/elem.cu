// Normalisation, activation, layout and small-op kernels (channels-last fp32).
#include <cmath>

#include <algorithm>

#include "kernels.h"

namespace bsml {

namespace {

inline int grid_for(int64_t n, int threads = 256) {
    int64_t g = ceil_div(n, threads);
    if (g > 148 * 32) g = 148 * 32;
    return (int)(g < 1 ? 1 : g);
}

// Row chunking for the per-(b, c) reductions: each CTA takes up to ROWS rows of
// one clip; threads own channels (coalesced across the warp).
constexpr int ROWS = 64;

__global__ void zero_d(double* p, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = 0.0;
}

__device__ __forceinline__ float act_fwd(float z, int act, float slope, float al) {
    if (act == ACT_LEAKY) return z > 0.f ? z : slope * z;
    if (act == ACT_SNAKE) {
        const float sn = sinf(al * z);
        return z + sn * sn / al;
    }
    return z;
}

__global__ void snake_fwd_kernel(Act x, const float* alpha, Act y) {
    const int64_t n = x.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % x.C);
        const int64_t r = i / x.C;
        const int l = (int)(r % x.L), b = (int)(r / x.L);
        y.row(b, l)[c] = act_fwd(x.row(b, l)[c], ACT_SNAKE, 0.f, alpha[c]);
    }
}

__global__ void snake_bwd_kernel(Act x, const float* alpha, Act dy, Act dx, double* acc) {
    const int b = blockIdx.y;
    const int l0 = blockIdx.x * ROWS, l1 = min(x.L, l0 + ROWS);
    for (int c = threadIdx.x; c < x.C; c += blockDim.x) {
        const float al = alpha[c];
        double s = 0;
        for (int l = l0; l < l1; ++l) {
            const float z = x.row(b, l)[c], g = dy.row(b, l)[c];
            const float sn = sinf(al * z), s2a = sinf(2.f * al * z);
            dx.row(b, l)[c] = g * (1.f + s2a);
            s += (double)g * (double)(z * s2a / al - sn * sn / (al * al));
        }
        atomicAdd(&acc[(int64_t)b * x.C + c], s);
    }
}

__global__ void snake_alpha_final_kernel(const double* acc, int B, int C, float* dalpha) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    double s = 0;
    for (int b = 0; b < B; ++b) s += acc[(int64_t)b * C + c];
    dalpha[c] = (float)s;
}

__global__ void leaky_kernel(Act x, float slope, Act y) {
    const int64_t n = x.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % x.C);
        const int64_t r = i / x.C;
        const int l = (int)(r % x.L), b = (int)(r / x.L);
        const float v = x.row(b, l)[c];
        y.row(b, l)[c] = v > 0.f ? v : slope * v;
    }
}

__global__ void leaky_bwd_kernel(Act x, float slope, Act dy, Act dx) {
    const int64_t n = x.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % x.C);
        const int64_t r = i / x.C;
        const int l = (int)(r % x.L), b = (int)(r / x.L);
        const float g = dy.row(b, l)[c];
        dx.row(b, l)[c] = x.row(b, l)[c] > 0.f ? g : slope * g;
    }
}

__global__ void copy_kernel(Act s, Act d) {
    const int64_t n = s.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % s.C);
        const int64_t r = i / s.C;
        const int l = (int)(r % s.L), b = (int)(r / s.L);
        d.row(b, l)[c] = s.row(b, l)[c];
    }
}

__global__ void add_kernel(Act s, Act d, float alpha) {
    const int64_t n = s.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % s.C);
        const int64_t r = i / s.C;
        const int l = (int)(r % s.L), b = (int)(r / s.L);
        d.row(b, l)[c] += alpha * s.row(b, l)[c];
    }
}

__global__ void scale_kernel(Act x, float alpha) {
    const int64_t n = x.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % x.C);
        const int64_t r = i / x.C;
        const int l = (int)(r % x.L), b = (int)(r / x.L);
        x.row(b, l)[c] *= alpha;
    }
}

__global__ void pair_sum_kernel(Act s, Act d) {
    const int64_t n = d.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % d.C);
        const int64_t r = i / d.C;
        const int l = (int)(r % d.L), b = (int)(r / d.L);
        d.row(b, l)[c] = s.row(b, 2 * l)[c] + s.row(b, 2 * l + 1)[c];
    }
}

__global__ void reflect_fwd_kernel(Act y) {
    const int64_t n = (int64_t)y.B * y.C;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % y.C), b = (int)(i / y.C);
        y.row(b, 0)[c] = y.row(b, 2)[c];
    }
}
__global__ void reflect_bwd_kernel(Act d) {
    const int64_t n = (int64_t)d.B * d.C;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % d.C), b = (int)(i / d.C);
        d.row(b, 2)[c] += d.row(b, 0)[c];
        d.row(b, 0)[c] = 0.f;
    }
}

// (B, C, L) <-> channels-last through 32x32 shared-memory tiles
__global__ void ncl_to_cl_kernel(const float* src, Act d) {
    __shared__ float tile[32][33];
    const int b = blockIdx.z;
    const int l0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int c = c0 + j, l = l0 + threadIdx.x;
        tile[j][threadIdx.x] = (c < d.C && l < d.L) ? src[((int64_t)b * d.C + c) * d.L + l] : 0.f;
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int l = l0 + j, c = c0 + threadIdx.x;
        if (c < d.C && l < d.L) d.row(b, l)[c] = tile[threadIdx.x][j];
    }
}
__global__ void cl_to_ncl_kernel(Act s, float* dst) {
    __shared__ float tile[32][33];
    const int b = blockIdx.z;
    const int l0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int l = l0 + j, c = c0 + threadIdx.x;
        tile[j][threadIdx.x] = (c < s.C && l < s.L) ? s.row(b, l)[c] : 0.f;
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int c = c0 + j, l = l0 + threadIdx.x;
        if (c < s.C && l < s.L) dst[((int64_t)b * s.C + c) * s.L + l] = tile[threadIdx.x][j];
    }
}

__global__ void fill_kernel(float* p, int64_t n, float v) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = v;
}

// depthwise ConvTranspose1d: y[b,j,c] = bias[c] + sum_{t,l: j = l*s - p + t} W[c,t] x[b,l,c]
__global__ void dwconvT_fwd_kernel(Act x, const float* W, const float* bias, int k, int s, int p, Act y) {
    const int64_t n = y.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % y.C);
        const int64_t r = i / y.C;
        const int j = (int)(r % y.L), b = (int)(r / y.L);
        float v = bias ? bias[c] : 0.f;
        for (int t = 0; t < k; ++t) {
            const int num = j + p - t;
            if (num < 0 || num % s) continue;
            const int l = num / s;
            if (l < x.L) v += W[c * k + t] * x.row(b, l)[c];
        }
        y.row(b, j)[c] = v;
    }
}
__global__ void dwconvT_dgrad_kernel(Act dy, const float* W, int k, int s, int p, Act dx) {
    const int64_t n = dx.numel();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % dx.C);
        const int64_t r = i / dx.C;
        const int l = (int)(r % dx.L), b = (int)(r / dx.L);
        float v = 0.f;
        for (int t = 0; t < k; ++t) {
            const int j = l * s - p + t;
            if (j >= 0 && j < dy.L) v += W[c * k + t] * dy.row(b, j)[c];
        }
        dx.row(b, l)[c] = v;
    }
}
// one thread per (c, t) + bias; rows reduced serially in double (C*k small)
// dW[c*k + t] += sum over a chunk of input rows (b, l) of x[b, l, c] * dy[b, l*s - p + t, c]
constexpr int DW_MAXK = 8;
__global__ void dwconvT_wgrad_kernel(Act dy, Act x, int k, int s, int p, int rows_per, double* acc) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= x.C) return;
    const int r0 = blockIdx.y * rows_per, r1 = min(x.B * x.L, r0 + rows_per);
    double a[DW_MAXK] = {};
    for (int r = r0; r < r1; ++r) {
        const int b = r / x.L, l = r - b * x.L;
        const double xv = x.row(b, l)[c];
#pragma unroll
        for (int t = 0; t < DW_MAXK; ++t) {
            const int j = l * s - p + t;
            if (t < k && j >= 0 && j < dy.L) a[t] += xv * (double)dy.row(b, j)[c];
        }
    }
#pragma unroll
    for (int t = 0; t < DW_MAXK; ++t)
        if (t < k) atomicAdd(&acc[(int64_t)c * k + t], a[t]);
}

// d (op)= s on 4-channel groups (128-bit loads / stores), one clip per blockIdx.y
enum { EW_COPY = 0, EW_ADD = 1, EW_SCALE = 2 };
template <int OP>
__global__ void ew4_kernel(Act s, Act d, float alpha) {
    const int b = blockIdx.y;
    const int C4 = (s.C + 3) >> 2, n = s.L * C4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const int l = i / C4, c = 4 * (i - l * C4), nv = min(4, s.C - c);
        const float4 a = *reinterpret_cast<const float4*>(s.row(b, l) + c);
        float4 r = a;
        if (OP == EW_ADD) {
            const float4 o = *reinterpret_cast<const float4*>(d.row(b, l) + c);
            r = make_float4(fmaf(alpha, a.x, o.x), fmaf(alpha, a.y, o.y), fmaf(alpha, a.z, o.z), fmaf(alpha, a.w, o.w));
        } else if (OP == EW_SCALE) {
            r = make_float4(alpha * a.x, alpha * a.y, alpha * a.z, alpha * a.w);
        }
        float* dp = d.row(b, l) + c;
        if (nv == 4) {
            *reinterpret_cast<float4*>(dp) = r;
        } else {
            dp[0] = r.x;
            if (nv > 1) dp[1] = r.y;
            if (nv > 2) dp[2] = r.z;
        }
    }
}

bool vec_ok(const Act& a) {
    return (reinterpret_cast<uintptr_t>(a.p) & 15) == 0 && (a.ld & 3) == 0 && (a.bstride & 3) == 0;
}

template <int OP>
void ew4(const Act& s, const Act& d, float alpha, cudaStream_t st) {
    const int64_t n = (int64_t)s.L * ceil_div(s.C, 4);
    const int gx = (int)std::min<int64_t>(std::max<int64_t>(ceil_div(n, 256), 1), std::max(1, 148 * 8 / std::max(s.B, 1)));
    ::bsml::count_launch();
    ew4_kernel<OP><<<dim3((unsigned)gx, (unsigned)s.B), 256, 0, st>>>(s, d, alpha);
    BSML_LAUNCH("ew4");
}

// ── AdaIN fc: one warp per output row o of every AdaIN, all clips
__global__ void fc_fwd_kernel(const FcRow* tab, int total_rows, const int* row_entry, const float* P,
                              const float* style, int B, int S, float* out) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= total_rows) return;
    const int e = row_entry[warp];
    const FcRow f = tab[e];
    const int o = warp - f.row0;   // local row within this AdaIN's fc
    const float* w = P + f.w_off + (int64_t)o * S;
    for (int b = 0; b < B; ++b) {
        float s = 0.f;
        for (int i = lane; i < S; i += 32) s += w[i] * style[b * S + i];
#pragma unroll
        for (int q = 16; q > 0; q >>= 1) s += __shfl_xor_sync(0xffffffffu, s, q);
        if (lane == 0) out[f.out_off + (int64_t)b * f.n_out + o] = s + P[f.b_off + o];
    }
}

// dW[o, i] = sum_b daff[b, o] style[b, i]; db[o] = sum_b daff[b, o]
__global__ void fc_bwd_w_kernel(const FcRow* tab, int total_rows, const int* row_entry, const float* style,
                                const float* daff, int B, int S, float* G) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= total_rows) return;
    const FcRow f = tab[row_entry[warp]];
    const int o = warp - f.row0;
    for (int i = lane; i < S; i += 32) {
        double s = 0;
        for (int b = 0; b < B; ++b) s += (double)daff[f.out_off + (int64_t)b * f.n_out + o] * style[b * S + i];
        G[f.w_off + (int64_t)o * S + i] = (float)s;
    }
    if (lane == 0) {
        double s = 0;
        for (int b = 0; b < B; ++b) s += daff[f.out_off + (int64_t)b * f.n_out + o];
        G[f.b_off + o] = (float)s;
    }
}

// d_style[b, i] partials over row chunks: part[chunk][b][i]. FC_RY rows of a chunk are
// walked at once (threadIdx.y), each row's weights loaded once per FC_CLIPS clips and
// applied to them from registers; the row lanes are summed in shared memory at the end.
constexpr int FC_CHUNK = 256;
constexpr int FC_CLIPS = 8;
constexpr int FC_RY = 8;
__global__ void fc_bwd_style_kernel(const FcRow* tab, int total_rows, const int* row_entry, const float* P,
                                    const float* daff, int B, int S, float* part) {
    __shared__ float red[FC_RY][FC_CLIPS][128];
    const int chunk = blockIdx.x;
    const int x = threadIdx.x, y = threadIdx.y;   // blockDim.x <= 128
    const int r0 = chunk * FC_CHUNK, r1 = min(total_rows, r0 + FC_CHUNK);
    for (int i0 = 0; i0 < S; i0 += blockDim.x)
    for (int b0 = 0; b0 < B; b0 += FC_CLIPS) {
        const int i = i0 + x;
        const int nb = min(FC_CLIPS, B - b0);
        float s[FC_CLIPS] = {};
        if (i < S)
            for (int r = r0 + y; r < r1; r += FC_RY) {
                const FcRow f = tab[row_entry[r]];
                const int o = r - f.row0;
                const float p = P[f.w_off + (int64_t)o * S + i];
                const float* d = daff + f.out_off + (int64_t)b0 * f.n_out + o;
#pragma unroll
                for (int u = 0; u < FC_CLIPS; ++u)
                    if (u < nb) s[u] = fmaf(p, d[(int64_t)u * f.n_out], s[u]);
            }
#pragma unroll
        for (int u = 0; u < FC_CLIPS; ++u) red[y][u][x] = s[u];
        __syncthreads();
        if (y == 0 && i < S)
            for (int u = 0; u < nb; ++u) {
                float t = 0.f;
#pragma unroll
                for (int q = 0; q < FC_RY; ++q) t += red[q][u][x];
                part[((int64_t)chunk * B + b0 + u) * S + i] = t;
            }
        __syncthreads();
    }
}
__global__ void fc_style_reduce_kernel(const float* part, int chunks, int n, float* d_style) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    double s = 0;
    for (int q = 0; q < chunks; ++q) s += part[(int64_t)q * n + i];
    d_style[i] = (float)s;
}

}  // namespace

void snake_fwd(const Act& x, const float* alpha, const Act& y, cudaStream_t st) {
    ::bsml::count_launch();
    snake_fwd_kernel<<<grid_for(x.numel()), 256, 0, st>>>(x, alpha, y);
    BSML_LAUNCH("snake_fwd");
}
void snake_bwd(const Act& x, const float* alpha, const Act& dy, const Act& dx, float* dalpha, double* acc,
               cudaStream_t st) {
    const int64_t n = (int64_t)x.B * x.C;
    ::bsml::count_launch();
    zero_d<<<grid_for(n), 256, 0, st>>>(acc, n);
    dim3 grid((unsigned)ceil_div(x.L, ROWS), (unsigned)x.B);
    ::bsml::count_launch();
    snake_bwd_kernel<<<grid, x.C >= 256 ? 256 : (int)round_up(x.C, 32), 0, st>>>(x, alpha, dy, dx, acc);
    ::bsml::count_launch();
    snake_alpha_final_kernel<<<(unsigned)ceil_div(x.C, 128), 128, 0, st>>>(acc, x.B, x.C, dalpha);
    BSML_LAUNCH("snake_bwd");
}

void leaky_fwd(const Act& x, float slope, const Act& y, cudaStream_t st) {
    ::bsml::count_launch();
    leaky_kernel<<<grid_for(x.numel()), 256, 0, st>>>(x, slope, y);
    BSML_LAUNCH("leaky_fwd");
}
void leaky_bwd(const Act& x, float slope, const Act& dy, const Act& dx, cudaStream_t st) {
    ::bsml::count_launch();
    leaky_bwd_kernel<<<grid_for(x.numel()), 256, 0, st>>>(x, slope, dy, dx);
    BSML_LAUNCH("leaky_bwd");
}
void copy_act(const Act& s, const Act& d, cudaStream_t st) {
    if (s.numel() > 0 && vec_ok(s) && vec_ok(d)) return ew4<EW_COPY>(s, d, 1.f, st);
    ::bsml::count_launch();
    copy_kernel<<<grid_for(s.numel()), 256, 0, st>>>(s, d);
    BSML_LAUNCH("copy_act");
}
void add_act(const Act& s, const Act& d, float alpha, cudaStream_t st) {
    if (s.numel() > 0 && vec_ok(s) && vec_ok(d)) return ew4<EW_ADD>(s, d, alpha, st);
    ::bsml::count_launch();
    add_kernel<<<grid_for(s.numel()), 256, 0, st>>>(s, d, alpha);
    BSML_LAUNCH("add_act");
}
void scale_act(const Act& x, float alpha, cudaStream_t st) {
    if (x.numel() > 0 && vec_ok(x)) return ew4<EW_SCALE>(x, x, alpha, st);
    ::bsml::count_launch();
    scale_kernel<<<grid_for(x.numel()), 256, 0, st>>>(x, alpha);
    BSML_LAUNCH("scale_act");
}
void pair_sum_rows(const Act& s, const Act& d, cudaStream_t st) {
    ::bsml::count_launch();
    pair_sum_kernel<<<grid_for(d.numel()), 256, 0, st>>>(s, d);
    BSML_LAUNCH("pair_sum_rows");
}
void reflect_left1_fwd(const Act& y, cudaStream_t st) {
    ::bsml::count_launch();
    reflect_fwd_kernel<<<grid_for((int64_t)y.B * y.C), 256, 0, st>>>(y);
    BSML_LAUNCH("reflect_left1_fwd");
}
void reflect_left1_bwd(const Act& d, cudaStream_t st) {
    ::bsml::count_launch();
    reflect_bwd_kernel<<<grid_for((int64_t)d.B * d.C), 256, 0, st>>>(d);
    BSML_LAUNCH("reflect_left1_bwd");
}
void ncl_to_cl(const float* src, const Act& d, cudaStream_t st) {
    dim3 grid((unsigned)ceil_div(d.L, 32), (unsigned)ceil_div(d.C, 32), (unsigned)d.B);
    ::bsml::count_launch();
    ncl_to_cl_kernel<<<grid, dim3(32, 8), 0, st>>>(src, d);
    BSML_LAUNCH("ncl_to_cl");
}
void cl_to_ncl(const Act& s, float* dst, cudaStream_t st) {
    dim3 grid((unsigned)ceil_div(s.L, 32), (unsigned)ceil_div(s.C, 32), (unsigned)s.B);
    ::bsml::count_launch();
    cl_to_ncl_kernel<<<grid, dim3(32, 8), 0, st>>>(s, dst);
    BSML_LAUNCH("cl_to_ncl");
}
void fill(float* p, int64_t n, float v, cudaStream_t st) {
    if (n <= 0) return;
    ::bsml::count_launch();
    fill_kernel<<<grid_for(n), 256, 0, st>>>(p, n, v);
    BSML_LAUNCH("fill");
}
void dwconvT_fwd(const Act& x, const float* W, const float* bias, int k, int s, int p, const Act& y, cudaStream_t st) {
    ::bsml::count_launch();
    dwconvT_fwd_kernel<<<grid_for(y.numel()), 256, 0, st>>>(x, W, bias, k, s, p, y);
    BSML_LAUNCH("dwconvT_fwd");
}
void dwconvT_dgrad(const Act& dy, const float* W, int k, int s, int p, const Act& dx, cudaStream_t st) {
    ::bsml::count_launch();
    dwconvT_dgrad_kernel<<<grid_for(dx.numel()), 256, 0, st>>>(dy, W, k, s, p, dx);
    BSML_LAUNCH("dwconvT_dgrad");
}
void dwconvT_wgrad(const Act& dy, const Act& x, int k, int s, int p, float* dW, float* db, double* acc,
                   float* part, cudaStream_t st) {
    if (k > DW_MAXK) fail("dwconvT_wgrad", "kernel size above 8");
    BSML_CUDA(cudaMemsetAsync(acc, 0, sizeof(double) * x.C * k, st));
    const int rows_per = 64;
    dim3 grid((unsigned)ceil_div(x.C, 128), (unsigned)ceil_div((int64_t)x.B * x.L, rows_per));
    ::bsml::count_launch();
    dwconvT_wgrad_kernel<<<grid, 128, 0, st>>>(dy, x, k, s, p, rows_per, acc);
    BSML_LAUNCH("dwconvT_wgrad");
    d2f(acc, x.C * k, dW, false, st);
    if (db) colsum(dy, db, false, part, st);
}

void affine_fc_fwd(const FcRow* table, int n_entries, int total_rows, const int* row_entry, const float* params,
                   const float* style, int B, int S, float* out, cudaStream_t st) {
    (void)n_entries;
    ::bsml::count_launch();
    fc_fwd_kernel<<<(unsigned)ceil_div((int64_t)total_rows * 32, 256), 256, 0, st>>>(table, total_rows, row_entry,
                                                                                       params, style, B, S, out);
    BSML_LAUNCH("affine_fc_fwd");
}

void affine_fc_bwd(const FcRow* table, int n_entries, int total_rows, const int* row_entry, const float* params,
                   const float* style, const float* daff, int B, int S, float* grads, float* d_style, float* part,
                   cudaStream_t st) {
    (void)n_entries;
    if (grads) {
        ::bsml::count_launch();
        fc_bwd_w_kernel<<<(unsigned)ceil_div((int64_t)total_rows * 32, 256), 256, 0, st>>>(
            table, total_rows, row_entry, style, daff, B, S, grads);
    }
    if (d_style) {
        const int chunks = (int)ceil_div(total_rows, FC_CHUNK);
        ::bsml::count_launch();
        fc_bwd_style_kernel<<<chunks, dim3((unsigned)std::min(round_up(S, 32), (int64_t)128), FC_RY), 0, st>>>(
            table, total_rows, row_entry, params, daff, B, S, part);
        ::bsml::count_launch();
        fc_style_reduce_kernel<<<(unsigned)ceil_div(B * S, 128), 128, 0, st>>>(part, chunks, B * S, d_style);
    }
    BSML_LAUNCH("affine_fc_bwd");
}

}  // namespace bsml
