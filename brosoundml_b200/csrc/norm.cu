// Instance-norm / AdaIN + activation kernels, forward and backward, fused with
// the operand-plane output the tensor-core convolutions read and with the
// per-channel column sums of the produced tensor (the following conv's bias
// gradient). These are the reference's adain_affine_forward / _backward and
// snake_forward / _backward (src/kokoro_decoder_backward.h:37-56,
// src/kokoro_decoder_backward.cpp:305,352) applied batched on channels-last
// buffers.
//
// Geometry: one CTA takes a run of rows of one clip (blockIdx.y = b). The block
// is 2-D: threadIdx.x walks 4-channel groups (128-bit loads and stores),
// threadIdx.y walks rows, so each thread keeps its channels' constants in
// registers while streaming down the rows. Row reductions are summed per thread
// in double, combined across threadIdx.y in shared memory and added to the
// per-(b, c) accumulators with one double atomic per channel and CTA.
#include <algorithm>
#include <cmath>

#include "kernels.h"
#include "planes.cuh"

namespace bsml {

namespace {

constexpr int NT = 256;   // threads per CTA
constexpr int UNR = 4;    // rows whose loads a thread issues before it stores (memory-level parallelism)
// the two passes of the AdaIN backward trade occupancy for loads in flight: 2 CTAs
// per SM with more rows each measured faster on B200 than 3-4 CTAs with fewer
constexpr int RR_UNR = 6;    // adain_recompute_reduce_kernel: rows of (x, dy) loads in flight
constexpr int APPLY_ROWS = 4;  // adain_bwd_apply_kernel: rows of (x, dy, skip) loads in flight

struct Out4 {
    float* y = nullptr; int64_t y_bs = 0; int y_ld = 0;                 // fp32 output (nullable)
    void* hi = nullptr; void* lo = nullptr; int64_t p_bs = 0; int p_ld = 0; int mode = 1;   // planes (nullable)
    const float* skip = nullptr; int64_t s_bs = 0; int s_ld = 0;       // added before the store (nullable)
    float s_scale = 1.f;                                                // factor on skip
    void* hi2 = nullptr; void* lo2 = nullptr; int64_t p_bs2 = 0; int p_ld2 = 0; int mode2 = 1;   // second planes
};

__device__ __forceinline__ void put(const Out4& o, int b, int l, int c, const float4& v, int nv) {
    if (o.y) st4(o.y + (int64_t)b * o.y_bs + (int64_t)l * o.y_ld + c, v, nv);
    if (o.hi) st_planes4(o.hi, o.lo, o.mode, (int64_t)b * o.p_bs + (int64_t)l * o.p_ld + c, v, nv);
    if (o.hi2) st_planes4(o.hi2, o.lo2, o.mode2, (int64_t)b * o.p_bs2 + (int64_t)l * o.p_ld2 + c, v, nv);
}

// Adds the per-thread partials s[k][j] (k < NS sums, j < 4 channels of group v)
// over threadIdx.y and then, one atomic per channel, into dst[c * NS + k].
template <int NS>
__device__ __forceinline__ void combine_rows(double (&s)[NS][4], int v, int C4, int C, double* dst) {
    __shared__ double red[NS * 4 * NT];
    const int tid = threadIdx.y * blockDim.x + threadIdx.x;
    if (blockDim.y > 1) {
#pragma unroll
        for (int k = 0; k < NS; ++k)
#pragma unroll
            for (int j = 0; j < 4; ++j) red[(k * 4 + j) * NT + tid] = s[k][j];
        __syncthreads();
        if (threadIdx.y == 0) {
            for (int y = 1; y < (int)blockDim.y; ++y)
#pragma unroll
                for (int k = 0; k < NS; ++k)
#pragma unroll
                    for (int j = 0; j < 4; ++j) s[k][j] += red[(k * 4 + j) * NT + y * blockDim.x + threadIdx.x];
        }
    }
    if (threadIdx.y == 0 && v < C4) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (4 * v + j < C)
#pragma unroll
                for (int k = 0; k < NS; ++k) atomicAdd(&dst[(int64_t)(4 * v + j) * NS + k], s[k][j]);
    }
    if (blockDim.y > 1) __syncthreads();
}

// sums[(b*C + c)*2 + {0,1}] += sum_l x, sum_l x^2
__global__ void __launch_bounds__(NT) sums_kernel(Act x, int rows, double* sums) {
    const int b = blockIdx.y;
    const int l0 = blockIdx.x * rows, l1 = min(x.L, l0 + rows);
    const int C4 = (x.C + 3) >> 2;
    for (int v0 = 0; v0 < C4; v0 += blockDim.x) {
        const int v = v0 + threadIdx.x;
        double s[2][4] = {};
        if (v < C4) {
            const float* base = x.p + (int64_t)b * x.bstride + 4 * v;
            const int dl = blockDim.y;
            int l = l0 + threadIdx.y;
            for (; l + 3 * dl < l1; l += 4 * dl) {
                float4 a[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) a[u] = ldg4(base + (int64_t)(l + u * dl) * x.ld);
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const double e = get(a[u], j);
                        s[0][j] += e;
                        s[1][j] = fma(e, e, s[1][j]);
                    }
            }
            for (; l < l1; l += dl) {
                const float4 a = ldg4(base + (int64_t)l * x.ld);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const double e = get(a, j);
                    s[0][j] += e;
                    s[1][j] = fma(e, e, s[1][j]);
                }
            }
        }
        combine_rows<2>(s, v, C4, x.C, sums + (int64_t)b * x.C * 2);
    }
}

__global__ void stats_final_kernel(const double* acc, int64_t n, int L, float eps, float* mean, float* rstd) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const double m = acc[2 * i] / L;
        double v = acc[2 * i + 1] / L - m * m;
        v = v > 0 ? v : 0;
        mean[i] = (float)m;
        rstd[i] = (float)(1.0 / sqrt(v + (double)eps));
    }
}

// Per-channel constants of one 4-channel group.
struct Chan {
    float m[4], rs[4], g1[4], be[4], al[4], ial[4];
};

// With sums: mean / rstd from the per-(b, c) sums (and stored to mean_out /
// rstd_out when write_stats); otherwise read from mean_in / rstd_in.
template <int ACT>
__device__ __forceinline__ void load_chan(Chan& k, int b, int c0, int C, int L, const double* sums, float eps,
                                          float* mean_out, float* rstd_out, const float* mean_in,
                                          const float* rstd_in, const float* gb, const float* alpha,
                                          bool write_stats) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = min(c0 + j, C - 1);
        const int64_t bc = (int64_t)b * C + c;
        if (sums) {
            const double mm = sums[bc * 2] / L;
            double var = sums[bc * 2 + 1] / L - mm * mm;
            var = var > 0 ? var : 0;
            k.m[j] = (float)mm;
            k.rs[j] = (float)(1.0 / sqrt(var + (double)eps));
            if (write_stats && c0 + j < C) {
                mean_out[bc] = k.m[j];
                rstd_out[bc] = k.rs[j];
            }
        } else {
            k.m[j] = mean_in[bc];
            k.rs[j] = rstd_in[bc];
        }
        k.g1[j] = 1.f + gb[(int64_t)b * 2 * C + c];
        k.be[j] = gb[(int64_t)b * 2 * C + C + c];
        if (ACT == ACT_SNAKE) {
            k.al[j] = alpha[c];
            k.ial[j] = 1.f / k.al[j];
        }
    }
}

// Snake's sine and cosine: Cody-Waite reduction by 2*pi to [-pi, pi] (2*pi split
// as C1 + C2 with C1 = 201/32, exact in 8 bits, so k*C1 is exact for |k| < 2^16),
// then the SFU sine / cosine, whose absolute error on [-pi, pi] is about 2^-21.4.
__device__ __forceinline__ float reduce_2pi(float x) {
    const float k = rintf(x * 0.15915494309189535f);
    return fmaf(-k, 1.9353071795864769e-3f, fmaf(-k, 6.28125f, x));
}

template <int ACT>
__device__ __forceinline__ float act_f(float z, float slope, float al, float ial) {
    if (ACT == ACT_LEAKY) return z > 0.f ? z : slope * z;
    if (ACT == ACT_SNAKE) {
        const float sn = __sinf(reduce_2pi(al * z));
        return fmaf(sn * sn, ial, z);
    }
    return z;
}

// y = act((1 + gamma) * (x - mean) * rstd + beta)
template <int ACT>
__global__ void __launch_bounds__(NT) adain_fwd_kernel(Act x, int rows, const double* sums, float eps, float* mean,
                                                       float* rstd, const float* gb, float slope, const float* alpha,
                                                       Out4 o) {
    const int b = blockIdx.y;
    const int l0 = blockIdx.x * rows, l1 = min(x.L, l0 + rows);
    const int C = x.C, C4 = (C + 3) >> 2;
    for (int v = threadIdx.x; v < C4; v += blockDim.x) {
        const int c0 = 4 * v, nv = min(4, C - c0);
        Chan k;
        load_chan<ACT>(k, b, c0, C, x.L, sums, eps, mean, rstd, mean, rstd, gb, alpha,
                       blockIdx.x == 0 && threadIdx.y == 0);
        const float* base = x.p + (int64_t)b * x.bstride + c0;
        auto row = [&](const float4& a, int l) {
            float r[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float z = fmaf(k.g1[j], (get(a, j) - k.m[j]) * k.rs[j], k.be[j]);
                r[j] = act_f<ACT>(z, slope, k.al[j], k.ial[j]);
            }
            put(o, b, l, c0, make_float4(r[0], r[1], r[2], r[3]), nv);
        };
        // UNR rows per step, all loads issued before any store
        const int dl = blockDim.y;
        int l = l0 + threadIdx.y;
        for (; l + (UNR - 1) * dl < l1; l += UNR * dl) {
            float4 a[UNR];
#pragma unroll
            for (int u = 0; u < UNR; ++u) a[u] = ldg4(base + (int64_t)(l + u * dl) * x.ld);
#pragma unroll
            for (int u = 0; u < UNR; ++u) row(a[u], l + u * dl);
        }
        for (; l < l1; l += dl) row(ldg4(base + (int64_t)l * x.ld), l);
    }
}

// dz = dy * act'(z); also dy * d act / d alpha (Snake)
template <int ACT>
__device__ __forceinline__ float act_b(float z, float g, float slope, float al, float ial, float& dal) {
    if (ACT == ACT_LEAKY) return z > 0.f ? g : slope * g;
    if (ACT == ACT_SNAKE) {
        const float r = reduce_2pi(al * z);
        const float sn = __sinf(r), cs = __cosf(r);
        const float s2a = 2.f * sn * cs;   // sin(2 alpha z)
        dal = g * (z * s2a * ial - sn * sn * ial * ial);
        return fmaf(g, s2a, g);
    }
    return g;
}

// acc[(b*C + c)*3 + {0,1,2}] += sum dz, sum dz * xhat, sum dy * d act / d alpha
template <int ACT>
__global__ void __launch_bounds__(NT, 4) adain_bwd_reduce_kernel(Act x, int rows, const float* mean, const float* rstd,
                                                              const float* gb, float slope, const float* alpha, Act dy,
                                                              double* acc) {
    const int b = blockIdx.y;
    const int l0 = blockIdx.x * rows, l1 = min(x.L, l0 + rows);
    const int C = x.C, C4 = (C + 3) >> 2;
    for (int v0 = 0; v0 < C4; v0 += blockDim.x) {
        const int v = v0 + threadIdx.x;
        double s[3][4] = {};
        if (v < C4) {
            const int c0 = 4 * v;
            Chan k;
            load_chan<ACT>(k, b, c0, C, x.L, nullptr, 0.f, nullptr, nullptr, mean, rstd, gb, alpha, false);
            // a thread's rows (at most a few dozen) are summed in fp32, then combined in double
            float f[3][4] = {};
            const float* xb = x.p + (int64_t)b * x.bstride + c0;
            const float* gbp = dy.p + (int64_t)b * dy.bstride + c0;
            auto row = [&](const float4& a, const float4& g) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float xh = (get(a, j) - k.m[j]) * k.rs[j];
                    const float z = fmaf(k.g1[j], xh, k.be[j]);
                    float dal = 0.f;
                    const float dz = act_b<ACT>(z, get(g, j), slope, k.al[j], k.ial[j], dal);
                    f[0][j] += dz;
                    f[1][j] = fmaf(dz, xh, f[1][j]);
                    if (ACT == ACT_SNAKE) f[2][j] += dal;
                }
            };
            const int dl = blockDim.y;
            int l = l0 + threadIdx.y;
            for (; l + (UNR - 1) * dl < l1; l += UNR * dl) {
                float4 a[UNR], g[UNR];
#pragma unroll
                for (int u = 0; u < UNR; ++u) {
                    a[u] = ldg4(xb + (int64_t)(l + u * dl) * x.ld);
                    g[u] = ldg4(gbp + (int64_t)(l + u * dl) * dy.ld);
                }
#pragma unroll
                for (int u = 0; u < UNR; ++u) row(a[u], g[u]);
            }
            for (; l < l1; l += dl) row(ldg4(xb + (int64_t)l * x.ld), ldg4(gbp + (int64_t)l * dy.ld));
#pragma unroll
            for (int q = 0; q < 3; ++q)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[q][j] = f[q][j];
        }
        combine_rows<3>(s, v, C4, C, acc + (int64_t)b * C * 3);
    }
}

// The backward's first pass fused with the recomputation of the forward output:
// o = act(z) (the weight gradient's operand, recomputed instead of cached) and
// acc += sum dz, sum dz * xhat, sum dy * d act / d alpha, from one read of x and dy.
template <int ACT>
__global__ void __launch_bounds__(NT, 2) adain_recompute_reduce_kernel(Act x, int rows, const float* mean,
                                                                       const float* rstd, const float* gb,
                                                                       float slope, const float* alpha, Act dy,
                                                                       double* acc, Out4 o) {
    const int b = blockIdx.y;
    const int l0 = blockIdx.x * rows, l1 = min(x.L, l0 + rows);
    const int C = x.C, C4 = (C + 3) >> 2;
    for (int v0 = 0; v0 < C4; v0 += blockDim.x) {
        const int v = v0 + threadIdx.x;
        double s[3][4] = {};
        if (v < C4) {
            const int c0 = 4 * v, nv = min(4, C - c0);
            Chan k;
            load_chan<ACT>(k, b, c0, C, x.L, nullptr, 0.f, nullptr, nullptr, mean, rstd, gb, alpha, false);
            float f[3][4] = {};
            const float* xb = x.p + (int64_t)b * x.bstride + c0;
            const float* gbp = dy.p + (int64_t)b * dy.bstride + c0;
            auto row = [&](const float4& a, const float4& g, int l) {
                float r[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float xh = (get(a, j) - k.m[j]) * k.rs[j];
                    const float z = fmaf(k.g1[j], xh, k.be[j]);
                    float dal = 0.f;
                    r[j] = act_f<ACT>(z, slope, k.al[j], k.ial[j]);
                    const float dz = act_b<ACT>(z, get(g, j), slope, k.al[j], k.ial[j], dal);
                    f[0][j] += dz;
                    f[1][j] = fmaf(dz, xh, f[1][j]);
                    if (ACT == ACT_SNAKE) f[2][j] += dal;
                }
                put(o, b, l, c0, make_float4(r[0], r[1], r[2], r[3]), nv);
            };
            const int dl = blockDim.y;
            int l = l0 + threadIdx.y;
            for (; l + (RR_UNR - 1) * dl < l1; l += RR_UNR * dl) {
                float4 a[RR_UNR], g[RR_UNR];
#pragma unroll
                for (int u = 0; u < RR_UNR; ++u) {
                    a[u] = ldg4(xb + (int64_t)(l + u * dl) * x.ld);
                    g[u] = ldg4(gbp + (int64_t)(l + u * dl) * dy.ld);
                }
#pragma unroll
                for (int u = 0; u < RR_UNR; ++u) row(a[u], g[u], l + u * dl);
            }
            for (; l < l1; l += dl) row(ldg4(xb + (int64_t)l * x.ld), ldg4(gbp + (int64_t)l * dy.ld), l);
#pragma unroll
            for (int q = 0; q < 3; ++q)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[q][j] = f[q][j];
        }
        combine_rows<3>(s, v, C4, C, acc + (int64_t)b * C * 3);
    }
}

// out = rstd * g1 * (dz - mean(dz) - xhat * mean(dz * xhat)) (+ s_scale * skip)
// (+ the prior out when YACC); colsum[c] += sum out
template <int ACT, bool YACC>
__global__ void __launch_bounds__(NT, 2) adain_bwd_apply_kernel(Act x, int rows, const float* mean, const float* rstd,
                                                             const float* gb, float slope, const float* alpha, Act dy,
                                                             const double* acc, Out4 o, double* colsum) {
    const int b = blockIdx.y;
    const int l0 = blockIdx.x * rows, l1 = min(x.L, l0 + rows);
    const int C = x.C, C4 = (C + 3) >> 2;
    const double invL = 1.0 / x.L;
    for (int v0 = 0; v0 < C4; v0 += blockDim.x) {
        const int v = v0 + threadIdx.x;
        double cs[1][4] = {};
        if (v < C4) {
            const int c0 = 4 * v, nv = min(4, C - c0);
            Chan k;
            load_chan<ACT>(k, b, c0, C, x.L, nullptr, 0.f, nullptr, nullptr, mean, rstd, gb, alpha, false);
            float m0[4], m1[4], kk[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int64_t bc = (int64_t)b * C + min(c0 + j, C - 1);
                m0[j] = (float)(acc[bc * 3] * invL);
                m1[j] = (float)(acc[bc * 3 + 1] * invL);
                kk[j] = k.rs[j] * k.g1[j];
            }
            const float* xb = x.p + (int64_t)b * x.bstride + c0;
            const float* gbp = dy.p + (int64_t)b * dy.bstride + c0;
            auto row = [&](const float4& a, const float4& g, const float4& sk, int l) {
                float r[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float xh = (get(a, j) - k.m[j]) * k.rs[j];
                    const float z = fmaf(k.g1[j], xh, k.be[j]);
                    float dal = 0.f;
                    const float dz = act_b<ACT>(z, get(g, j), slope, k.al[j], k.ial[j], dal);
                    r[j] = kk[j] * (dz - m0[j] - xh * m1[j]) + get(sk, j);
                    cs[0][j] += r[j];
                }
                put(o, b, l, c0, make_float4(r[0], r[1], r[2], r[3]), nv);
            };
            // the terms added to the gradient: s_scale * skip and, accumulating, the prior output
            auto skip_at = [&](int l) {
                float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
                if (o.skip) {
                    const float4 v = ld4(o.skip + (int64_t)b * o.s_bs + (int64_t)l * o.s_ld + c0);
                    s = make_float4(o.s_scale * v.x, o.s_scale * v.y, o.s_scale * v.z, o.s_scale * v.w);
                }
                if (YACC) {
                    const float4 v = ld4(o.y + (int64_t)b * o.y_bs + (int64_t)l * o.y_ld + c0);
                    s = make_float4(s.x + v.x, s.y + v.y, s.z + v.z, s.w + v.w);
                }
                return s;
            };
            constexpr int U2 = YACC ? 3 : APPLY_ROWS;   // up to four loads per row (fewer rows in flight with four)
            const int dl = blockDim.y;
            int l = l0 + threadIdx.y;
            for (; l + (U2 - 1) * dl < l1; l += U2 * dl) {
                float4 a[U2], g[U2], sk[U2];
#pragma unroll
                for (int u = 0; u < U2; ++u) {
                    a[u] = ldg4(xb + (int64_t)(l + u * dl) * x.ld);
                    g[u] = ldg4(gbp + (int64_t)(l + u * dl) * dy.ld);
                    sk[u] = skip_at(l + u * dl);
                }
#pragma unroll
                for (int u = 0; u < U2; ++u) row(a[u], g[u], sk[u], l + u * dl);
            }
            for (; l < l1; l += dl)
                row(ldg4(xb + (int64_t)l * x.ld), ldg4(gbp + (int64_t)l * dy.ld), skip_at(l), l);
        }
        if (colsum) combine_rows<1>(cs, v, C4, C, colsum);
    }
}

__global__ void adain_bwd_final_kernel(const double* acc, int B, int C, float* dgb, float* dalpha) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    double sa = 0;
    // eight clips' sums loaded before any is used (the loop is latency-bound otherwise)
    for (int b0 = 0; b0 < B; b0 += 8) {
        double v0[8], v1[8], v2[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int64_t bc = (int64_t)min(b0 + u, B - 1) * C + c;
            v0[u] = acc[bc * 3];
            v1[u] = acc[bc * 3 + 1];
            v2[u] = acc[bc * 3 + 2];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int b = b0 + u;
            if (b >= B) break;
            if (dgb) {
                dgb[(int64_t)b * 2 * C + c] = (float)v1[u];
                dgb[(int64_t)b * 2 * C + C + c] = (float)v0[u];
            }
            sa += v2[u];
        }
    }
    if (dalpha) dalpha[c] += (float)sa;
}

// out = alpha * src; colsum[c] += sum out
__global__ void __launch_bounds__(NT) scale_out_kernel(Act s, int rows, float alpha, Out4 o, double* colsum) {
    const int b = blockIdx.y;
    const int l0 = blockIdx.x * rows, l1 = min(s.L, l0 + rows);
    const int C = s.C, C4 = (C + 3) >> 2;
    for (int v0 = 0; v0 < C4; v0 += blockDim.x) {
        const int v = v0 + threadIdx.x;
        double cs[1][4] = {};
        if (v < C4) {
            const int c0 = 4 * v, nv = min(4, C - c0);
            const float* base = s.p + (int64_t)b * s.bstride + c0;
            auto row = [&](const float4& a, int l) {
                const float4 r = make_float4(alpha * a.x, alpha * a.y, alpha * a.z, alpha * a.w);
#pragma unroll
                for (int j = 0; j < 4; ++j) cs[0][j] += get(r, j);
                put(o, b, l, c0, r, nv);
            };
            const int dl = blockDim.y;
            int l = l0 + threadIdx.y;
            for (; l + (UNR - 1) * dl < l1; l += UNR * dl) {
                float4 a[UNR];
#pragma unroll
                for (int u = 0; u < UNR; ++u) a[u] = ldg4(base + (int64_t)(l + u * dl) * s.ld);
#pragma unroll
                for (int u = 0; u < UNR; ++u) row(a[u], l + u * dl);
            }
            for (; l < l1; l += dl) row(ldg4(base + (int64_t)l * s.ld), l);
        }
        if (colsum) combine_rows<1>(cs, v, C4, C, colsum);
    }
}

__global__ void d2f_kernel(const double* src, int n, float* dst, int accum) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = (float)(accum ? dst[i] + src[i] : src[i]);
}

// ── host side
struct Geo {
    dim3 grid, block;
    int rows;
};

Geo geo(const Act& x) {
    const int C4 = (int)ceil_div(x.C, 4);
    const int bx = (int)std::min<int64_t>(round_up(C4, 32), NT);
    const int by = std::max(1, NT / bx);
    // about 6 CTAs per SM over the whole tensor, whole multiples of by rows, at least
    // 32 rows and at most 64 rows per thread (the per-thread fp32 partial sums)
    int64_t rows = ceil_div((int64_t)x.B * x.L, 148 * 6);
    rows = std::min<int64_t>(std::max<int64_t>(round_up(rows, by), 32), 64 * by);
    Geo g;
    g.rows = (int)rows;
    g.block = dim3((unsigned)bx, (unsigned)by);
    g.grid = dim3((unsigned)ceil_div(x.L, rows), (unsigned)x.B);
    return g;
}

void need_vec(const Act& a, const char* where) {
    if ((reinterpret_cast<uintptr_t>(a.p) & 15) != 0 || (a.ld & 3) != 0 || (a.bstride & 3) != 0)
        fail(where, "channels-last buffer must have 16-byte aligned rows");
}

Out4 make_out(const Act* y, const PlaneOut* pl, const Act* skip, const Act& geom, const char* where,
              const PlaneOut* pl2 = nullptr) {
    Out4 o;
    if (pl2 && pl2->hi) {
        if ((pl2->ld & 3) != 0 || (reinterpret_cast<uintptr_t>(pl2->hi) & 15) != 0)
            fail(where, "operand planes must have 16-byte aligned rows");
        o.hi2 = pl2->hi; o.lo2 = pl2->lo; o.p_ld2 = pl2->ld; o.p_bs2 = (int64_t)geom.L * pl2->ld; o.mode2 = pl2->mode;
    }
    if (y) {
        need_vec(*y, where);
        o.y = y->p; o.y_bs = y->bstride; o.y_ld = y->ld;
    }
    if (pl && pl->hi) {
        if ((pl->ld & 3) != 0 || (reinterpret_cast<uintptr_t>(pl->hi) & 15) != 0)
            fail(where, "operand planes must have 16-byte aligned rows");
        o.hi = pl->hi; o.lo = pl->lo; o.p_ld = pl->ld; o.p_bs = (int64_t)geom.L * pl->ld; o.mode = pl->mode;
    }
    if (skip) {
        need_vec(*skip, where);
        o.skip = skip->p; o.s_bs = skip->bstride; o.s_ld = skip->ld;
    }
    return o;
}

}  // namespace

void norm_sums(const Act& x, double* sums, cudaStream_t st) {
    if (x.numel() == 0) return;
    need_vec(x, "norm_sums");
    const Geo g = geo(x);
    ::bsml::count_launch();
    sums_kernel<<<g.grid, g.block, 0, st>>>(x, g.rows, sums);
    BSML_LAUNCH("norm_sums");
}

void in_stats(const Act& x, float eps, double* acc, float* mean, float* rstd, cudaStream_t st) {
    const int64_t n = (int64_t)x.B * x.C;
    BSML_CUDA(cudaMemsetAsync(acc, 0, sizeof(double) * 2 * n, st));
    norm_sums(x, acc, st);
    ::bsml::count_launch();
    stats_final_kernel<<<(unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), 4096)), 256, 0, st>>>(
        acc, n, x.L, eps, mean, rstd);
    BSML_LAUNCH("in_stats_final");
}

void adain_act_fwd_v(const Act& x, const double* sums, float eps, float* mean, float* rstd, const float* gb, int act,
                     float slope, const float* alpha, const Act* y, const PlaneOut* planes, cudaStream_t st) {
    if (x.numel() == 0) return;
    need_vec(x, "adain_act_fwd");
    const Out4 o = make_out(y, planes, nullptr, x, "adain_act_fwd");
    const Geo g = geo(x);
    ::bsml::count_launch();
    if (act == ACT_SNAKE)
        adain_fwd_kernel<ACT_SNAKE><<<g.grid, g.block, 0, st>>>(x, g.rows, sums, eps, mean, rstd, gb, slope, alpha, o);
    else if (act == ACT_LEAKY)
        adain_fwd_kernel<ACT_LEAKY><<<g.grid, g.block, 0, st>>>(x, g.rows, sums, eps, mean, rstd, gb, slope, alpha, o);
    else
        adain_fwd_kernel<ACT_NONE><<<g.grid, g.block, 0, st>>>(x, g.rows, sums, eps, mean, rstd, gb, slope, alpha, o);
    BSML_LAUNCH("adain_act_fwd");
}

void adain_act_fwd(const Act& x, const float* mean, const float* rstd, const float* gb, int act, float slope,
                   const float* alpha, const Act& y, cudaStream_t st) {
    adain_act_fwd_v(x, nullptr, 0.f, const_cast<float*>(mean), const_cast<float*>(rstd), gb, act, slope, alpha, &y,
                    nullptr, st);
}

void adain_recompute_reduce(const Act& x, const float* mean, const float* rstd, const float* gb, int act,
                            float slope, const float* alpha, const Act* y, const PlaneOut* planes, const Act& dy,
                            double* acc, cudaStream_t st) {
    BSML_CUDA(cudaMemsetAsync(acc, 0, sizeof(double) * 3 * (size_t)x.B * x.C, st));
    if (x.numel() == 0) return;
    need_vec(x, "adain_recompute_reduce");
    need_vec(dy, "adain_recompute_reduce");
    const Out4 o = make_out(y, planes, nullptr, x, "adain_recompute_reduce");
    const Geo g = geo(x);
    ::bsml::count_launch();
    if (act == ACT_SNAKE)
        adain_recompute_reduce_kernel<ACT_SNAKE><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha,
                                                                             dy, acc, o);
    else if (act == ACT_LEAKY)
        adain_recompute_reduce_kernel<ACT_LEAKY><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha,
                                                                             dy, acc, o);
    else
        adain_recompute_reduce_kernel<ACT_NONE><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha,
                                                                            dy, acc, o);
    BSML_LAUNCH("adain_recompute_reduce");
}

void adain_act_bwd_v(const Act& x, const float* mean, const float* rstd, const float* gb, int act, float slope,
                     const float* alpha, const Act& dy, const Act* dx, const Act* skip, const PlaneOut* planes,
                     double* colsum, float* dgb, float* dalpha, double* acc, cudaStream_t st, bool acc_ready,
                     float skip_scale, bool dx_accum, const PlaneOut* planes2) {
    const int64_t n = (int64_t)x.B * x.C;
    if (dx_accum && !dx) fail("adain_act_bwd", "accumulating into a missing dx");
    if (!acc_ready) BSML_CUDA(cudaMemsetAsync(acc, 0, sizeof(double) * 3 * n, st));
    if (x.numel() > 0) {
        need_vec(x, "adain_act_bwd");
        need_vec(dy, "adain_act_bwd");
        Out4 o = make_out(dx, planes, skip, x, "adain_act_bwd", planes2);
        o.s_scale = skip_scale;
        const Geo g = geo(x);
        if (!acc_ready) {
            ::bsml::count_launch();
            if (act == ACT_SNAKE)
                adain_bwd_reduce_kernel<ACT_SNAKE><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha,
                                                                               dy, acc);
            else if (act == ACT_LEAKY)
                adain_bwd_reduce_kernel<ACT_LEAKY><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha,
                                                                               dy, acc);
            else
                adain_bwd_reduce_kernel<ACT_NONE><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha,
                                                                              dy, acc);
            BSML_LAUNCH("adain_bwd_reduce");
        }
        ::bsml::count_launch();
        if (act == ACT_SNAKE && dx_accum)
            adain_bwd_apply_kernel<ACT_SNAKE, true><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha, dy, acc, o, colsum);
        else if (act == ACT_SNAKE)
            adain_bwd_apply_kernel<ACT_SNAKE, false><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha, dy, acc, o, colsum);
        else if (dx_accum)
            fail("adain_act_bwd", "accumulating output is implemented for Snake only");
        else if (act == ACT_LEAKY)
            adain_bwd_apply_kernel<ACT_LEAKY, false><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha, dy, acc, o, colsum);
        else
            adain_bwd_apply_kernel<ACT_NONE, false><<<g.grid, g.block, 0, st>>>(x, g.rows, mean, rstd, gb, slope, alpha, dy, acc, o, colsum);
        BSML_LAUNCH("adain_bwd_apply");
    }
    ::bsml::count_launch();
    adain_bwd_final_kernel<<<(unsigned)ceil_div(x.C, 128), 128, 0, st>>>(acc, x.B, x.C, dgb,
                                                                         act == ACT_SNAKE ? dalpha : nullptr);
    BSML_LAUNCH("adain_bwd_final");
}

void adain_act_bwd(const Act& x, const float* mean, const float* rstd, const float* gb, int act, float slope,
                   const float* alpha, const Act& dy, const Act& dx, const Act* skip, float* dgb, float* dalpha,
                   double* acc, cudaStream_t st) {
    adain_act_bwd_v(x, mean, rstd, gb, act, slope, alpha, dy, &dx, skip, nullptr, nullptr, dgb, dalpha, acc, st,
                    false);
}

void scale_out_v(const Act& src, float alpha, const Act* dst, const PlaneOut* planes, double* colsum,
                 cudaStream_t st, const PlaneOut* planes2) {
    if (src.numel() == 0) return;
    need_vec(src, "scale_out");
    const Out4 o = make_out(dst, planes, nullptr, src, "scale_out", planes2);
    const Geo g = geo(src);
    ::bsml::count_launch();
    scale_out_kernel<<<g.grid, g.block, 0, st>>>(src, g.rows, alpha, o, colsum);
    BSML_LAUNCH("scale_out");
}

void d2f(const double* src, int n, float* dst, bool accum, cudaStream_t st) {
    if (n <= 0) return;
    ::bsml::count_launch();
    d2f_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(src, n, dst, accum ? 1 : 0);
    BSML_LAUNCH("d2f");
}

}  // namespace bsml
