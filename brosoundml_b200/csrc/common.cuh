// Shared helpers for the sm_100a kernels and the host engine.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace bsml {

// Errors cross the C ABI as a status code plus a thread-local message in the
// reference's format: "brosoundml: <where>: <reason>".
struct Error : std::runtime_error {
    explicit Error(const std::string& m) : std::runtime_error(m) {}
};

[[noreturn]] inline void fail(const char* where, const std::string& why) {
    throw Error(std::string("brosoundml: ") + where + ": " + why);
}

inline void check_cuda(cudaError_t e, const char* where) {
    if (e != cudaSuccess) fail(where, cudaGetErrorString(e));
}

#define BSML_CUDA(call) ::bsml::check_cuda((call), #call)
#define BSML_LAUNCH(where) ::bsml::check_cuda(cudaGetLastError(), where)

// Message returned by bsml_last_error() on this thread.
void set_last_error(const std::string& msg);

// Kernel launches issued by this library (every launch site counts itself).
void count_launch();
int64_t launch_count();

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline int64_t round_up(int64_t a, int64_t b) { return ceil_div(a, b) * b; }

#if defined(BSML_DEBUG_BOUNDS) && defined(__CUDACC__)
// Debug builds (make DEBUG=1: relocatable device code, one copy of this word for
// the whole library): the first out-of-range row access of any kernel is recorded
// here as (1, b, l, B, L) and the access is clamped into range, so the kernel
// finishes and the host reads the record (bsml_debug_bounds).
extern __device__ int g_dbg_bounds[5];
#endif

// Channels-last activation view: element (b, l, c) at p[b*bstride + l*ld + c].
struct Act {
    float* p = nullptr;
    int B = 0, L = 0, C = 0, ld = 0;
    int64_t bstride = 0;
#if defined(BSML_DEBUG_BOUNDS) && defined(__CUDA_ARCH__)
    __device__ float* row(int b, int l) const {
        if (b < 0 || b >= B || l < 0 || l >= L) {
            if (atomicCAS(&g_dbg_bounds[0], 0, 1) == 0) {
                g_dbg_bounds[1] = b; g_dbg_bounds[2] = l; g_dbg_bounds[3] = B; g_dbg_bounds[4] = L;
            }
            b = b < 0 ? 0 : (b >= B ? B - 1 : b);
            l = l < 0 ? 0 : (l >= L ? L - 1 : l);
        }
        return p + (int64_t)b * bstride + (int64_t)l * ld;
    }
#else
    __host__ __device__ float* row(int b, int l) const { return p + (int64_t)b * bstride + (int64_t)l * ld; }
#endif
    Act slice_c(int c0, int nc) const {
        Act a = *this;
        a.p = p + c0;
        a.C = nc;
        return a;
    }
    __host__ __device__ int64_t numel() const { return (int64_t)B * L * C; }
};

// Padded row pitch used for every channels-last buffer: 16-byte aligned rows
// (a TMA requirement for the tensor-core path).
inline int pitch(int C) { return (int)round_up(C, 4); }

#ifdef __CUDACC__
// sum_{q < n} p[q * stride] in double, in order q = 0, 1, ..., with eight loads in
// flight per thread (split-K partials are latency-bound when read one by one)
__device__ __forceinline__ double sum_strided(const float* p, int64_t stride, int n) {
    double s = 0.0;
    int q = 0;
    for (; q + 8 <= n; q += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldg(p + (int64_t)(q + u) * stride);
#pragma unroll
        for (int u = 0; u < 8; ++u) s += v[u];
    }
    for (; q < n; ++q) s += __ldg(p + (int64_t)q * stride);
    return s;
}
#endif

}  // namespace bsml
