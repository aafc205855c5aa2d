// Device helpers shared by the kernels that produce tensor-core operands:
// 128-bit channels-last loads/stores and the split of an fp32 value into the
// operand planes the tcgen05 convolutions read (tf32 hi + fp32 remainder, or bf16).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace bsml {

// TcMode values (conv_tc.h): 0 = bf16 plane, 1 = tf32 hi + fp32 lo planes,
// 2 = bf16 hi + bf16 lo planes.
constexpr int PLANES_BF16 = 0;
constexpr int PLANES_TF32X3 = 1;
constexpr int PLANES_BF16X3 = 2;

__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

__device__ __forceinline__ float4 ldg4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }
__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__device__ __forceinline__ float get(const float4& v, int j) { return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w; }

// Store the first nv (1..4) lanes of v at p (p 16-byte aligned when nv == 4).
__device__ __forceinline__ void st4(float* p, const float4& v, int nv) {
    if (nv == 4) {
        *reinterpret_cast<float4*>(p) = v;
    } else {
        p[0] = v.x;
        if (nv > 1) p[1] = v.y;
        if (nv > 2) p[2] = v.z;
    }
}

// Operand planes at element offset `off`: tf32 (hi, lo = v - hi, both fp32
// containers) or bf16 (hi only). Only the first nv lanes are written.
__device__ __forceinline__ void st_planes4(void* hi, void* lo, int mode, int64_t off, const float4& v, int nv) {
    if (mode == PLANES_TF32X3) {
        const float4 h = make_float4(tf32_rna(v.x), tf32_rna(v.y), tf32_rna(v.z), tf32_rna(v.w));
        const float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
        st4(static_cast<float*>(hi) + off, h, nv);
        st4(static_cast<float*>(lo) + off, l, nv);
    } else if (mode == PLANES_BF16X3) {
        __nv_bfloat16* ph = static_cast<__nv_bfloat16*>(hi) + off;
        __nv_bfloat16* pl = static_cast<__nv_bfloat16*>(lo) + off;
        const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        const float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
        const __nv_bfloat162 c = __floats2bfloat162_rn(v.x - fa.x, v.y - fa.y);
        const __nv_bfloat162 d = __floats2bfloat162_rn(v.z - fb.x, v.w - fb.y);
        if (nv == 4) {
            uint2 u, w;
            u.x = *reinterpret_cast<const uint32_t*>(&a);
            u.y = *reinterpret_cast<const uint32_t*>(&b);
            w.x = *reinterpret_cast<const uint32_t*>(&c);
            w.y = *reinterpret_cast<const uint32_t*>(&d);
            *reinterpret_cast<uint2*>(ph) = u;
            *reinterpret_cast<uint2*>(pl) = w;
        } else {
            const __nv_bfloat16 hs[4] = {a.x, a.y, b.x, b.y}, ls[4] = {c.x, c.y, d.x, d.y};
            for (int j = 0; j < nv; ++j) {
                ph[j] = hs[j];
                pl[j] = ls[j];
            }
        }
    } else {
        __nv_bfloat16* p = static_cast<__nv_bfloat16*>(hi) + off;
        if (nv == 4) {
            const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
            uint2 u;
            u.x = *reinterpret_cast<const uint32_t*>(&a);
            u.y = *reinterpret_cast<const uint32_t*>(&b);
            *reinterpret_cast<uint2*>(p) = u;
        } else {
            for (int j = 0; j < nv; ++j) p[j] = __float2bfloat16_rn(get(v, j));
        }
    }
}

}  // namespace bsml
