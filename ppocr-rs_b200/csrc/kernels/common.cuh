// Shared device helpers for the PP-OCRv6 sm_100a kernels.
//
// Activations are NHWC with the channel axis contiguous.  Storage type T is
// float (FP32 mode) or __nv_bfloat16 (BF16 mode); all arithmetic is FP32 in
// registers.  Activation formulas follow ppocr-rs src/cpu/kernels/mod.rs:2365-2403.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"

namespace ppocr {

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Abramowitz-Stegun 7.1.26 erf with the reference's coefficients
// (src/cpu/kernels/mod.rs:2393-2403).
__device__ __forceinline__ float erf_as(float x) {
    float s = x < 0.f ? -1.f : 1.f;
    float a = fabsf(x);
    float t = 1.f / fmaf(a, 0.3275911f, 1.f);
    float p = t * (0.2548296f + t * (-0.28449672f + t * (1.4214138f + t * (-1.4531521f + t * 1.0614054f))));
    return s * (1.f - p * expf(-a * a));
}

// Same formulas with hardware-approximate exp (ex2-based, ~2 ulp) and
// approximate reciprocal / division: for epilogues whose results are rounded
// to BF16 (8-bit mantissa), where the difference to apply_act is far below
// one BF16 ulp.
template <int ACT>
__device__ __forceinline__ float apply_act_fast(float v) {
    if (ACT == ACT_RELU) return fmaxf(v, 0.f);
    if (ACT == ACT_SILU) return __fdividef(v, 1.f + __expf(-v));
    if (ACT == ACT_GELU) {
        const float x = v * 0.70710678118654752f;
        const float a = fabsf(x);
        const float t = __fdividef(1.f, fmaf(a, 0.3275911f, 1.f));
        const float p = t * (0.2548296f + t * (-0.28449672f + t * (1.4214138f + t * (-1.4531521f + t * 1.0614054f))));
        const float e = 1.f - p * __expf(-a * a);
        return 0.5f * v * (1.f + copysignf(e, x));
    }
    if (ACT == ACT_HSWISH) return v * fminf(fmaxf(v * (1.f / 6.f) + 0.5f, 0.f), 1.f);
    if (ACT == ACT_SIGMOID) return __fdividef(1.f, 1.f + __expf(-v));
    return v;
}

__device__ __forceinline__ float apply_act(float v, int act) {
    switch (act) {
        case ACT_RELU: return fmaxf(v, 0.f);
        case ACT_SILU: return v / (1.f + expf(-v));
        case ACT_GELU: return 0.5f * v * (1.f + erf_as(v * 0.70710678118654752f));
        case ACT_HSWISH: return v * fminf(fmaxf(v / 6.f + 0.5f, 0.f), 1.f);
        case ACT_SIGMOID: return 1.f / (1.f + expf(-v));
        default: return v;
    }
}

// Four consecutive channels, loaded/stored as one 16-byte (float) or 8-byte
// (bf16) access.  Callers guarantee 4-element alignment.
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
    uint2 u = *reinterpret_cast<const uint2*>(p);
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&u.x);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&u.y);
    float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
}
__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(__nv_bfloat16* p, float4 v) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
}

__device__ __forceinline__ float4 f4_fma(float a, float4 b, float4 c) {
    return make_float4(fmaf(a, b.x, c.x), fmaf(a, b.y, c.y), fmaf(a, b.z, c.z), fmaf(a, b.w, c.w));
}
__device__ __forceinline__ float4 f4_mul(float4 a, float4 b) { return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
__device__ __forceinline__ float4 f4_add(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float4 f4_max(float4 a, float4 b) {
    return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
}
// Two FP32 FMAs in one packed sm_100 instruction: (c0, c1) += (a0, a1) * (b0, b1),
// each lane rounded once, exactly as fmaf.  Halves the issue slots FP32 FMA
// loops spend on arithmetic.
__device__ __forceinline__ void fma2(float& c0, float& c1, float a0, float a1, float b0, float b1) {
    const float2 r = __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), make_float2(c0, c1));
    c0 = r.x;
    c1 = r.y;
}
__device__ __forceinline__ float4 f4_vfma(float4 a, float4 b, float4 c) {
    fma2(c.x, c.y, a.x, a.y, b.x, b.y);
    fma2(c.z, c.w, a.z, a.w, b.z, b.w);
    return c;
}
__device__ __forceinline__ float4 f4_act(float4 v, int act) {
    return make_float4(apply_act(v.x, act), apply_act(v.y, act), apply_act(v.z, act), apply_act(v.w, act));
}

}  // namespace ppocr
