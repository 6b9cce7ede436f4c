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

// GELU of two values for the tensor-core epilogues (BF16 results), with the
// arithmetic in packed f32x2 FMAs and one hardware exp per value: the A&S
// 7.1.26 erf of apply_act_fast, its reciprocal 1 / (1 + 0.3275911 a) from an
// integer-subtraction estimate (within 5 %) refined by two Newton-Raphson
// steps (relative error below 1e-5, under 1/400 of a BF16 ulp), so a GELU
// costs one MUFU operation instead of two.
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ void gelu_fast2(float& v0, float& v1) {
    const float2 v = make_float2(v0, v1);
    const float2 x = __fmul2_rn(v, make_float2(0.70710678118654752f, 0.70710678118654752f));
    const float2 a = make_float2(fabsf(x.x), fabsf(x.y));
    const float2 d = __ffma2_rn(a, make_float2(0.3275911f, 0.3275911f), make_float2(1.f, 1.f));
    float2 t = make_float2(__int_as_float(0x7EF311C3 - __float_as_int(d.x)), __int_as_float(0x7EF311C3 - __float_as_int(d.y)));
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const float2 e = __ffma2_rn(make_float2(-d.x, -d.y), t, make_float2(1.f, 1.f));
        t = __ffma2_rn(t, e, t);
    }
    float2 q = __ffma2_rn(t, make_float2(1.0614054f, 1.0614054f), make_float2(-1.4531521f, -1.4531521f));
    q = __ffma2_rn(t, q, make_float2(1.4214138f, 1.4214138f));
    q = __ffma2_rn(t, q, make_float2(-0.28449672f, -0.28449672f));
    q = __ffma2_rn(t, q, make_float2(0.2548296f, 0.2548296f));
    q = __fmul2_rn(t, q);
    // exp(-a^2) = 2^(-a^2 log2 e)
    const float2 m = __fmul2_rn(a, make_float2(-1.4426950408889634f, -1.4426950408889634f));
    const float2 y = __fmul2_rn(m, a);
    const float2 ex = make_float2(ex2_approx(y.x), ex2_approx(y.y));
    const float2 e = __ffma2_rn(make_float2(-q.x, -q.y), ex, make_float2(1.f, 1.f));
    const float2 h = __fmul2_rn(v, make_float2(0.5f, 0.5f));
    const float2 r = __ffma2_rn(h, make_float2(copysignf(e.x, x.x), copysignf(e.y, x.y)), h);
    v0 = r.x;
    v1 = r.y;
}

// apply_act_fast over an array, GELU two values at a time.
template <int ACT, int N>
__device__ __forceinline__ void apply_act_fast_array(float (&o)[N]) {
    if constexpr (ACT == ACT_GELU && N % 2 == 0) {
#pragma unroll
        for (int j = 0; j < N; j += 2) gelu_fast2(o[j], o[j + 1]);
    } else {
#pragma unroll
        for (int j = 0; j < N; ++j) o[j] = apply_act_fast<ACT>(o[j]);
    }
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
    // A BF16 value is the upper half of the FP32 with the same value: widening
    // is a shift (even channel, low half) or a mask (odd channel, high half).
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
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
