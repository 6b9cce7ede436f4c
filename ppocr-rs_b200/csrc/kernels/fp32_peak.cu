// FP32 CUDA-core throughput probe: the denominator of the roofline for the
// FP32 mode's SIMT kernels (measured on the running GPU, since no driver
// figure covers the CUDA cores).  Each thread runs 16 independent FMA chains
// with no memory traffic; `packed` issues them as two-lane f32x2 FMAs.
#include "kernels.h"

namespace ppocr {
namespace {

template <bool PACKED>
__global__ void __launch_bounds__(512) fp32_peak_kernel(float* sink, int iters, float s) {
    float a[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = threadIdx.x * 1e-7f + (float)i;
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
            if (PACKED) {
                const float2 r = __ffma2_rn(make_float2(a[i], a[i + 1]), make_float2(s, s), make_float2(1e-7f, 2e-7f));
                a[i] = r.x;
                a[i + 1] = r.y;
            } else {
                a[i] = fmaf(a[i], s, 1e-7f);
                a[i + 1] = fmaf(a[i + 1], s, 2e-7f);
            }
        }
    }
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) t += a[i];
    if (t == 1234.5f) sink[0] = t;   // keeps the chains live; never true for these inputs
}

}  // namespace

cudaError_t launch_fp32_peak(float* sink, int blocks, int iters, bool packed, cudaStream_t stream) {
    if (blocks <= 0 || iters <= 0) return cudaErrorInvalidValue;
    if (packed) fp32_peak_kernel<true><<<blocks, 512, 0, stream>>>(sink, iters, 0.999999f);
    else fp32_peak_kernel<false><<<blocks, 512, 0, stream>>>(sink, iters, 0.999999f);
    return cudaGetLastError();
}

}  // namespace ppocr
