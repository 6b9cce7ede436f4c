// Depthwise convolution with fused bias, activation and residual.
//
// Covers the LCNet token convs (3x3, stride 1 / (2,2) / (2,1), folded BN or
// bias, src/cpu/model.rs:526-587), the RepLkFpn depthwise 5x5 / 7x7
// (src/cpu/model.rs:1145-1195), the medium neck's rank-one 9x9 depthwise
// halves (src/cpu/model.rs:165-219), the SVTR local 1x7 conv + SiLU + residual
// (src/cpu/model.rs:1825-1830) and the tiny recognizer's 1x5 head conv.
//
// NHWC: a thread owns 4 consecutive channels of one output pixel, so a warp
// reads contiguous channel runs of neighbouring pixels (coalesced 16- or
// 8-byte accesses); the k x k window re-reads hit L1/L2.  Bandwidth-bound:
// algorithmic bytes = input + output (+ residual) + weights.
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) dwconv_kernel(DwParams p) {
    const int cg = p.c >> 2;
    const long long total = (long long)p.n * p.ho * p.wo * cg;
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(idx % cg) * 4;
        const long long pix = idx / cg;
        const int ox = (int)(pix % p.wo);
        const int oy = (int)((pix / p.wo) % p.ho);
        const int img = (int)(pix / ((long long)p.wo * p.ho));
        const T* in = static_cast<const T*>(p.in) + p.in_coff + c;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int ky = 0; ky < p.kh; ++ky) {
            const int iy = oy * p.sh - p.pt + ky;
            if (iy < 0 || iy >= p.hi) continue;
            const T* row = in + (size_t)(img * p.hi + iy) * p.wi * p.in_cstride;
            const float* wrow = p.weight + (size_t)ky * p.kw * p.c + c;
            for (int kx = 0; kx < p.kw; ++kx) {
                const int ix = ox * p.sw - p.pl + kx;
                if (ix < 0 || ix >= p.wi) continue;
                const float4 v = load4(row + (size_t)ix * p.in_cstride);
                const float4 w = *reinterpret_cast<const float4*>(wrow + (size_t)kx * p.c);
                acc = f4_vfma(v, w, acc);
            }
        }
        if (p.bias) acc = f4_add(acc, *reinterpret_cast<const float4*>(p.bias + c));
        acc = f4_act(acc, p.act);
        const size_t o = (size_t)pix * p.c + c;
        if (p.residual) acc = f4_add(acc, load4(static_cast<const T*>(p.residual) + o));
        store4(static_cast<T*>(p.out) + o, acc);
    }
}

template <typename T>
cudaError_t launch_dw_t(const DwParams& p, cudaStream_t stream) {
    const long long total = (long long)p.n * p.ho * p.wo * (p.c / 4);
    long long blocks = (total + 255) / 256;
    const long long cap = 148LL * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    dwconv_kernel<T><<<(unsigned)blocks, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_dwconv(const DwParams& p, cudaStream_t stream) {
    if (p.c % 4) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_dw_t<float>(p, stream) : launch_dw_t<__nv_bfloat16>(p, stream);
}

}  // namespace ppocr
