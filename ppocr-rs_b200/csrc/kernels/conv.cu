// Direct convolution (groups = 1) over a virtual concatenation of sources.
//
// Covers every dense non-pointwise conv of the PP-OCRv6 graphs: the stems
// (3x3 s2 from the NCHW image, 2x2 "same-upper" pairs, the 3x3 s2 over
// cat(maxpool(stem1), stem2b)), the medium neck's 3x3 s2 path-aggregation
// convs and fused intraclass k x k convs, and the detector head's 3x3
// conv_down over the upsample-concat of the four neck outputs
// (src/cpu/model.rs:626-693, 1022-1066, 1479-1521).
//
// One thread computes one output pixel for a tile of CO output channels
// (16 when cout >= 16, else 8), so the input window is read once per
// 16 channels; the block's weight tile [kh][kw][cin][CO] sits in shared
// memory and is read by broadcast.  Input channels are read four at a time.
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int kConvThreads = 128;

template <typename T>
__device__ __forceinline__ float4 read_source4(const ConvSource& s, int img, int iy, int ix, int hi, int wi, int c) {
    const int hs = hi / s.scale, ws = wi / s.scale;
    const T* base = static_cast<const T*>(s.ptr);
    if (s.mode == SRC_NHWC_MAXPOOL) {
        // 2x2 window anchored at (iy, ix); positions past the bottom/right edge
        // are padding and never win (pads [0, 0, 1, 1]).
        float4 m = load4(base + ((size_t)(img * hs + iy) * ws + ix) * s.cstride + s.coff + c);
        if (ix + 1 < ws) {
            float4 v = load4(base + ((size_t)(img * hs + iy) * ws + ix + 1) * s.cstride + s.coff + c);
            m = make_float4(fmaxf(m.x, v.x), fmaxf(m.y, v.y), fmaxf(m.z, v.z), fmaxf(m.w, v.w));
        }
        if (iy + 1 < hs) {
            float4 v = load4(base + ((size_t)(img * hs + iy + 1) * ws + ix) * s.cstride + s.coff + c);
            m = make_float4(fmaxf(m.x, v.x), fmaxf(m.y, v.y), fmaxf(m.z, v.z), fmaxf(m.w, v.w));
            if (ix + 1 < ws) {
                v = load4(base + ((size_t)(img * hs + iy + 1) * ws + ix + 1) * s.cstride + s.coff + c);
                m = make_float4(fmaxf(m.x, v.x), fmaxf(m.y, v.y), fmaxf(m.z, v.z), fmaxf(m.w, v.w));
            }
        }
        return m;
    }
    const int sy = iy / s.scale, sx = ix / s.scale;
    return load4(base + ((size_t)(img * hs + sy) * ws + sx) * s.cstride + s.coff + c);
}

template <typename T, int CO>
__global__ void __launch_bounds__(kConvThreads) conv_kernel(ConvParams p) {
    extern __shared__ float wsm[];
    const int tile = blockIdx.y;
    const int taps = p.kh * p.kw;
    const int wcount = taps * p.cin * CO;
    const float* wsrc = p.weight + (size_t)tile * wcount;
    for (int i = threadIdx.x * 4; i < wcount; i += kConvThreads * 4) {
        *reinterpret_cast<float4*>(wsm + i) = *reinterpret_cast<const float4*>(wsrc + i);
    }
    __syncthreads();

    const long long total = (long long)p.n * p.ho * p.wo;
    const long long pix = (long long)blockIdx.x * kConvThreads + threadIdx.x;
    if (pix >= total) return;
    const int ox = (int)(pix % p.wo);
    const int oy = (int)((pix / p.wo) % p.ho);
    const int img = (int)(pix / ((long long)p.wo * p.ho));

    float acc[CO];
#pragma unroll
    for (int o = 0; o < CO; ++o) acc[o] = 0.f;

    for (int ky = 0; ky < p.kh; ++ky) {
        const int iy = oy * p.sh - p.pt + ky;
        if (iy < 0 || iy >= p.hi) continue;
        for (int kx = 0; kx < p.kw; ++kx) {
            const int ix = ox * p.sw - p.pl + kx;
            if (ix < 0 || ix >= p.wi) continue;
            const float* wt = wsm + (size_t)(ky * p.kw + kx) * p.cin * CO;
            int cbase = 0;
            for (int s = 0; s < p.nsrc; ++s) {
                const ConvSource& src = p.src[s];
                if (src.mode == SRC_NCHW_F32) {
                    const float* base = static_cast<const float*>(src.ptr);
                    for (int c = 0; c < src.channels; ++c) {
                        const float v = base[((size_t)(img * src.channels + c) * p.hi + iy) * p.wi + ix];
                        const float* wr = wt + (cbase + c) * CO;
#pragma unroll
                        for (int o = 0; o < CO; ++o) acc[o] = fmaf(v, wr[o], acc[o]);
                    }
                } else {
                    for (int c = 0; c < src.channels; c += 4) {
                        const float4 v = read_source4<T>(src, img, iy, ix, p.hi, p.wi, c);
                        const float* wr = wt + (cbase + c) * CO;
#pragma unroll
                        for (int o = 0; o < CO; o += 4) {
                            const float4 w0 = *reinterpret_cast<const float4*>(wr + o);
                            const float4 w1 = *reinterpret_cast<const float4*>(wr + CO + o);
                            const float4 w2 = *reinterpret_cast<const float4*>(wr + 2 * CO + o);
                            const float4 w3 = *reinterpret_cast<const float4*>(wr + 3 * CO + o);
                            acc[o] = fmaf(v.x, w0.x, acc[o]);
                            acc[o + 1] = fmaf(v.x, w0.y, acc[o + 1]);
                            acc[o + 2] = fmaf(v.x, w0.z, acc[o + 2]);
                            acc[o + 3] = fmaf(v.x, w0.w, acc[o + 3]);
                            acc[o] = fmaf(v.y, w1.x, acc[o]);
                            acc[o + 1] = fmaf(v.y, w1.y, acc[o + 1]);
                            acc[o + 2] = fmaf(v.y, w1.z, acc[o + 2]);
                            acc[o + 3] = fmaf(v.y, w1.w, acc[o + 3]);
                            acc[o] = fmaf(v.z, w2.x, acc[o]);
                            acc[o + 1] = fmaf(v.z, w2.y, acc[o + 1]);
                            acc[o + 2] = fmaf(v.z, w2.z, acc[o + 2]);
                            acc[o + 3] = fmaf(v.z, w2.w, acc[o + 3]);
                            acc[o] = fmaf(v.w, w3.x, acc[o]);
                            acc[o + 1] = fmaf(v.w, w3.y, acc[o + 1]);
                            acc[o + 2] = fmaf(v.w, w3.z, acc[o + 2]);
                            acc[o + 3] = fmaf(v.w, w3.w, acc[o + 3]);
                        }
                    }
                }
                cbase += src.channels;
            }
        }
    }

    const int co0 = tile * CO;
    T* out = static_cast<T*>(p.out) + (size_t)pix * p.out_cstride + p.out_coff + co0;
    const T* res = nullptr;
    if (p.residual) {
        const int rh = p.ho / p.res_scale, rw = p.wo / p.res_scale;
        res = static_cast<const T*>(p.residual) +
              ((size_t)(img * rh + oy / p.res_scale) * rw + ox / p.res_scale) * p.cout + co0;
    }
#pragma unroll
    for (int g = 0; g < CO; g += 4) {
        if (co0 + g >= p.cout) break;
        float4 v = make_float4(acc[g], acc[g + 1], acc[g + 2], acc[g + 3]);
        if (p.bias) v = f4_add(v, *reinterpret_cast<const float4*>(p.bias + co0 + g));
        v = f4_act(v, p.act);
        if (res) v = f4_add(v, load4(res + g));
        store4(out + g, v);
    }
}

template <typename T, int CO>
cudaError_t launch_conv_t(const ConvParams& p, cudaStream_t stream) {
    const int tiles = (p.cout + CO - 1) / CO;
    const size_t smem = (size_t)p.kh * p.kw * p.cin * CO * sizeof(float);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(conv_kernel<T, CO>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    if (smem > 200 * 1024) return cudaErrorInvalidConfiguration;
    const long long total = (long long)p.n * p.ho * p.wo;
    dim3 grid((unsigned)((total + kConvThreads - 1) / kConvThreads), (unsigned)tiles);
    conv_kernel<T, CO><<<grid, kConvThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_conv(const ConvParams& p, cudaStream_t stream) {
    if (p.co_tile == 16)
        return p.dtype == DT_F32 ? launch_conv_t<float, 16>(p, stream) : launch_conv_t<__nv_bfloat16, 16>(p, stream);
    if (p.co_tile != 8) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_conv_t<float, 8>(p, stream) : launch_conv_t<__nv_bfloat16, 8>(p, stream);
}

}  // namespace ppocr
