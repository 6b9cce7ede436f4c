// Direct convolution (groups = 1) over a virtual concatenation of sources.
//
// Covers every dense non-pointwise conv of the PP-OCRv6 graphs: the stems
// (3x3 s2 from the NCHW image, 2x2 "same-upper" pairs, the 3x3 s2 over
// cat(maxpool(stem1), stem2b)), the medium neck's 3x3 s2 path-aggregation
// convs and fused intraclass k x k convs, and the detector head's 3x3
// conv_down over the upsample-concat of the four neck outputs
// (src/cpu/model.rs:626-693, 1022-1066, 1479-1521).
//
// One thread computes PIX output pixels (one in the launched configuration)
// for a tile of CO output channels (16 when cout >= 16, else 8; 32 or 64 for
// the 3-channel image input, whose few inputs per pixel would otherwise be
// re-read once per 16 output channels), so the input window is read once per
// CO channels; the block's weight tile
// [kh][kw][cin][CO] sits in shared memory and is read by broadcast.
// Input channels are read four at a time; source addresses are computed
// once per (tap, source).
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int kConvThreads = 128;

// Address of one NHWC source pixel for the logical (upsampled) position
// (iy, ix); `shift` = log2 of the source's upsampling factor (a power of two,
// checked on the host).  For max-pool sources the window's right / bottom
// neighbours are flagged when they exist.
struct SrcPix {
    int off;        // element offset of the pixel's channel 0 of the view
    bool right, down;
};

__device__ __forceinline__ SrcPix source_pixel(const ConvSource& s, int shift, int img, int iy, int ix, int hi, int wi) {
    const int hs = hi >> shift, ws = wi >> shift;
    const int sy = iy >> shift, sx = ix >> shift;
    SrcPix r;
    r.off = ((img * hs + sy) * ws + sx) * s.cstride + s.coff;
    r.right = sx + 1 < ws;
    r.down = sy + 1 < hs;
    return r;
}

template <typename T>
__device__ __forceinline__ float4 read_pixel4(const ConvSource& s, const T* base, const SrcPix& px, int ws, int c) {
    float4 m = load4(base + px.off + c);
    if (s.mode == SRC_NHWC_MAXPOOL) {
        // 2x2 window anchored at the pixel; positions past the bottom/right
        // edge are padding and never win (pads [0, 0, 1, 1]).
        if (px.right) m = f4_max(m, load4(base + px.off + s.cstride + c));
        if (px.down) {
            m = f4_max(m, load4(base + px.off + ws * s.cstride + c));
            if (px.right) m = f4_max(m, load4(base + px.off + (ws + 1) * s.cstride + c));
        }
    }
    return m;
}

template <int CO>
__device__ __forceinline__ void fma_quad(float (&acc)[CO], const float4 v, const float* wr) {
#pragma unroll
    for (int o = 0; o < CO; o += 4) {
        const float4 w0 = *reinterpret_cast<const float4*>(wr + o);
        const float4 w1 = *reinterpret_cast<const float4*>(wr + CO + o);
        const float4 w2 = *reinterpret_cast<const float4*>(wr + 2 * CO + o);
        const float4 w3 = *reinterpret_cast<const float4*>(wr + 3 * CO + o);
        fma2(acc[o], acc[o + 1], v.x, v.x, w0.x, w0.y);
        fma2(acc[o + 2], acc[o + 3], v.x, v.x, w0.z, w0.w);
        fma2(acc[o], acc[o + 1], v.y, v.y, w1.x, w1.y);
        fma2(acc[o + 2], acc[o + 3], v.y, v.y, w1.z, w1.w);
        fma2(acc[o], acc[o + 1], v.z, v.z, w2.x, w2.y);
        fma2(acc[o + 2], acc[o + 3], v.z, v.z, w2.z, w2.w);
        fma2(acc[o], acc[o + 1], v.w, v.w, w3.x, w3.y);
        fma2(acc[o + 2], acc[o + 3], v.w, v.w, w3.z, w3.w);
    }
}

// One thread computes PIX horizontally adjacent output pixels (of the
// flattened pixel index) for CO output channels; the weight reads from
// shared memory are shared by the PIX pixels.  Per output, the FMAs run in
// the order (ky, kx, source, channel), the same for every PIX.
template <typename T, int CO, int PIX>
__global__ void __launch_bounds__(kConvThreads) conv_kernel(ConvParams p, int4 shifts) {
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
    const long long pix0 = ((long long)blockIdx.x * kConvThreads + threadIdx.x) * PIX;
    if (pix0 >= total) return;
    int ox[PIX], oy[PIX], img[PIX];
    bool live[PIX];
#pragma unroll
    for (int q = 0; q < PIX; ++q) {
        const long long pix = pix0 + q;
        live[q] = pix < total;
        const long long pc = live[q] ? pix : pix0;
        ox[q] = (int)(pc % p.wo);
        oy[q] = (int)((pc / p.wo) % p.ho);
        img[q] = (int)(pc / ((long long)p.wo * p.ho));
    }
    const int shift[4] = {shifts.x, shifts.y, shifts.z, shifts.w};

    float acc[PIX][CO];
#pragma unroll
    for (int q = 0; q < PIX; ++q)
#pragma unroll
        for (int o = 0; o < CO; ++o) acc[q][o] = 0.f;

    for (int ky = 0; ky < p.kh; ++ky) {
        for (int kx = 0; kx < p.kw; ++kx) {
            bool in[PIX];
            int iy[PIX], ix[PIX];
            bool any = false;
#pragma unroll
            for (int q = 0; q < PIX; ++q) {
                iy[q] = oy[q] * p.sh - p.pt + ky;
                ix[q] = ox[q] * p.sw - p.pl + kx;
                in[q] = live[q] && iy[q] >= 0 && iy[q] < p.hi && ix[q] >= 0 && ix[q] < p.wi;
                any |= in[q];
            }
            if (!any) continue;
            const float* wt = wsm + (size_t)(ky * p.kw + kx) * p.cin * CO;
            int cbase = 0;
            for (int s = 0; s < p.nsrc; ++s) {
                const ConvSource& src = p.src[s];
                if (src.mode == SRC_NCHW_F32) {
                    const float* base = static_cast<const float*>(src.ptr);
                    const size_t plane = (size_t)p.hi * p.wi;
                    size_t off[PIX];
#pragma unroll
                    for (int q = 0; q < PIX; ++q)
                        off[q] = in[q] ? ((size_t)img[q] * src.channels * p.hi + iy[q]) * p.wi + ix[q] : 0;
                    for (int c = 0; c < src.channels; ++c) {
                        const float* wr = wt + (cbase + c) * CO;
#pragma unroll
                        for (int q = 0; q < PIX; ++q) {
                            if (!in[q]) continue;
                            const float v = base[off[q] + (size_t)c * plane];
#pragma unroll
                            for (int o = 0; o < CO; o += 2) fma2(acc[q][o], acc[q][o + 1], v, v, wr[o], wr[o + 1]);
                        }
                    }
                } else {
                    const T* base = static_cast<const T*>(src.ptr);
                    const int sh = shift[s];
                    const int ws = p.wi >> sh;
                    SrcPix px[PIX];
#pragma unroll
                    for (int q = 0; q < PIX; ++q)
                        px[q] = in[q] ? source_pixel(src, sh, img[q], iy[q], ix[q], p.hi, p.wi) : SrcPix{0, false, false};
                    for (int c = 0; c < src.channels; c += 4) {
                        const float* wr = wt + (cbase + c) * CO;
#pragma unroll
                        for (int q = 0; q < PIX; ++q) {
                            if (!in[q]) continue;
                            fma_quad<CO>(acc[q], read_pixel4<T>(src, base, px[q], ws, c), wr);
                        }
                    }
                }
                cbase += src.channels;
            }
        }
    }

    const int co0 = tile * CO;
#pragma unroll
    for (int q = 0; q < PIX; ++q) {
        if (!live[q]) break;
        T* out = static_cast<T*>(p.out) + (size_t)(pix0 + q) * p.out_cstride + p.out_coff + co0;
        const T* res = nullptr;
        if (p.residual) {
            const int rh = p.ho / p.res_scale, rw = p.wo / p.res_scale;
            res = static_cast<const T*>(p.residual) +
                  ((size_t)(img[q] * rh + oy[q] / p.res_scale) * rw + ox[q] / p.res_scale) * p.cout + co0;
        }
#pragma unroll
        for (int g = 0; g < CO; g += 4) {
            if (co0 + g >= p.cout) break;
            float4 v = make_float4(acc[q][g], acc[q][g + 1], acc[q][g + 2], acc[q][g + 3]);
            if (p.bias) v = f4_add(v, *reinterpret_cast<const float4*>(p.bias + co0 + g));
            v = f4_act(v, p.act);
            if (res) v = f4_add(v, load4(res + g));
            store4(out + g, v);
        }
    }
}

template <typename T, int CO>
cudaError_t launch_conv_t(const ConvParams& p, cudaStream_t stream) {
    constexpr int PIX = 1;
    const int tiles = (p.cout + CO - 1) / CO;
    const size_t smem = (size_t)p.kh * p.kw * p.cin * CO * sizeof(float);
    {
        cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(conv_kernel<T, CO, PIX>), 200 * 1024);
        if (e != cudaSuccess) return e;
    }
    if (smem > 200 * 1024 || p.nsrc < 1 || p.nsrc > 4) return cudaErrorInvalidConfiguration;
    // Upsampling factors are powers of two (nearest x2/x4/x8 in the necks);
    // the kernel divides by shifting.
    int sh[4] = {0, 0, 0, 0};
    for (int s = 0; s < p.nsrc; ++s) {
        const int sc = p.src[s].scale;
        if (sc < 1 || (sc & (sc - 1)) || p.hi % sc || p.wi % sc) return cudaErrorInvalidValue;
        while ((1 << sh[s]) < sc) ++sh[s];
    }
    const long long total = (long long)p.n * p.ho * p.wo;
    const long long threads = (total + PIX - 1) / PIX;
    dim3 grid((unsigned)((threads + kConvThreads - 1) / kConvThreads), (unsigned)tiles);
    conv_kernel<T, CO, PIX><<<grid, kConvThreads, smem, stream>>>(p, make_int4(sh[0], sh[1], sh[2], sh[3]));
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_conv(const ConvParams& p, cudaStream_t stream) {
    if (p.w_tc) return launch_conv_tc(p, stream);
    if (p.halo) return launch_conv_halo(p, stream);
    if (p.weight_kn) return launch_conv_gemm(p, stream);
    if (p.co_tile == 64)
        return p.dtype == DT_F32 ? launch_conv_t<float, 64>(p, stream) : launch_conv_t<__nv_bfloat16, 64>(p, stream);
    if (p.co_tile == 32)
        return p.dtype == DT_F32 ? launch_conv_t<float, 32>(p, stream) : launch_conv_t<__nv_bfloat16, 32>(p, stream);
    if (p.co_tile == 16)
        return p.dtype == DT_F32 ? launch_conv_t<float, 16>(p, stream) : launch_conv_t<__nv_bfloat16, 16>(p, stream);
    if (p.co_tile != 8) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_conv_t<float, 8>(p, stream) : launch_conv_t<__nv_bfloat16, 8>(p, stream);
}

}  // namespace ppocr
