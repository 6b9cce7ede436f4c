// Depthwise convolution with fused bias, activation and residual.
//
// Covers the LCNet token convs (3x3, stride 1 / (2,2) / (2,1), folded BN or
// bias, src/cpu/model.rs:526-587), the RepLkFpn depthwise 5x5 / 7x7
// (src/cpu/model.rs:1145-1195), the medium neck's rank-one 9x9 depthwise
// halves (src/cpu/model.rs:165-219), the SVTR local 1x7 conv + SiLU + residual
// (src/cpu/model.rs:1825-1830) and the tiny recognizer's 1x5 head conv.
//
// Bandwidth-bound (algorithmic bytes = input + output (+ residual) +
// weights).  A block owns a TH x TW output tile of CG channel quads: it
// stages the input tile plus halo in shared memory once (coalesced 16-byte
// loads, CG quads of a pixel contiguous), so every input element is read from
// HBM about once instead of k^2 times.  Each thread then computes RUN = 4
// horizontally adjacent outputs of one channel quad: per kernel row it loads
// the (RUN - 1) * SW + KW window pixels once into registers and each weight
// once for all RUN outputs.  Kernel size, strides and so the tile extents
// are template parameters: the window stays in registers and the tile index
// arithmetic has no runtime division.
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int kThreads = 256;
constexpr int kRun = 4;

// Output tile TH x TW: 8 x 32 at stride 1, halved along a strided axis.  The
// input tile covers every window the tile's outputs read.
template <int KH, int KW, int SH, int SW>
struct DwTile {
    static constexpr int TH = SH == 1 ? 8 : 4;
    static constexpr int TW = SW == 1 ? 32 : 16;
    static constexpr int IH = (TH - 1) * SH + KH;
    static constexpr int IW = (TW - 1) * SW + KW;
};

template <typename T, int CG, int KH, int KW, int SH, int SW>
__global__ void __launch_bounds__(kThreads) dwconv_tiled_kernel(DwParams p) {
    using G = DwTile<KH, KW, SH, SW>;
    constexpr int TH = G::TH, TW = G::TW, IH = G::IH, IW = G::IW;
    extern __shared__ float4 sm4[];
    float4* tile = sm4;                        // [IH][IW][CG]
    float4* wts = sm4 + IH * IW * CG;          // [taps][CG]
    constexpr int taps = KH * KW;
    const int groups = p.c / (4 * CG);
    const int img = blockIdx.z / groups, grp = blockIdx.z % groups;
    const int c0 = grp * CG * 4;
    const int oy0 = blockIdx.y * TH, ox0 = blockIdx.x * TW;
    const int iy0 = oy0 * SH - p.pt, ix0 = ox0 * SW - p.pl;
    const T* in = static_cast<const T*>(p.in) + (size_t)img * p.hi * p.wi * p.in_cstride + p.in_coff + c0;

    for (int i = threadIdx.x; i < taps * CG; i += kThreads) {
        const int t = i / CG, q = i % CG;
        wts[i] = *reinterpret_cast<const float4*>(p.weight + (size_t)t * p.c + c0 + q * 4);
    }
    // Tile rows, pixels and channel quads are compile-time extents, so the
    // index split below is multiplies and shifts.
    for (int i = threadIdx.x; i < IH * IW * CG; i += kThreads) {
        const int q = i % CG, pix = i / CG;
        const int ty = pix / IW, tx = pix - ty * IW;
        const int y = iy0 + ty, x = ix0 + tx;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (y >= 0 && y < p.hi && x >= 0 && x < p.wi) v = load4(in + ((size_t)y * p.wi + x) * p.in_cstride + q * 4);
        tile[i] = v;
    }
    __syncthreads();

    const int q = threadIdx.x % CG;
    const int c = c0 + q * 4;
    const float4 bias = p.bias ? *reinterpret_cast<const float4*>(p.bias + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int PX = kThreads / CG;
    constexpr int SPAN = (kRun - 1) * SW + KW;
    constexpr int runs = TW / kRun;
    for (int pp = threadIdx.x / CG; pp < TH * runs; pp += PX) {
        const int ty = pp / runs, tx0 = (pp % runs) * kRun;
        const int oy = oy0 + ty;
        if (oy >= p.ho || ox0 + tx0 >= p.wo) continue;
        float4 acc[kRun];
#pragma unroll
        for (int r = 0; r < kRun; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int ky = 0; ky < KH; ++ky) {
            const float4* row = tile + ((ty * SH + ky) * IW + tx0 * SW) * CG + q;
            const float4* wr = wts + ky * KW * CG + q;
            float4 win[SPAN];
#pragma unroll
            for (int i = 0; i < SPAN; ++i) win[i] = row[i * CG];
#pragma unroll
            for (int kx = 0; kx < KW; ++kx) {
                const float4 w = wr[kx * CG];
#pragma unroll
                for (int r = 0; r < kRun; ++r) acc[r] = f4_vfma(win[r * SW + kx], w, acc[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < kRun; ++r) {
            const int ox = ox0 + tx0 + r;
            if (ox >= p.wo) break;
            float4 v = f4_act(f4_add(acc[r], bias), p.act);
            const size_t o = ((size_t)(img * p.ho + oy) * p.wo + ox) * p.c + c;
            if (p.residual) v = f4_add(v, load4(static_cast<const T*>(p.residual) + o));
            store4(static_cast<T*>(p.out) + o, v);
        }
    }
}

template <typename T, int CG, int KH, int KW, int SH, int SW>
cudaError_t launch_tiled(const DwParams& p, cudaStream_t stream) {
    using G = DwTile<KH, KW, SH, SW>;
    const size_t smem = ((size_t)G::IH * G::IW * CG + (size_t)KH * KW * CG) * sizeof(float4);
    if (smem > 200 * 1024) return cudaErrorInvalidConfiguration;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(dwconv_tiled_kernel<T, CG, KH, KW, SH, SW>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const long long z = (long long)p.n * (p.c / (4 * CG));
    if (z > 65535 || (p.ho + G::TH - 1) / G::TH > 65535) return cudaErrorInvalidConfiguration;
    dim3 grid((p.wo + G::TW - 1) / G::TW, (p.ho + G::TH - 1) / G::TH, (unsigned)z);
    dwconv_tiled_kernel<T, CG, KH, KW, SH, SW><<<grid, kThreads, smem, stream>>>(p);
    return cudaGetLastError();
}

template <typename T, int KH, int KW, int SH, int SW>
cudaError_t launch_cg(const DwParams& p, cudaStream_t stream) {
    const int quads = p.c / 4;
    if (quads % 8 == 0) return launch_tiled<T, 8, KH, KW, SH, SW>(p, stream);
    if (quads % 4 == 0) return launch_tiled<T, 4, KH, KW, SH, SW>(p, stream);
    if (quads % 2 == 0) return launch_tiled<T, 2, KH, KW, SH, SW>(p, stream);
    return launch_tiled<T, 1, KH, KW, SH, SW>(p, stream);
}

// The geometries of the PP-OCRv6 graphs: 3x3 at strides (1,1), (2,2), (2,1);
// square 5x5 / 7x7 / 9x9 at stride 1; 1x5 / 1x7 (recognizer heads).
template <typename T>
cudaError_t launch_dw_t(const DwParams& p, cudaStream_t stream) {
    if (p.kh == 3 && p.kw == 3) {
        if (p.sh == 1 && p.sw == 1) return launch_cg<T, 3, 3, 1, 1>(p, stream);
        if (p.sh == 2 && p.sw == 2) return launch_cg<T, 3, 3, 2, 2>(p, stream);
        if (p.sh == 2 && p.sw == 1) return launch_cg<T, 3, 3, 2, 1>(p, stream);
        return cudaErrorInvalidValue;
    }
    if (p.sh != 1 || p.sw != 1) return cudaErrorInvalidValue;
    if (p.kh == p.kw) {
        switch (p.kh) {
            case 5: return launch_cg<T, 5, 5, 1, 1>(p, stream);
            case 7: return launch_cg<T, 7, 7, 1, 1>(p, stream);
            case 9: return launch_cg<T, 9, 9, 1, 1>(p, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    if (p.kh == 1 && p.kw == 5) return launch_cg<T, 1, 5, 1, 1>(p, stream);
    if (p.kh == 1 && p.kw == 7) return launch_cg<T, 1, 7, 1, 1>(p, stream);
    return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_dwconv(const DwParams& p, cudaStream_t stream) {
    if (p.c % 4 || p.in_coff % 4 || p.in_cstride % 4) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_dw_t<float>(p, stream) : launch_dw_t<__nv_bfloat16>(p, stream);
}

}  // namespace ppocr
