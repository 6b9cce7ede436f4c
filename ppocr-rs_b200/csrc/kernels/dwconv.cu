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
// once for all RUN outputs.  KW and SW are template parameters so the window
// stays in registers; KH is a runtime loop.
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int kThreads = 256;
constexpr int kRun = 4;

template <typename T, int CG, int KW, int SW>
__global__ void __launch_bounds__(kThreads) dwconv_tiled_kernel(DwParams p, int th, int tw, int ih, int iw) {
    extern __shared__ float4 sm4[];
    float4* tile = sm4;                        // [ih][iw][CG]
    float4* wts = sm4 + (size_t)ih * iw * CG;  // [taps][CG]
    const int taps = p.kh * KW;
    const int groups = p.c / (4 * CG);
    const int img = blockIdx.z / groups, grp = blockIdx.z % groups;
    const int c0 = grp * CG * 4;
    const int oy0 = blockIdx.y * th, ox0 = blockIdx.x * tw;
    const int iy0 = oy0 * p.sh - p.pt, ix0 = ox0 * SW - p.pl;
    const T* in = static_cast<const T*>(p.in);

    for (int i = threadIdx.x; i < taps * CG; i += kThreads) {
        const int t = i / CG, q = i % CG;
        wts[i] = *reinterpret_cast<const float4*>(p.weight + (size_t)t * p.c + c0 + q * 4);
    }
    const int n_in = ih * iw * CG;
    for (int i = threadIdx.x; i < n_in; i += kThreads) {
        const int q = i % CG, pix = i / CG;
        const int y = iy0 + pix / iw, x = ix0 + pix % iw;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (y >= 0 && y < p.hi && x >= 0 && x < p.wi)
            v = load4(in + ((size_t)(img * p.hi + y) * p.wi + x) * p.in_cstride + p.in_coff + c0 + q * 4);
        tile[i] = v;
    }
    __syncthreads();

    const int q = threadIdx.x % CG;
    const int c = c0 + q * 4;
    const float4 bias = p.bias ? *reinterpret_cast<const float4*>(p.bias + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int PX = kThreads / CG;
    constexpr int SPAN = (kRun - 1) * SW + KW;
    const int runs = tw / kRun;
    for (int pp = threadIdx.x / CG; pp < th * runs; pp += PX) {
        const int ty = pp / runs, tx0 = (pp % runs) * kRun;
        const int oy = oy0 + ty;
        if (oy >= p.ho || ox0 + tx0 >= p.wo) continue;
        float4 acc[kRun];
#pragma unroll
        for (int r = 0; r < kRun; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int ky = 0; ky < p.kh; ++ky) {
            const float4* row = tile + ((size_t)(ty * p.sh + ky) * iw + tx0 * SW) * CG + q;
            const float4* wr = wts + (size_t)ky * KW * CG + q;
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

template <typename T, int CG, int KW, int SW>
cudaError_t launch_tiled(const DwParams& p, cudaStream_t stream) {
    // Output tile: 8 rows x 32 columns at stride 1; halve along a strided axis.
    // The input tile covers every window the tile's outputs read: SPAN of the
    // last run ends at ((tw - 1) * SW + KW) - 1.
    const int th = p.sh == 1 ? 8 : 4;
    const int tw = SW == 1 ? 32 : 16;
    const int ih = (th - 1) * p.sh + p.kh, iw = (tw - 1) * SW + KW;
    const size_t smem = ((size_t)ih * iw * CG + (size_t)p.kh * KW * CG) * sizeof(float4);
    if (smem > 200 * 1024) return cudaErrorInvalidConfiguration;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(dwconv_tiled_kernel<T, CG, KW, SW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             200 * 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const long long z = (long long)p.n * (p.c / (4 * CG));
    if (z > 65535 || (p.ho + th - 1) / th > 65535) return cudaErrorInvalidConfiguration;
    dim3 grid((p.wo + tw - 1) / tw, (p.ho + th - 1) / th, (unsigned)z);
    dwconv_tiled_kernel<T, CG, KW, SW><<<grid, kThreads, smem, stream>>>(p, th, tw, ih, iw);
    return cudaGetLastError();
}

template <typename T, int KW, int SW>
cudaError_t launch_cg(const DwParams& p, cudaStream_t stream) {
    const int quads = p.c / 4;
    if (quads % 8 == 0) return launch_tiled<T, 8, KW, SW>(p, stream);
    if (quads % 4 == 0) return launch_tiled<T, 4, KW, SW>(p, stream);
    if (quads % 2 == 0) return launch_tiled<T, 2, KW, SW>(p, stream);
    return launch_tiled<T, 1, KW, SW>(p, stream);
}

template <typename T>
cudaError_t launch_dw_t(const DwParams& p, cudaStream_t stream) {
    if (p.sw == 1) {
        switch (p.kw) {
            case 3: return launch_cg<T, 3, 1>(p, stream);
            case 5: return launch_cg<T, 5, 1>(p, stream);
            case 7: return launch_cg<T, 7, 1>(p, stream);
            case 9: return launch_cg<T, 9, 1>(p, stream);
            default: return cudaErrorInvalidValue;
        }
    }
    if (p.sw == 2 && p.kw == 3) return launch_cg<T, 3, 2>(p, stream);
    return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_dwconv(const DwParams& p, cudaStream_t stream) {
    if (p.c % 4 || p.in_coff % 4 || p.in_cstride % 4) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_dw_t<float>(p, stream) : launch_dw_t<__nv_bfloat16>(p, stream);
}

}  // namespace ppocr
