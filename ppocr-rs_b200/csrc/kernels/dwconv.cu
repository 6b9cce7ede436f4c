// Depthwise convolution with fused bias, activation and residual.
//
// Covers the LCNet token convs (3x3, stride 1 / (2,2) / (2,1), folded BN or
// bias, src/cpu/model.rs:526-587), the RepLkFpn depthwise 5x5 / 7x7
// (src/cpu/model.rs:1145-1195), the medium neck's rank-one 9x9 depthwise
// halves (src/cpu/model.rs:165-219), the SVTR local 1x7 conv + SiLU + residual
// (src/cpu/model.rs:1825-1830) and the tiny recognizer's 1x5 head conv.
//
// Bandwidth-bound (algorithmic bytes = input + output (+ residual) +
// weights).  A block owns a th x tw output tile of CG channel quads at a
// time: the input tile plus halo arrives in shared memory through 16-byte
// cp.async copies (CG quads of a pixel contiguous, out-of-image halo
// zero-filled), so every input element is read from HBM about once instead
// of k^2 times.  Blocks are persistent and double-buffer the input tile: the
// copies of the next tile are in flight while the current one is computed.
// Each thread computes RUN = 4 horizontally adjacent outputs of one channel
// quad: per kernel row it loads the (RUN - 1) * SW + KW window pixels once
// into registers and each weight once for all RUN outputs.  Kernel size and
// strides are template parameters, so the window stays in registers; the
// tile shape is chosen per launch to divide the output evenly.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int kThreads = 256;
constexpr int kRun = 4;

// Tile geometry, chosen per launch from the output extent: about TH0 x TW0
// outputs (8 x 32 at stride 1, halved along a strided axis) reshaped so the
// tiles divide the output evenly (a 3-row recognizer map gets 3-row tiles
// twice as wide instead of 8-row tiles that are mostly empty).  The input tile
// (ih x iw) covers every window the tile's outputs read.
struct DwGeom {
    int th, tw, ih, iw, runs;          // output tile, input tile, kRun-wide runs per tile row
    int tiles_x, tiles_y, groups, total;
    float inv_runs, inv_iw;            // reciprocals for exact small-integer division
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    // Out-of-image parts of the halo: source size 0 zero-fills the 16 bytes.
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float4 to4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 to4(const __nv_bfloat16* p) { return load4(p); }

// Persistent blocks walk the output tiles; the raw input tile (plus halo) of
// the next tile is copied into the other of two shared buffers with cp.async
// while the current one is computed, so loads and arithmetic overlap.
// Small-integer division q = floor(i / d) through a float reciprocal: for
// i < 2^14 and d < 2^10 the product (i + 0.5) * (1/d) lies at least 0.5/d
// from an integer, far outside its rounding error, so the floor is exact.
__device__ __forceinline__ int div_small(int i, float inv_d) { return (int)(((float)i + 0.5f) * inv_d); }

template <typename T, int CG, int KH, int KW, int SH, int SW>
__global__ void __launch_bounds__(kThreads) dwconv_tiled_kernel(DwParams p, DwGeom g) {
    constexpr int QPC = 16 / (4 * sizeof(T));          // channel quads per 16-byte copy
    constexpr int CPP = CG / QPC;                      // 16-byte copies per pixel
    const int copies = g.ih * g.iw * CPP;              // 16-byte copies per tile
    const int TILE_ELEMS = g.ih * g.iw * CG * 4;
    extern __shared__ float4 sm4[];
    T* const buf = reinterpret_cast<T*>(sm4);                                              // [2][TILE_ELEMS]
    float4* wts = reinterpret_cast<float4*>(reinterpret_cast<T*>(sm4) + 2 * TILE_ELEMS);   // [taps][CG]
    constexpr int taps = KH * KW;

    const int per_z = g.tiles_x * g.tiles_y;
    auto issue = [&](int tile, T* dst) {
        const int z = tile / per_z, rem = tile - z * per_z;
        const int img = z / g.groups, grp = z - img * g.groups;
        const int tyi = rem / g.tiles_x, txi = rem - tyi * g.tiles_x;
        const int iy0 = tyi * g.th * SH - p.pt, ix0 = txi * g.tw * SW - p.pl;
        const T* in = static_cast<const T*>(p.in) + (size_t)img * p.hi * p.wi * p.in_cstride + p.in_coff + grp * CG * 4;
        for (int i = threadIdx.x; i < copies; i += kThreads) {
            const int qq = (i % CPP) * QPC, pix = i / CPP;
            const int ty = div_small(pix, g.inv_iw), tx = pix - ty * g.iw;
            const int y = iy0 + ty, x = ix0 + tx;
            const bool ok = y >= 0 && y < p.hi && x >= 0 && x < p.wi;
            const T* src = ok ? in + ((size_t)y * p.wi + x) * p.in_cstride + qq * 4 : in;
            cp_async16(dst + (size_t)(pix * CG + qq) * 4, src, ok);
        }
        cp_async_commit();
    };

    int tile = blockIdx.x;
    if (tile >= g.total) return;
    issue(tile, buf);
    int parity = 0, wgrp = -1;
    for (; tile < g.total; tile += gridDim.x, parity ^= 1) {
        const int next = tile + gridDim.x;
        if (next < g.total) issue(next, buf + (parity ^ 1) * TILE_ELEMS);
        else cp_async_commit();   // keep one group per iteration
        const int z = tile / per_z, rem = tile - z * per_z;
        const int img = z / g.groups, grp = z - img * g.groups;
        const int c0 = grp * CG * 4;
        if (grp != wgrp) {
            __syncthreads();   // every thread is done with the previous weights
            for (int i = threadIdx.x; i < taps * CG; i += kThreads) {
                const int t = i / CG, q = i % CG;
                wts[i] = *reinterpret_cast<const float4*>(p.weight + (size_t)t * p.c + c0 + q * 4);
            }
            wgrp = grp;
        }
        cp_async_wait<1>();    // this tile's copies have landed (the next tile's may be in flight)
        __syncthreads();
        const T* tileb = buf + parity * TILE_ELEMS;
        const int tyi = rem / g.tiles_x;
        const int oy0 = tyi * g.th, ox0 = (rem - tyi * g.tiles_x) * g.tw;
        const int q = threadIdx.x % CG;
        const int c = c0 + q * 4;
        const float4 bias = p.bias ? *reinterpret_cast<const float4*>(p.bias + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        constexpr int PX = kThreads / CG;
        constexpr int SPAN = (kRun - 1) * SW + KW;
        const int items = g.th * g.runs;
        for (int pp = threadIdx.x / CG; pp < items; pp += PX) {
            const int ty = div_small(pp, g.inv_runs), tx0 = (pp - ty * g.runs) * kRun;
            const int oy = oy0 + ty;
            if (oy >= p.ho || ox0 + tx0 >= p.wo) continue;
            float4 acc[kRun];
#pragma unroll
            for (int r = 0; r < kRun; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int ky = 0; ky < KH; ++ky) {
                const T* row = tileb + ((size_t)((ty * SH + ky) * g.iw + tx0 * SW) * CG + q) * 4;
                const float4* wr = wts + ky * KW * CG + q;
                float4 win[SPAN];
#pragma unroll
                for (int i = 0; i < SPAN; ++i) win[i] = to4(row + (size_t)i * CG * 4);
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
        __syncthreads();       // the buffer is free for the copies two tiles ahead
    }
    cp_async_wait<0>();
}

constexpr size_t kSmemLimit = 200 * 1024;

// Splits the output into tiles of about th0 x tw0 outputs that divide it
// evenly, then fits the double-buffered input tile into shared memory.
inline DwGeom dw_geometry(const DwParams& p, int th0, int tw0, int groups, size_t pix_bytes, size_t wbytes) {
    DwGeom g{};
    g.tiles_y = (p.ho + th0 - 1) / th0;
    g.th = (p.ho + g.tiles_y - 1) / g.tiles_y;
    int tw_max = (th0 * tw0 / g.th) / kRun * kRun;
    if (tw_max < kRun) tw_max = kRun;
    for (;;) {
        g.tiles_x = (p.wo + tw_max - 1) / tw_max;
        const int tw = (p.wo + g.tiles_x - 1) / g.tiles_x;
        g.tw = (tw + kRun - 1) / kRun * kRun;
        g.ih = (g.th - 1) * p.sh + p.kh;
        g.iw = (g.tw - 1) * p.sw + p.kw;
        if (2 * (size_t)g.ih * g.iw * pix_bytes + wbytes <= kSmemLimit || tw_max == kRun) break;
        tw_max -= kRun;
    }
    g.runs = g.tw / kRun;
    g.groups = groups;
    const long long total = (long long)p.n * groups * g.tiles_x * g.tiles_y;
    g.total = total > 0x7fffffffLL ? -1 : (int)total;
    g.inv_runs = 1.0f / (float)g.runs;
    g.inv_iw = 1.0f / (float)g.iw;
    return g;
}

template <typename T, int CG, int KH, int KW, int SH, int SW>
cudaError_t launch_tiled(const DwParams& p, cudaStream_t stream) {
    const size_t pix_bytes = (size_t)CG * 4 * sizeof(T), wbytes = (size_t)KH * KW * CG * sizeof(float4);
    const DwGeom g = dw_geometry(p, SH == 1 ? 8 : 4, SW == 1 ? 32 : 16, p.c / (4 * CG), pix_bytes, wbytes);
    const size_t smem = 2 * (size_t)g.ih * g.iw * pix_bytes + wbytes;
    // div_small is exact for tile indices below 2^14 and divisors below 2^10.
    if (g.total < 0 || smem > kSmemLimit || g.ih * g.iw >= (1 << 14) || g.iw >= (1 << 10) || g.runs >= (1 << 10))
        return cudaErrorInvalidConfiguration;
    if (g.total == 0) return cudaSuccess;
    auto kernel = dwconv_tiled_kernel<T, CG, KH, KW, SH, SW>;
    // Resident blocks per SM, from the kernel's registers (queried once) and
    // this launch's shared memory: the occupancy API is far too slow to call
    // for every tile shape the recognizer's varying widths produce.
    static std::atomic<int> regs{0};
    int nregs = regs.load(std::memory_order_acquire);
    if (!nregs) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemLimit);
        if (e != cudaSuccess) return e;
        cudaFuncAttributes fa{};
        e = cudaFuncGetAttributes(&fa, kernel);
        if (e != cudaSuccess) return e;
        nregs = fa.numRegs > 0 ? fa.numRegs : 1;
        regs.store(nregs, std::memory_order_release);
    }
    int dev = 0, sms = 148, smem_sm = 0, reserved = 0, regs_sm = 65536, threads_sm = 2048;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    const int warp_regs = (nregs + 7) / 8 * 8 * 32;   // registers are allocated per warp in 256-register units
    int blocks_per_sm = threads_sm / kThreads;
    blocks_per_sm = std::min(blocks_per_sm, regs_sm / (warp_regs * (kThreads / 32)));
    blocks_per_sm = std::min(blocks_per_sm, (int)(smem_sm / (smem + (size_t)reserved)));
    if (blocks_per_sm < 1) blocks_per_sm = 1;
    const long long cap = (long long)sms * blocks_per_sm;
    const int grid = (int)(g.total < cap ? g.total : cap);
    kernel<<<grid, kThreads, smem, stream>>>(p, g);
    return cudaGetLastError();
}

template <typename T, int KH, int KW, int SH, int SW>
cudaError_t launch_cg(const DwParams& p, cudaStream_t stream) {
    // 16-byte copies hold one FP32 or two BF16 channel quads.
    const int quads = p.c / 4;
    if (quads % 8 == 0) return launch_tiled<T, 8, KH, KW, SH, SW>(p, stream);
    if (quads % 4 == 0) return launch_tiled<T, 4, KH, KW, SH, SW>(p, stream);
    if (quads % 2 == 0) return launch_tiled<T, 2, KH, KW, SH, SW>(p, stream);
    if constexpr (sizeof(T) == 4) return launch_tiled<T, 1, KH, KW, SH, SW>(p, stream);
    return cudaErrorInvalidValue;
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
    // 16-byte copies: BF16 views need 8-channel alignment.
    if (p.dtype == DT_BF16 && (p.c % 8 || p.in_coff % 8 || p.in_cstride % 8)) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_dw_t<float>(p, stream) : launch_dw_t<__nv_bfloat16>(p, stream);
}

}  // namespace ppocr
