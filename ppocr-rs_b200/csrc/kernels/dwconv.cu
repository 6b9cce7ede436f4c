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
// Each thread computes RUN horizontally adjacent outputs of one channel
// quad (tiled_run: 8 for square kernels of 5x5 and up, else 4): per kernel
// row it loads the (RUN - 1) * SW + KW window pixels once into registers and
// each weight once for all RUN outputs.  Kernel size and
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

// Outputs per thread along a tile row in the tiled kernel: 8 for the square
// 5x5 and larger kernels, whose wide windows are mostly shared between
// neighbouring outputs (a 9x9 run of 8 loads 16 window pixels per row for 72
// multiply-adds), 4 for the rest.
__host__ __device__ constexpr int tiled_run(int kh, int kw) { return kh == kw && kh >= 5 ? 8 : kRun; }

// Tile geometry, chosen per launch from the output extent: about TH0 x TW0
// outputs (8 x 32 at stride 1, halved along a strided axis) reshaped so the
// tiles divide the output evenly (a 3-row recognizer map gets 3-row tiles
// twice as wide instead of 8-row tiles that are mostly empty).  The input tile
// (ih x iw) covers every window the tile's outputs read.
struct DwGeom {
    int th, tw, ih, iw, runs;          // output tile, input tile, tiled_run-wide runs per tile row
    int tiles_x, tiles_y, groups, total;
    float inv_runs, inv_iw;            // reciprocals for exact small-integer division
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    // Out-of-image parts of the halo: source size 0 zero-fills the 16 bytes.
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async16_u32(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
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

// PLAIN: no activation and no residual, so the epilogue is the bias add and
// the store (the per-element activation switch is a large share of the
// instructions of a depthwise conv).
template <typename T, int CG, int KH, int KW, int SH, int SW, bool PLAIN>
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
        constexpr int RUN = tiled_run(KH, KW);
        constexpr int SPAN = (RUN - 1) * SW + KW;
        const int items = g.th * g.runs;
        for (int pp = threadIdx.x / CG; pp < items; pp += PX) {
            const int ty = div_small(pp, g.inv_runs), tx0 = (pp - ty * g.runs) * RUN;
            const int oy = oy0 + ty;
            if (oy >= p.ho || ox0 + tx0 >= p.wo) continue;
            float4 acc[RUN];
#pragma unroll
            for (int r = 0; r < RUN; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
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
                    for (int r = 0; r < RUN; ++r) acc[r] = f4_vfma(win[r * SW + kx], w, acc[r]);
                }
            }
#pragma unroll
            for (int r = 0; r < RUN; ++r) {
                const int ox = ox0 + tx0 + r;
                if (ox >= p.wo) break;
                float4 v = f4_add(acc[r], bias);
                const size_t o = ((size_t)(img * p.ho + oy) * p.wo + ox) * p.c + c;
                if constexpr (!PLAIN) {
                    v = f4_act(v, p.act);
                    if (p.residual) v = f4_add(v, load4(static_cast<const T*>(p.residual) + o));
                }
                store4(static_cast<T*>(p.out) + o, v);
            }
        }
        __syncthreads();       // the buffer is free for the copies two tiles ahead
    }
    cp_async_wait<0>();
}

constexpr size_t kSmemLimit = 200 * 1024;

// Resident blocks per SM from a kernel's registers (queried once per kernel)
// and a launch's threads and shared memory: the occupancy API is far too slow
// to call for every tile shape the recognizer's varying widths produce.
inline int resident_blocks(int nregs, int threads, size_t smem) {
    int dev = 0, smem_sm = 0, reserved = 0, regs_sm = 65536, threads_sm = 2048;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    const int warps = (threads + 31) / 32;
    const int warp_regs = (nregs + 7) / 8 * 8 * 32;   // registers are allocated per warp in 256-register units
    int blocks = threads_sm / (warps * 32);
    blocks = std::min(blocks, regs_sm / (warp_regs * warps));
    blocks = std::min(blocks, (int)(smem_sm / (smem + (size_t)reserved)));
    return blocks < 1 ? 1 : blocks;
}

// Splits the output into tiles of about th0 x tw0 outputs that divide it
// evenly, then fits the double-buffered input tile into shared memory.
inline DwGeom dw_geometry(const DwParams& p, int th0, int tw0, int groups, size_t pix_bytes, size_t wbytes) {
    DwGeom g{};
    const int run = tiled_run(p.kh, p.kw);
    g.tiles_y = (p.ho + th0 - 1) / th0;
    g.th = (p.ho + g.tiles_y - 1) / g.tiles_y;
    int tw_max = (th0 * tw0 / g.th) / run * run;
    if (tw_max < run) tw_max = run;
    for (;;) {
        g.tiles_x = (p.wo + tw_max - 1) / tw_max;
        const int tw = (p.wo + g.tiles_x - 1) / g.tiles_x;
        g.tw = (tw + run - 1) / run * run;
        g.ih = (g.th - 1) * p.sh + p.kh;
        g.iw = (g.tw - 1) * p.sw + p.kw;
        if (2 * (size_t)g.ih * g.iw * pix_bytes + wbytes <= kSmemLimit || tw_max == run) break;
        tw_max -= run;
    }
    g.runs = g.tw / run;
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
    const bool plain = p.act == ACT_NONE && !p.residual;
    auto kernel = plain ? dwconv_tiled_kernel<T, CG, KH, KW, SH, SW, true> : dwconv_tiled_kernel<T, CG, KH, KW, SH, SW, false>;
    static std::atomic<int> regs_by_plain[2] = {0, 0};   // each kernel's registers, queried once
    std::atomic<int>& regs = regs_by_plain[plain ? 1 : 0];
    // The shared-memory limit is a per-device attribute: set on every device
    // the kernel runs on (the register count below is the same on all).
    {
        const cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), (int)kSmemLimit);
        if (e != cudaSuccess) return e;
    }
    int nregs = regs.load(std::memory_order_acquire);
    if (!nregs) {
        cudaFuncAttributes fa{};
        cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
        if (e != cudaSuccess) return e;
        nregs = fa.numRegs > 0 ? fa.numRegs : 1;
        regs.store(nregs, std::memory_order_release);
    }
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long cap = (long long)sms * resident_blocks(nregs, kThreads, smem);
    const int grid = (int)(g.total < cap ? g.total : cap);
    kernel<<<grid, kThreads, smem, stream>>>(p, g);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// 3x3 depthwise conv over rolling rows.
//
// A unit is one image x one segment of bh output rows x one band of bw output
// columns x one channel group of CG quads (units numbered with the group
// fastest, so blocks running side by side read all channels of the same
// pixels).  Each thread owns one channel quad and RUN adjacent output columns
// of the band and walks down the segment's input rows: each input row is read
// from shared memory once and feeds every output row it belongs to (three at
// stride 1, up to two at stride 2), whose partial sums stay in registers until
// their last tap.  The taps of each output are still summed in (ky, kx) order,
// so the results are bit-identical to the tiled kernel's.  Input rows arrive
// through an NR-slot cp.async ring, NR - 1 rows ahead and continuous across a
// persistent block's units; a unit's weights and bias ride with its first row
// (the weights are read from shared memory by broadcast, which leaves the
// registers to the three rows of partial sums).
// ---------------------------------------------------------------------------
struct DwBand {
    int bw, bh, sx, iw;          // outputs per band row, output rows per segment, runs per band, input columns per row
    int bands, segs, groups;     // units: ((img * segs + seg) * bands + bx) * groups + grp
    int ni, total;               // input rows per segment, units
};

// Outputs per thread along a row: 4 for 3x3; 2 for 5x5, whose five rows of
// partial sums in flight would otherwise not fit the registers (the models
// run their 5x5 convs on the tiled kernel, which is faster there).
__host__ __device__ constexpr int band_run(int k) { return k == 3 ? 4 : 2; }

__device__ __forceinline__ void band_decode(const DwBand& g, int u, int& img, int& seg, int& bx, int& grp) {
    grp = u % g.groups;
    int r = u / g.groups;
    bx = r % g.bands;
    r /= g.bands;
    seg = r % g.segs;
    img = r / g.segs;
}

// Positive remainder and floor division for the static set bookkeeping.
__host__ __device__ constexpr int pmod(int a, int m) { return ((a % m) + m) % m; }
__host__ __device__ constexpr int fdiv(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }

// PLAIN: no activation and no residual (the token convs), so the epilogue is
// the bias add and the store.
template <typename T, int CG, int K, int SH, int SW, int NR, bool PLAIN>
__global__ void __launch_bounds__(256, 2) dwconv_band_kernel(DwParams p, DwBand g) {
    constexpr int RUN = band_run(K);
    constexpr int D = NR - 1;                  // rows in flight ahead of the one being computed
    constexpr int QPC = 16 / (4 * sizeof(T));  // channel quads per 16-byte copy
    constexpr int CPP = CG / QPC;              // 16-byte copies per pixel
    constexpr int SPAN = (RUN - 1) * SW + K;   // window columns of one run
    constexpr int NS = SH == 1 ? K : 2;        // output rows whose sums are in flight (stride 2: 3x3 only)
    constexpr int U = SH == 1 ? K : 4;         // steps per unrolled group: set indices stay static
    constexpr int TAPS = K * K;
    constexpr int WQ = (TAPS + 1) * CG;        // float4 per weight slot: taps + bias
    extern __shared__ float4 sm4[];
    float4* const wslot = sm4;                                  // [2][10][CG]
    T* const ring = reinterpret_cast<T*>(sm4 + 2 * WQ);         // [NR][iw][CG * 4]
    const int row_elems = g.iw * CG * 4;
    const int nt = blockDim.x, tid = threadIdx.x;
    if ((int)blockIdx.x >= g.total) return;

    // Issue side: the next row to copy is row `it` of unit `iu` (this block's
    // ik-th unit).  Thread tid copies the 16-byte chunk cq of pixels p0,
    // p0 + pstep, ... of each row, so its source and destination addresses
    // advance by fixed steps and only the row start changes per row.
    const int cq = tid % CPP, p0 = tid / CPP, pstep = nt / CPP;
    const size_t row_pitch = (size_t)p.wi * p.in_cstride;           // elements between input rows
    const size_t src_step = (size_t)pstep * p.in_cstride;
    const uint32_t dst_step = (uint32_t)(pstep * CG * 4 * sizeof(T));
    const uint32_t ring_u32 = (uint32_t)__cvta_generic_to_shared(ring) + (uint32_t)((p0 * CG + cq * QPC) * 4 * sizeof(T));
    const T* const in_base = static_cast<const T*>(p.in) + p.in_coff + cq * QPC * 4;
    int iu = blockIdx.x, it = 0, ik = 0, islot = 0;
    int i_y0 = 0, i_x0 = 0, i_grp = 0;   // unit's first input row, this thread's first column, channel group
    const T* i_img = nullptr;            // unit's image at this thread's channels
    auto start_unit = [&]() {
        int img, seg, bx;
        band_decode(g, iu, img, seg, bx, i_grp);
        i_y0 = seg * g.bh * SH - p.pt;
        i_x0 = bx * g.bw * SW - p.pl + p0;
        i_img = in_base + (size_t)img * p.hi * row_pitch + i_grp * CG * 4;
    };
    start_unit();
    auto issue_row = [&]() {
        if (iu < g.total) {
            const int y = i_y0 + it;
            if (y >= 0 && y < p.hi) {
                const T* src = i_img + (size_t)y * row_pitch + (ptrdiff_t)i_x0 * p.in_cstride;
                uint32_t dst = ring_u32 + (uint32_t)(islot * row_elems * sizeof(T));
                for (int pix = p0, x = i_x0; pix < g.iw; pix += pstep, x += pstep, src += src_step, dst += dst_step) {
                    const bool ok = (unsigned)x < (unsigned)p.wi;
                    cp_async16_u32(dst, ok ? src : i_img, ok);
                }
            } else {   // a padding row: zero-fill
                uint32_t dst = ring_u32 + (uint32_t)(islot * row_elems * sizeof(T));
                for (int pix = p0; pix < g.iw; pix += pstep, dst += dst_step) cp_async16_u32(dst, i_img, false);
            }
            if (it == 0) {
                float4* wd = wslot + (ik & 1) * WQ;
                const int c0 = i_grp * CG * 4;
                for (int i = tid; i < WQ; i += nt) {
                    const int t = i / CG, q = i - t * CG;
                    if (t < TAPS) cp_async16(wd + i, p.weight + (size_t)t * p.c + c0 + q * 4, true);
                    else cp_async16(wd + i, p.bias ? p.bias + c0 + q * 4 : p.weight, p.bias != nullptr);
                }
            }
            if (++it == g.ni) {
                it = 0;
                ++ik;
                iu += gridDim.x;
                if (iu < g.total) start_unit();
            }
        }
        cp_async_commit();   // one group per row, empty past the last unit
        islot = islot == NR - 1 ? 0 : islot + 1;
    };

    for (int k = 0; k < D; ++k) issue_row();

    const int q = tid % CG, rx = tid / CG;
    const bool active = rx < g.sx;
    int cslot = 0, kord = 0;
    for (int u = blockIdx.x; u < g.total; u += gridDim.x, ++kord) {
        int img, seg, bx, grp;
        band_decode(g, u, img, seg, bx, grp);
        const int oy0 = seg * g.bh, ox0 = bx * g.bw + rx * RUN;
        const int rows = min(g.bh, p.ho - oy0);
        const int c = grp * CG * 4 + q * 4;
        const size_t obase = ((size_t)img * p.ho + oy0) * p.wo * p.c + c;   // + (j * wo + ox) * c
        float4 bias = make_float4(0.f, 0.f, 0.f, 0.f);
        const float4* const w = wslot + (kord & 1) * WQ + q;   // [tap * CG]: broadcast reads
        float4 acc[NS][RUN];
#pragma unroll
        for (int s = 0; s < NS; ++s)
#pragma unroll
            for (int r = 0; r < RUN; ++r) acc[s][r] = bias;
        for (int t0 = 0; t0 < g.ni; t0 += U) {
#pragma unroll
            for (int r = 0; r < U; ++r) {
                const int t = t0 + r;
                if (t >= g.ni) break;   // block-uniform
                cp_async_wait<D - 1>();  // row t (and, at t == 0, the unit's weights) has landed
                __syncthreads();         // ... for every thread; the slot of row t - 1 is free
                issue_row();
                if (r == 0 && t0 == 0) bias = w[TAPS * CG];
                if (active) {
                    const T* row = ring + cslot * row_elems + (rx * RUN * SW * CG + q) * 4;
                    float4 win[SPAN];
#pragma unroll
                    for (int i = 0; i < SPAN; ++i) win[i] = to4(row + i * CG * 4);
#pragma unroll
                    for (int ky = K - 1; ky >= 0; --ky) {
                        if (pmod(r - ky, SH) != 0) continue;          // static: row t is not tap row ky of any output
                        const int j = (t - ky) / SH;                   // output row (in the segment) this tap row feeds
                        if (t < ky || j >= rows) continue;
                        float4* a = acc[pmod(fdiv(r - ky, SH), NS)];
                        if (ky == 0) {
#pragma unroll
                            for (int rr = 0; rr < RUN; ++rr) a[rr] = make_float4(0.f, 0.f, 0.f, 0.f);
                        }
#pragma unroll
                        for (int kx = 0; kx < K; ++kx) {
                            const float4 wv = w[(ky * K + kx) * CG];
#pragma unroll
                            for (int rr = 0; rr < RUN; ++rr) a[rr] = f4_vfma(win[rr * SW + kx], wv, a[rr]);
                        }
                        if (ky == K - 1) {   // output row j is complete
                            const size_t orow = obase + ((size_t)j * p.wo + ox0) * p.c;
                            T* o = static_cast<T*>(p.out) + orow;
#pragma unroll
                            for (int rr = 0; rr < RUN; ++rr) {
                                if (ox0 + rr >= p.wo) break;
                                float4 v = f4_add(a[rr], bias);
                                if constexpr (!PLAIN) {
                                    v = f4_act(v, p.act);
                                    if (p.residual)
                                        v = f4_add(v, load4(static_cast<const T*>(p.residual) + orow + (size_t)rr * p.c));
                                }
                                store4(o + (size_t)rr * p.c, v);
                            }
                        }
                    }
                }
                cslot = cslot == NR - 1 ? 0 : cslot + 1;
            }
        }
    }
    cp_async_wait<0>();
}

// Units, bands and the ring depth for one launch.  Bands are at most 32 runs
// (128 outputs) wide so a block is at most 8 quads x 32 runs = 256 threads;
// tall maps are cut into segments of at least 8 rows until there are a few
// units per resident block.
template <typename T, int CG, int K, int SH, int SW>
DwBand band_geometry(const DwParams& p, int resident) {
    constexpr int RUN = band_run(K);
    DwBand g{};
    const int runs = (p.wo + RUN - 1) / RUN;
    const int sx_max = 256 / CG < 32 ? 256 / CG : 32;
    g.bands = (runs + sx_max - 1) / sx_max;
    g.sx = (runs + g.bands - 1) / g.bands;
    g.bw = g.sx * RUN;
    g.iw = (g.bw - 1) * SW + K;
    g.groups = p.c / (4 * CG);
    const long long base = (long long)p.n * g.groups * g.bands;
    const long long want = 4LL * resident;
    int segs = 1;
    if (base < want) {
        const long long need = (want + base - 1) / base;
        const int max_segs = (p.ho + 7) / 8;
        segs = (int)(need < max_segs ? need : max_segs);
        if (segs < 1) segs = 1;
    }
    g.bh = (p.ho + segs - 1) / segs;
    g.segs = (p.ho + g.bh - 1) / g.bh;
    g.ni = (g.bh - 1) * SH + K;
    const long long total = base * g.segs;
    g.total = total > 0x7fffffffLL ? -1 : (int)total;
    return g;
}

template <typename T, int CG, int K, int SH, int SW, int NR, bool PLAIN>
cudaError_t launch_band_nr(const DwParams& p, const DwBand& g, int nt, cudaStream_t stream) {
    auto kernel = dwconv_band_kernel<T, CG, K, SH, SW, NR, PLAIN>;
    const size_t smem = 2 * (K * K + 1) * CG * sizeof(float4) + (size_t)NR * g.iw * CG * 4 * sizeof(T);
    static std::atomic<int> regs{0};
    // The shared-memory limit is a per-device attribute: set on every device
    // the kernel runs on (the register count below is the same on all).
    {
        const cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), (int)kSmemLimit);
        if (e != cudaSuccess) return e;
    }
    int nregs = regs.load(std::memory_order_acquire);
    if (!nregs) {
        cudaFuncAttributes fa{};
        cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
        if (e != cudaSuccess) return e;
        nregs = fa.numRegs > 0 ? fa.numRegs : 1;
        regs.store(nregs, std::memory_order_release);
    }
    if (smem > kSmemLimit) return cudaErrorInvalidConfiguration;
    const int blocks_per_sm = resident_blocks(nregs, nt, smem);
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long cap = (long long)sms * blocks_per_sm;
    const int grid = (int)(g.total < cap ? g.total : cap);
    kernel<<<grid, nt, smem, stream>>>(p, g);
    return cudaGetLastError();
}

template <typename T, int CG, int K, int SH, int SW>
cudaError_t launch_band(const DwParams& p, cudaStream_t stream) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const DwBand g = band_geometry<T, CG, K, SH, SW>(p, 2 * sms);
    if (g.total < 0) return cudaErrorInvalidConfiguration;
    if (g.total == 0) return cudaSuccess;
    const int nt = (CG * g.sx + 31) / 32 * 32;
    const size_t row_bytes = (size_t)g.iw * CG * 4 * sizeof(T);
    // The weight slot of a block's unit k + 2 is refilled D rows before that
    // unit starts while unit k still reads its own: a unit must span at least
    // D rows.
    const bool plain = p.act == ACT_NONE && !p.residual;
    if (row_bytes <= 6 * 1024 && g.ni >= 7)
        return plain ? launch_band_nr<T, CG, K, SH, SW, 8, true>(p, g, nt, stream)
                     : launch_band_nr<T, CG, K, SH, SW, 8, false>(p, g, nt, stream);
    return plain ? launch_band_nr<T, CG, K, SH, SW, 4, true>(p, g, nt, stream)
                 : launch_band_nr<T, CG, K, SH, SW, 4, false>(p, g, nt, stream);
}

template <typename T, int K, int SH, int SW>
cudaError_t launch_band_cg(const DwParams& p, cudaStream_t stream) {
    const int quads = p.c / 4;
    if (quads % 8 == 0) return launch_band<T, 8, K, SH, SW>(p, stream);
    if (quads % 4 == 0) return launch_band<T, 4, K, SH, SW>(p, stream);
    if (quads % 2 == 0) return launch_band<T, 2, K, SH, SW>(p, stream);
    if constexpr (sizeof(T) == 4) return launch_band<T, 1, K, SH, SW>(p, stream);
    return cudaErrorInvalidValue;
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
// 3x3 convs run on the rolling-row kernel unless `kernel` asks for the tiled
// one (1); every other geometry on the tiled kernel.  The rolling-row kernel
// also covers 5x5 (kernel 2 only): with the two-column runs that five rows of
// sums in flight leave room for, it is slower there than the tiled kernel
// (detector neck 5x5: 123 -> 131 us).
template <typename T>
cudaError_t launch_dw_t(const DwParams& p, cudaStream_t stream, int kernel) {
    if (p.kh == 3 && p.kw == 3) {
        const bool band = kernel != 1;
        if (p.sh == 1 && p.sw == 1) return band ? launch_band_cg<T, 3, 1, 1>(p, stream) : launch_cg<T, 3, 3, 1, 1>(p, stream);
        if (p.sh == 2 && p.sw == 2) return band ? launch_band_cg<T, 3, 2, 2>(p, stream) : launch_cg<T, 3, 3, 2, 2>(p, stream);
        if (p.sh == 2 && p.sw == 1) return band ? launch_band_cg<T, 3, 2, 1>(p, stream) : launch_cg<T, 3, 3, 2, 1>(p, stream);
        return cudaErrorInvalidValue;
    }
    if (p.sh != 1 || p.sw != 1) return cudaErrorInvalidValue;
    if (p.kh == 5 && p.kw == 5 && kernel == 2) return launch_band_cg<T, 5, 1, 1>(p, stream);
    if (kernel == 2) return cudaErrorInvalidValue;
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

cudaError_t launch_dwconv_kernel(const DwParams& p, cudaStream_t stream, int kernel) {
    if (p.c % 4 || p.in_coff % 4 || p.in_cstride % 4) return cudaErrorInvalidValue;
    // 16-byte copies: BF16 views need 8-channel alignment.
    if (p.dtype == DT_BF16 && (p.c % 8 || p.in_coff % 8 || p.in_cstride % 8)) return cudaErrorInvalidValue;
    if (kernel < 0 || kernel > 2) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_dw_t<float>(p, stream, kernel) : launch_dw_t<__nv_bfloat16>(p, stream, kernel);
}

cudaError_t launch_dwconv(const DwParams& p, cudaStream_t stream) { return launch_dwconv_kernel(p, stream, 0); }

}  // namespace ppocr
