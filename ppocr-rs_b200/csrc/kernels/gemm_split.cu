// FP32-class tcgen05 GEMM over FP32 activations and weights ("split" GEMM).
//
//   C[m, n] = act(sum_k (A[m, k] g[img, k]) W[n, k] + bias) (+ residual r[m, n] h[img, n])
//
// Both operands are carried as three BF16 pieces, x = x0 + x1 + x2 with
// x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1) (24 significand
// bits: the FP32 value for normal ranges), and the six products with
// i + j <= 2 are accumulated in FP32 in TMEM; the dropped x1 w2 + x2 w1 +
// x2 w2 are ~2^-24 relative, so every product carries FP32-class error.
// The weights are split once on the host; A is split on the fly:
//
//   warp 0 / lane 0   TMA: A as FP32 (two 128-row x 32-column 128-byte-swizzled
//                     boxes per 64-wide K block) and the three W pieces of the
//                     tile's BN output channels, into a two-stage ring;
//   warps 2-5         converters: one A row per thread, FP32 tile from shared
//                     memory, optional SE gate, split into the three BF16 planes
//                     in the UMMA K-major 128-byte-swizzled layout;
//   warp 1 / lane 0   MMA: per 16-wide K step three tcgen05.mma, plane-major:
//                     a0 x [w0 w1 w2] (N = 3 BN) into [D S1 S2], a1 x [w0 w1]
//                     (N = 2 BN) into [S1 S2] and a2 x w0 (N = BN) into S1, so
//                     TMEM holds D = a0 w0, S1 = a0 w1 + a1 w0 + a2 w0 and
//                     S2 = a0 w2 + a1 w1 side by side, each A plane is read
//                     once per step, and the dominant sum D is rounded once
//                     per step; two accumulators, so a tile's MMAs overlap
//                     the previous tile's epilogue (one, twice as wide, for
//                     the long-K GEMMs whose dominant-sum chunks fill TMEM);
//   warps 6-13        epilogue: (S2 + S1) + D, bias, activation, optional
//                     gated / upsampled residual, 64-byte-swizzled staging
//                     tile, TMA store.  Two groups of four warps (one per
//                     TMEM lane quarter) take alternate tiles, each owning
//                     one accumulator buffer, so two tiles' epilogues overlap
//                     (with one buffer each group takes half of every tile's
//                     columns); the residual is fetched one 16-column group
//                     ahead.
//
// Every mbarrier wait is bounded by the GPU's global timer; on expiry the
// kernel records a code in *err (or g_split_error), stops, lets its copies
// and MMAs in flight land, frees its TMEM and returns.  No clusters, no
// multicast: each CTA loads its own tiles from this GPU's memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace ppocr {

__device__ int g_split_error = 0;

namespace {

constexpr int BM = 128, BK = 64, THREADS = 448, MAX_BN = 64;
constexpr int MAX_A = 6, PLANE_STAGES = 2;             // FP32 ring depth bound; BF16 plane ring
constexpr int MAX_PLANE_STAGES = 4;                    // plane ring bound (pre-split A has no FP32 ring)
constexpr int BOX_BYTES = BM * 32 * 4;                 // one FP32 box: 128 rows x 32 columns
constexpr int PLANE_BYTES = BM * BK * 2;               // one BF16 piece of a 128 x 64 tile
constexpr int PLANES_STAGE = 3 * PLANE_BYTES;          // 48 KB
constexpr int EPI_WARPS = 8, STAGE_OUT = 32 * 64;      // staging: 32 rows x 16 FP32 columns
#ifndef SPLIT_STAGE_BUFS
#define SPLIT_STAGE_BUFS 2
#endif
#ifndef SPLIT_SINGLE_BLOCK_PLANES
#define SPLIT_SINGLE_BLOCK_PLANES 2
#endif
// Output staging buffers per epilogue warp: with two, a store drains while the
// next group is written (one when shared memory would leave a single FP32
// stage).  BF16 plane ring depth of single-K-block GEMMs: with two, the
// converters split tile i + 1 while the MMAs read tile i (measured 97 -> 86 us
// on the detector's stage-0 GEMMs against one buffer and a deeper FP32 ring).
constexpr int STAGE_BUFS = SPLIT_STAGE_BUFS;
#ifndef SPLIT_ROLE_BACKOFF
#define SPLIT_ROLE_BACKOFF 1
#endif
// The single-thread producer and MMA roles sleep briefly between polls once a
// wait has spun a while, leaving the issue slots of their sub-partitions to
// the converter and epilogue warps that share them.
constexpr bool ROLE_BACKOFF = SPLIT_ROLE_BACKOFF != 0;
// Resident W of a CTA's N tile (all K blocks) up to this size; larger W
// streams through the FP32 ring beside each A stage.
constexpr int W_RESIDENT_MAX = 48 * 1024;
constexpr int SINGLE_BLOCK_PLANES = SPLIT_SINGLE_BLOCK_PLANES;
constexpr int SMEM_MAX = 227 * 1024;                   // opt-in shared memory per block

// K blocks (64 wide) summed into one dominant-sum accumulator.  The tensor
// core rounds its FP32 accumulator toward zero once per 16-wide K step, so the
// error of a sum grows with the steps and the magnitude accumulated; 5 blocks
// (K = 320) keep it at the CUDA-core FP32 kernels' level, and longer sums are
// split over several accumulators added in the epilogue (round to nearest).
constexpr int KCHUNK = 5;
#ifndef SPLIT_SINGLE_ACC_CHUNKS
#define SPLIT_SINGLE_ACC_CHUNKS 3
#endif
constexpr int SINGLE_ACC_CHUNKS = SPLIT_SINGLE_ACC_CHUNKS;

// Shared memory, 1024-byte aligned pieces: [resident W] [plane ring]
// [epilogue staging] [FP32 ring: per stage the A boxes, then (streamed) W].
struct SplitArgs {
    SplitGemmParams p;
    int bn, kt, m_tiles, n_tiles, tmem_cols;
    int kchunk, dchunks;    // K blocks per dominant-sum accumulator, and their count
    int nacc;               // TMEM accumulator buffers: 2 (a tile's MMAs overlap the previous tile's epilogue) or 1
    int tiles_y, tiles_x;   // conv mode: tile grid per image
    int cpt;                // conv mode: input channels per tap (32: two taps per K block; a multiple of 64: cpt / 64 blocks per tap)
    int w_resident;         // 1: every tile of a CTA has the same N tile, whose W (all K blocks) is loaded once
    int w_block;            // resident W bytes per K block, 1024-aligned
    int stages;             // FP32 ring depth
    int plane_stages;       // BF16 plane ring depth (1 when one K block covers the GEMM)
    int stage_bufs;         // output staging buffers per epilogue warp (1 or 2)
    int presplit;           // 1: A arrives as BF16 pieces (p.a_planes) straight into the plane ring
    int a_stage_bytes;      // one FP32 ring stage (A boxes + streamed W), 1024-aligned
    int a_box_bytes;        // the A boxes of a stage (1 or 2 boxes of 16 KB)
    int w_bytes;            // the three W pieces of one (K block, N tile)
    int w_region;           // resident W bytes (0 when streamed), 1024-aligned
    uint64_t wait_ns;
};

__device__ __forceinline__ void report(const SplitGemmParams& p, int code) { atomicExch(p.err ? p.err : &g_split_error, code); }


// Eight consecutive values -> their three BF16 pieces, packed as 16-byte
// chunks.  A is split by truncation: x0 = the top 8 significant bits of x (its
// upper 16 bits), x1 = the top 8 of r = x - x0 (exact), x2 = r - x1 (exact,
// at most 8 significant bits, so a BF16 holds it exactly): x0 + x1 + x2 == x
// with no rounding, |x1| < 2^-7 |x|, |x2| < 2^-15 |x|.  With the weights split
// to nearest on the host (|w1| <= 2^-9 |w|, |w2| <= 2^-18 |w|), the three
// dropped products are below 2^-24 of |x w|.  Packed FP32 subtractions; each
// BF16 pair is the upper halves of two FP32 words (one byte permute).
__device__ __forceinline__ void split8(const float (&x)[8], uint4& hi, uint4& mid, uint4& lo) {
    uint32_t h[4], m[4], l[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const uint32_t ua = __float_as_uint(x[2 * t]), ub = __float_as_uint(x[2 * t + 1]);
        h[t] = __byte_perm(ua, ub, 0x7632);
        // -x0 in one logic op: the upper half with the sign flipped.
        const float2 nx0 = make_float2(__uint_as_float((ua & 0xFFFF0000u) ^ 0x80000000u),
                                       __uint_as_float((ub & 0xFFFF0000u) ^ 0x80000000u));
        const float2 r = __fadd2_rn(make_float2(x[2 * t], x[2 * t + 1]), nx0);
        const uint32_t ra = __float_as_uint(r.x), rb = __float_as_uint(r.y);
        m[t] = __byte_perm(ra, rb, 0x7632);
        const float2 nx1 = make_float2(__uint_as_float((ra & 0xFFFF0000u) ^ 0x80000000u),
                                       __uint_as_float((rb & 0xFFFF0000u) ^ 0x80000000u));
        const float2 r2 = __fadd2_rn(r, nx1);
        l[t] = __byte_perm(__float_as_uint(r2.x), __float_as_uint(r2.y), 0x7632);
    }
    hi = make_uint4(h[0], h[1], h[2], h[3]);
    mid = make_uint4(m[0], m[1], m[2], m[3]);
    lo = make_uint4(l[0], l[1], l[2], l[3]);
}

template <int ACT>
__device__ __forceinline__ float act_exact(float v) {
    if constexpr (ACT == ACT_NONE) return v;
    else return apply_act(v, ACT);
}

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU 0.5 v (1 + erf(v / sqrt 2)) with the Abramowitz-Stegun 7.1.26 erf of
// the reference (src/cpu/kernels/mod.rs:2395-2403), two values at a time in
// packed FP32: the reciprocal 1 / (1 + 0.3275911 a) from the hardware
// approximation refined by one Newton-Raphson step (within an ulp), exp(-a^2)
// as 2^(-a^2 log2 e) on the hardware exp2 (relative error ~2^-22).  FP32-class
// (a few ulps from the libm formula), at a quarter of its instructions.
__device__ __forceinline__ void gelu_f32x2(float& v0, float& v1) {
    const float2 v = make_float2(v0, v1);
    const float2 x = __fmul2_rn(v, make_float2(0.70710678118654752f, 0.70710678118654752f));
    const float2 a = make_float2(fabsf(x.x), fabsf(x.y));
    const float2 d = __ffma2_rn(a, make_float2(0.3275911f, 0.3275911f), make_float2(1.f, 1.f));
    float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
    const float2 r = __ffma2_rn(make_float2(-d.x, -d.y), t, make_float2(1.f, 1.f));
    t = __ffma2_rn(t, r, t);
    float2 q = __ffma2_rn(t, make_float2(1.0614054f, 1.0614054f), make_float2(-1.4531521f, -1.4531521f));
    q = __ffma2_rn(t, q, make_float2(1.4214138f, 1.4214138f));
    q = __ffma2_rn(t, q, make_float2(-0.28449672f, -0.28449672f));
    q = __ffma2_rn(t, q, make_float2(0.2548296f, 0.2548296f));
    q = __fmul2_rn(t, q);
    const float2 m = __fmul2_rn(a, make_float2(-1.4426950408889634f, -1.4426950408889634f));
    const float2 y = __fmul2_rn(m, a);
    const float2 ex = make_float2(ex2_approx(y.x), ex2_approx(y.y));
    const float2 e = __ffma2_rn(make_float2(-q.x, -q.y), ex, make_float2(1.f, 1.f));
    const float2 h = __fmul2_rn(v, make_float2(0.5f, 0.5f));
    const float2 o = __ffma2_rn(h, make_float2(copysignf(e.x, x.x), copysignf(e.y, x.y)), h);
    v0 = o.x;
    v1 = o.y;
}

template <int ACT>
__global__ void __launch_bounds__(THREADS, 1) gemm_split_kernel(const __grid_constant__ CUtensorMap tma_a,
                                                                const __grid_constant__ CUtensorMap tma_w,
                                                                const __grid_constant__ CUtensorMap tma_c, SplitArgs args) {
    const SplitGemmParams& p = args.p;
    extern __shared__ uint8_t smem_raw[];
    // full: TMA of a FP32 stage landed; f32_empty: its A rows converted;
    // w_free: the MMAs are done with its streamed W; planes_full / planes_empty:
    // the BF16 plane ring between converters and MMA.
    __shared__ __align__(8) uint64_t full[MAX_A], f32_empty[MAX_A], w_free[MAX_A], planes_full[MAX_PLANE_STAGES],
        planes_empty[MAX_PLANE_STAGES], w_ready, acc_full[2], acc_empty[2], drain_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    // Up to the next 1024-byte boundary by offsetting the shared pointer itself:
    // the compiler keeps its address space, so the tile reads and writes below
    // are shared-memory instructions rather than generic ones.
    uint8_t* smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sw_res = smem;
    uint8_t* splanes = smem + args.w_region;
    uint8_t* sout = splanes + args.plane_stages * PLANES_STAGE;
    uint8_t* sring = sout + EPI_WARPS * args.stage_bufs * STAGE_OUT;
    const int S = args.stages;
    const int PS = args.plane_stages;
    const int bn = args.bn;
    const bool wres = args.w_resident != 0;
    const bool presplit = args.presplit != 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = args.m_tiles * args.n_tiles;
    const uint64_t wait_ns = args.wait_ns;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(&full[s], 1);
            tc::mbar_init(&f32_empty[s], 128);
            tc::mbar_init(&w_free[s], 1);
        }
        for (int s = 0; s < PS; ++s) {
            // Converted planes: one arrival per converter thread; pre-split
            // planes: the producer's arrival plus the copies' bytes.
            tc::mbar_init(&planes_full[s], presplit ? 1 : 128);
            tc::mbar_init(&planes_empty[s], 1);
        }
        tc::mbar_init(&w_ready, 1);
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], (args.nacc == 2 ? 4 : 8) * 32);   // the epilogue warps of a buffer's tiles
        }
        tc::mbar_init(&drain_bar, 1);
        abort_flag = 0;
        tc::mbar_fence_init();
    }
    if (warp == 0) tc::tmem_alloc(&tmem_slot, (uint32_t)args.tmem_cols);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int last_it[MAX_A];
            for (int s = 0; s < MAX_A; ++s) last_it[s] = -1;
            if (wres) {
                // The CTA's tiles share one N tile (the grid is a multiple of
                // the N tile count, or one tile per CTA): its W never changes.
                const int n0w = (blockIdx.x % args.n_tiles) * bn;
                tc::mbar_expect_tx(&w_ready, (uint32_t)(args.kt * args.w_bytes));
                for (int kb = 0; kb < args.kt; ++kb)
#pragma unroll
                    for (int j = 0; j < 3; ++j)
                        tc::tma_load_2d(sw_res + kb * args.w_block + j * bn * 128, &tma_w, &w_ready, kb * BK, j * p.n_pad + n0w);
            }
            int it = 0;
            int last_pit[MAX_PLANE_STAGES];
            for (int s = 0; s < MAX_PLANE_STAGES; ++s) last_pit[s] = -1;
            for (int tile = blockIdx.x; tile < total && !abort_flag; tile += gridDim.x) {
                const int m0 = (tile / args.n_tiles) * BM, n0 = (tile % args.n_tiles) * bn;
                for (int kb = 0; kb < args.kt; ++kb, ++it) {
                    const int s = it % S;
                    if (presplit) {
                        // The three pieces of the A tile straight into plane
                        // stage sp once the MMAs have released it (piece j of
                        // row r is row j m + r of the planes; rows past m of
                        // the last tile read the next piece's rows, whose
                        // outputs are never stored), W as before.
                        const int sp = it % PS;
                        const uint32_t par = ((it / PS) + 1) & 1;
                        if ((it >= PS && !tc::mbar_wait(&planes_empty[sp], par, ROLE_BACKOFF, wait_ns, &abort_flag)) ||
                            (!wres && it >= S &&
                             !tc::mbar_wait(&w_free[s], ((it / S) + 1) & 1, ROLE_BACKOFF, wait_ns, &abort_flag))) {
                            report(p, 1);
                            abort_flag = 1;
                            break;
                        }
                        if (p.skip_load && it == 0 && blockIdx.x == 0) continue;
                        const int k0 = kb * BK;
                        uint8_t* pl = splanes + sp * PLANES_STAGE;
                        tc::mbar_expect_tx(&planes_full[sp], 3u * PLANE_BYTES);
#pragma unroll
                        for (int j = 0; j < 3; ++j) tc::tma_load_2d(pl + j * PLANE_BYTES, &tma_a, &planes_full[sp], k0, j * p.m + m0);
                        last_pit[sp] = it;
                        if (!wres) {
                            uint8_t* w = sring + (size_t)s * args.a_stage_bytes;
                            tc::mbar_expect_tx(&full[s], (uint32_t)args.w_bytes);
#pragma unroll
                            for (int j = 0; j < 3; ++j) tc::tma_load_2d(w + j * bn * 128, &tma_w, &full[s], k0, j * p.n_pad + n0);
                            last_it[s] = it;
                        }
                        continue;
                    }
                    if (it >= S) {
                        const uint32_t par = ((it / S) + 1) & 1;
                        if (!tc::mbar_wait(&f32_empty[s], par, ROLE_BACKOFF, wait_ns, &abort_flag) ||
                            (!wres && !tc::mbar_wait(&w_free[s], par, ROLE_BACKOFF, wait_ns, &abort_flag))) {
                            report(p, 1);
                            abort_flag = 1;
                            break;
                        }
                    }
                    if (p.skip_load && it == 0 && blockIdx.x == 0) continue;
                    const int k0 = kb * BK;
                    const bool two = k0 + 32 < p.k;
                    uint8_t* f = sring + (size_t)s * args.a_stage_bytes;
                    tc::mbar_expect_tx(&full[s], (two ? 2u : 1u) * BOX_BYTES + (wres ? 0u : (uint32_t)args.w_bytes));
                    if (p.conv) {
                        // K order (tap, channel).  32 channels: taps 2 kb and
                        // 2 kb + 1, one box each; a multiple of 64: block kb is
                        // channels [64 (kb mod bpt), + 64) of tap kb / bpt, in
                        // two 32-channel boxes.  The tile's 8 x 16 output pixels
                        // read input pixels (oy s + ky - pt, ox s + kx - pl);
                        // outside the image reads 0.
                        const int mt = tile / args.n_tiles, per = args.tiles_y * args.tiles_x;
                        const int img = mt / per, rt = mt - img * per;
                        const int yb = (rt / args.tiles_x) * 8 * p.stride - p.pt;
                        const int xb = (rt % args.tiles_x) * 16 * p.stride - p.pl;
                        const int bpt = args.cpt / 64;   // K blocks per tap (cpt >= 64)
                        for (int h = 0; h < (two ? 2 : 1); ++h) {
                            const int tap = args.cpt == 32 ? 2 * kb + h : kb / bpt;
                            const int c0 = args.cpt == 32 ? 0 : (kb - tap * bpt) * 64 + 32 * h;
                            const int ky = tap / p.kw, kx = tap - ky * p.kw;
                            tc::tma_load_4d(f + h * BOX_BYTES, &tma_a, &full[s], c0, xb + kx, yb + ky, img);
                        }
                    } else {
                        tc::tma_load_2d(f, &tma_a, &full[s], k0, m0);
                        if (two) tc::tma_load_2d(f + BOX_BYTES, &tma_a, &full[s], k0 + 32, m0);
                    }
                    if (!wres) {
                        uint8_t* w = f + args.a_box_bytes;   // after the boxes a stage can hold
#pragma unroll
                        for (int j = 0; j < 3; ++j) tc::tma_load_2d(w + j * bn * 128, &tma_w, &full[s], k0, j * p.n_pad + n0);
                    }
                    last_it[s] = it;
                }
            }
            // Every copy issued has landed before the CTA can exit.
            for (int s = 0; s < S; ++s)
                if (last_it[s] >= 0) tc::mbar_wait(&full[s], (last_it[s] / S) & 1, false, wait_ns);
            for (int s = 0; s < PS; ++s)
                if (last_pit[s] >= 0) tc::mbar_wait(&planes_full[s], (last_pit[s] / PS) & 1, false, wait_ns);
            if (wres) tc::mbar_wait(&w_ready, 0, false, wait_ns);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t id3 = tc::idesc_bf16(BM, 3 * bn), id2 = tc::idesc_bf16(BM, 2 * bn), id1 = tc::idesc_bf16(BM, bn);
            const uint64_t a_step = (uint64_t)(PLANE_BYTES >> 4);
            const uint64_t w1_step = (uint64_t)((bn * 128) >> 4);   // W piece 1 follows piece 0 (BN rows of 128 bytes)
            const int w_off = args.a_box_bytes;
            bool ok = !wres || tc::mbar_wait(&w_ready, 0, false, wait_ns, &abort_flag);
            if (!ok) {
                report(p, 6);
                abort_flag = 1;
            }
            int it = 0, ti = 0;
            for (int tile = blockIdx.x; ok && tile < total && !abort_flag; tile += gridDim.x, ++ti) {
                const int b = ti % args.nacc;
                if (ti >= args.nacc &&
                    !tc::mbar_wait(&acc_empty[b], ((ti / args.nacc) + 1) & 1, ROLE_BACKOFF, wait_ns, &abort_flag)) {
                    report(p, 2);
                    abort_flag = 1;
                    break;
                }
                tc::fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * (2 + args.dchunks) * bn);
                for (int kb = 0; kb < args.kt; ++kb, ++it) {
                    const int s = it % S, sp = it % PS;
                    if (!tc::mbar_wait(&planes_full[sp], (it / PS) & 1, ROLE_BACKOFF, wait_ns, &abort_flag) ||
                        (!wres && !tc::mbar_wait(&full[s], (it / S) & 1, ROLE_BACKOFF, wait_ns, &abort_flag))) {
                        report(p, 3);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc::fence_after();
                    const uint64_t ad = tc::sw128_desc(tc::smem_u32(splanes + sp * PLANES_STAGE));
                    const uint64_t bd = tc::sw128_desc(
                        tc::smem_u32(wres ? sw_res + kb * args.w_block : sring + (size_t)s * args.a_stage_bytes + w_off));
                    const int rem = (p.k - kb * BK) / 16;
                    const int nk = rem < 4 ? rem : 4;
                    const int chunk = kb / args.kchunk;
                    const bool chunk_start = kb == chunk * args.kchunk;
                    for (int kk = 0; kk < nk; ++kk) {   // +32 bytes per 16-element K step
                        // a0 x [w0 w1 w2] -> [D | S1 | S2]; a1 x [w0 w1] -> [S1 | S2];
                        // a2 x w0 -> S1.  D only ever receives a0 w0, so the
                        // accumulation rounding of the dominant sum happens once
                        // per step; S1 (2^-8 D) and S2 (2^-16 D) take the rest.
                        // Past the first kchunk K blocks the dominant sum moves to
                        // a fresh accumulator D_c (a0 x w0 alone, a0 x [w1 w2]
                        // into [S1 | S2]): the tensor core's accumulator rounding
                        // error grows with the magnitude summed into it.
                        if (chunk == 0) {
                            tc::mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, id3, (kb | kk) != 0 ? 1u : 0u);
                        } else {
                            tc::mma_bf16(acc + (uint32_t)((2 + chunk) * bn), ad + 2 * kk, bd + 2 * kk, id1,
                                         (chunk_start && kk == 0) ? 0u : 1u);
                            tc::mma_bf16(acc + (uint32_t)bn, ad + 2 * kk, bd + w1_step + 2 * kk, id2, 1u);
                        }
                        tc::mma_bf16(acc + (uint32_t)bn, ad + a_step + 2 * kk, bd + 2 * kk, id2, 1u);
                        tc::mma_bf16(acc + (uint32_t)bn, ad + 2 * a_step + 2 * kk, bd + 2 * kk, id1, 1u);
                    }
                    tc::commit(&planes_empty[sp]);
                    if (!wres) tc::commit(&w_free[s]);
                }
                if (!ok) break;
                tc::commit(&acc_full[b]);
            }
            tc::commit(&drain_bar);
            tc::mbar_wait(&drain_bar, 0, false, wait_ns);
        }
    } else if (warp < 6) {
        // Converters: thread r owns row r of every tile (idle when A arrives
        // pre-split).
        const int r = threadIdx.x - 64;
        const int swz = r & 7;
        int it = 0;
        for (int tile = presplit ? total : (int)blockIdx.x; tile < total; tile += gridDim.x) {
            if (abort_flag) break;
            const int m0 = (tile / args.n_tiles) * BM;
            const int row = m0 + r;
            const float* grow = (!p.conv && p.gate && row < p.m) ? p.gate + (size_t)(row / p.rows_per_image) * p.k : nullptr;
            bool ok = true;
            for (int kb = 0; kb < args.kt; ++kb, ++it) {
                const int s = it % S, sp = it % PS;
                if (!tc::mbar_wait(&full[s], (it / S) & 1, true, wait_ns, &abort_flag) ||
                    (it >= PS && !tc::mbar_wait(&planes_empty[sp], ((it / PS) + 1) & 1, true, wait_ns, &abort_flag))) {
                    report(p, 4);
                    abort_flag = 1;
                    ok = false;
                    break;
                }
                const uint8_t* f = sring + (size_t)s * args.a_stage_bytes + r * 128;
                uint8_t* pl = splanes + sp * PLANES_STAGE + r * 128;
                const int k0 = kb * BK;
                const int rem = (p.k - k0) / 8;
                const int nq = rem < 8 ? rem : 8;   // 8-value chunks that hold data
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (q >= nq) break;
                    const uint8_t* fb = f + (q >> 2) * BOX_BYTES;
                    const int c0 = (q & 3) * 2;
                    const float4 u = *reinterpret_cast<const float4*>(fb + ((c0 ^ swz) << 4));
                    const float4 v = *reinterpret_cast<const float4*>(fb + (((c0 + 1) ^ swz) << 4));
                    float x[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
                    if (grow) {
                        const float4 g0 = __ldg(reinterpret_cast<const float4*>(grow + k0 + q * 8));
                        const float4 g1 = __ldg(reinterpret_cast<const float4*>(grow + k0 + q * 8 + 4));
                        x[0] *= g0.x; x[1] *= g0.y; x[2] *= g0.z; x[3] *= g0.w;
                        x[4] *= g1.x; x[5] *= g1.y; x[6] *= g1.z; x[7] *= g1.w;
                    }
                    uint4 hi, mid, lo;
                    split8(x, hi, mid, lo);
                    const uint32_t off = (uint32_t)((q ^ swz) << 4);
                    *reinterpret_cast<uint4*>(pl + off) = hi;
                    *reinterpret_cast<uint4*>(pl + PLANE_BYTES + off) = mid;
                    *reinterpret_cast<uint4*>(pl + 2 * PLANE_BYTES + off) = lo;
                }
                tc::fence_proxy_async();
                tc::mbar_arrive(&planes_full[sp]);
                tc::mbar_arrive(&f32_empty[s]);
            }
            if (!ok) break;
        }
    } else {
        // Epilogue warps 6-13: two groups of four, one warp per TMEM lane
        // quarter (warp % 4) in each.  With two accumulator buffers group
        // g = (warp - 6) / 4 owns buffer g and so every other tile: two tiles'
        // epilogues run at once, and each warp walks all of its tile's
        // 16-column groups.  With one buffer both groups take every tile, group
        // g the g-th half of its 16-column groups (so neither can wait on a
        // later tile's phase of the shared barrier).
        const int q = warp & 3, grp = (warp - 6) >> 2;
        uint8_t* stage0 = sout + (warp - 6) * args.stage_bufs * STAGE_OUT;
        int sbuf = 0;
        const int swz = (lane >> 1) & 3;   // 64-byte swizzle: chunk ^= row bits 1-2
        int ti = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
            if (args.nacc == 2 && (ti & 1) != grp) continue;
            if (abort_flag) break;
            const int b = ti % args.nacc;
            const int m0 = (tile / args.n_tiles) * BM, n0 = (tile % args.n_tiles) * bn;
            const int row = m0 + q * 32 + lane;
            const bool live = row < p.m;
            const float* rp = nullptr;
            const float* hrow = nullptr;
            if (p.residual && p.conv) {
                // Conv mode: row r of the tile is output pixel (r / 16, r % 16)
                // of its 8 x 16 block; rows past the image edge add nothing.
                const int mt = tile / args.n_tiles, per = args.tiles_y * args.tiles_x;
                const int img = mt / per, rt = mt - img * per, r = q * 32 + lane;
                const int oy = (rt / args.tiles_x) * 8 + r / 16, ox = (rt % args.tiles_x) * 16 + r % 16;
                if (oy < p.ho && ox < p.wo) rp = p.residual + ((size_t)(img * p.ho + oy) * p.wo + ox) * p.ldr;
            }
            if (live && p.residual && !p.conv) {
                size_t rrow = (size_t)row;
                if (p.res_scale > 1) {
                    const int img_hw = p.out_h * p.out_w;
                    const int pimg = row / img_hw, rem = row % img_hw;
                    const int y = rem / p.out_w, x = rem % p.out_w;
                    const int rh = p.out_h / p.res_scale, rw = p.out_w / p.res_scale;
                    rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
                }
                rp = p.residual + rrow * p.ldr;
                if (p.res_gate) hrow = p.res_gate + (size_t)(row / p.rows_per_image) * p.n;
            }
            // The residual of a 16-column group, gated; issued one group ahead
            // (the first before the accumulator wait) so its latency overlaps.
            auto load_res = [&](int col0, float (&res)[16]) {
#pragma unroll
                for (int j = 0; j < 16; ++j) res[j] = 0.f;
                if (!rp || col0 >= p.n) return;
                if (col0 + 16 <= p.n && (p.ldr % 4) == 0) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        float4 v = __ldg(reinterpret_cast<const float4*>(rp + col0 + j));
                        if (hrow) v = f4_mul(v, __ldg(reinterpret_cast<const float4*>(hrow + col0 + j)));
                        res[j] = v.x; res[j + 1] = v.y; res[j + 2] = v.z; res[j + 3] = v.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (col0 + j < p.n) res[j] = hrow ? __ldg(rp + col0 + j) * __ldg(hrow + col0 + j) : __ldg(rp + col0 + j);
                }
            };
            float res[16];
            const int ngroups = bn / 16, gsplit = (ngroups + 1) / 2;
            const int cb0 = args.nacc == 2 || grp == 0 ? 0 : gsplit * 16;
            const int cb1 = args.nacc == 2 || grp == 1 ? bn : gsplit * 16;
            load_res(n0 + cb0, res);
            bool got = tc::mbar_wait(&acc_full[b], (ti / args.nacc) & 1, true, wait_ns, &abort_flag);
            got = __all_sync(0xffffffffu, got);
            if (!got) {
                if (lane == 0) report(p, 5);
                abort_flag = 1;
                break;
            }
            tc::fence_after();
            const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * (2 + args.dchunks) * bn);
            for (int cb = cb0; cb < cb1 && n0 + cb < p.n; cb += 16) {
                const int col0 = n0 + cb;
                uint32_t r0[16], r1[16], r2[16];
                tc::tmem_ld16_async(tb + (uint32_t)cb, r0);
                // Dominant sum: D_0 + D_1 + ... in order, rounded to nearest.
                for (int c = 1; c < args.dchunks; ++c) {
                    tc::tmem_ld16_async(tb + (uint32_t)((2 + c) * bn + cb), r1);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) r0[j] = __float_as_uint(__uint_as_float(r0[j]) + __uint_as_float(r1[j]));
                }
                tc::tmem_ld16_async(tb + (uint32_t)(bn + cb), r1);
                tc::tmem_ld16_async(tb + (uint32_t)(2 * bn + cb), r2);
                float nres[16];
                load_res(col0 + 16 < n0 + cb1 ? col0 + 16 : p.n, nres);
                const bool full_cols = col0 + 16 <= p.n;
                float bias[16];
                if (p.bias && full_cols) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        const float4 v = __ldg(reinterpret_cast<const float4*>(p.bias + col0 + j));
                        bias[j] = v.x; bias[j + 1] = v.y; bias[j + 2] = v.z; bias[j + 3] = v.w;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) bias[j] = (p.bias && col0 + j < p.n) ? __ldg(p.bias + col0 + j) : 0.f;
                }
                tc::tmem_wait_ld();
                float o[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    o[j] = ((__uint_as_float(r2[j]) + __uint_as_float(r1[j])) + __uint_as_float(r0[j])) + bias[j];
                if constexpr (ACT == ACT_GELU) {
#pragma unroll
                    for (int j = 0; j < 16; j += 2) gelu_f32x2(o[j], o[j + 1]);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) o[j] = act_exact<ACT>(o[j]);
                }
                if (rp) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) o[j] += res[j];
                }
                // This staging buffer's previous store (two groups back) has
                // finished reading it once at most one store is pending.
                uint8_t* stage = stage0 + sbuf * STAGE_OUT;
                uint8_t* line = stage + lane * 64;
                if (args.stage_bufs == 2) {
                    sbuf ^= 1;
                    if (lane == 0) tc::bulk_wait_read_1();
                } else if (lane == 0) {
                    tc::bulk_wait_read();
                }
                __syncwarp();
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    *reinterpret_cast<float4*>(line + ((c ^ swz) << 4)) = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
                tc::fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    if (p.conv) {
                        // The warp's 32 rows are two 16-pixel output rows of the tile.
                        const int mt = tile / args.n_tiles, per = args.tiles_y * args.tiles_x;
                        const int img = mt / per, rt = mt - img * per;
                        tc::tma_store_4d(&tma_c, stage, col0, (rt % args.tiles_x) * 16, (rt / args.tiles_x) * 8 + q * 2, img);
                    } else {
                        tc::tma_store_2d(&tma_c, stage, col0, m0 + q * 32);
                    }
                    tc::bulk_commit();
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) res[j] = nres[j];
            }
            tc::fence_before();
            tc::mbar_arrive(&acc_empty[b]);
        }
        if (lane == 0) tc::bulk_wait_all();
    }
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::tmem_dealloc(tmem, (uint32_t)args.tmem_cols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    }
    return fn;
}

bool make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
              uint32_t box_outer, CUtensorMapDataType type, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int ACT>
cudaError_t launch_act(const CUtensorMap& ma, const CUtensorMap& mw, const CUtensorMap& mc, const SplitArgs& a, int grid,
                       int smem, cudaStream_t stream) {
    cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(gemm_split_kernel<ACT>), SMEM_MAX - 1024);
    if (e != cudaSuccess) return e;
    gemm_split_kernel<ACT><<<grid, THREADS, smem, stream>>>(ma, mw, mc, a);
    return cudaGetLastError();
}

// 4D NHWC FP32 map: dims (channels, width, height, images), pixel pitch
// `pixel_bytes`; box (box_c, box_x, box_y, 1) traversed with element strides
// (1, stride, stride, 1).
bool make_map4(CUtensorMap* map, const void* base, uint64_t channels, uint64_t w, uint64_t h, uint64_t n, uint64_t pixel_bytes,
               uint32_t box_c, uint32_t box_x, uint32_t box_y, uint32_t stride, CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {channels, w, h, n};
    cuuint64_t strides[3] = {pixel_bytes, w * pixel_bytes, h * w * pixel_bytes};
    cuuint32_t box[4] = {box_c, box_x, box_y, 1};
    cuuint32_t estr[4] = {1, stride, stride, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

}  // namespace

int gemm_split_conv_cpt(int cin) {
    if (cin == 32) return 32;
    return cin > 32 && cin % 4 == 0 ? (cin + 63) / 64 * 64 : 0;
}

int gemm_split_tile_n(int n, int k) {
    // One tile when it fits, else equal tiles; any multiple of 16 (the
    // epilogue stores 16-column boxes, so none reaches the next tile).  The
    // widest tile is 64 columns, less when the dominant-sum accumulators of a
    // long K need the TMEM: two buffers of (2 + chunks) tile widths in 512
    // columns, or from SPLIT_SINGLE_ACC_CHUNKS chunks on one buffer of twice
    // the width (fewer N tiles, so A is read and split fewer times, for a
    // tile's MMAs no longer overlapping the previous tile's epilogue).  0 when
    // K needs more accumulators than fit at width 16.
    const int kt = (k + BK - 1) / BK;
    const int chunks = kt < 1 ? 1 : (kt + KCHUNK - 1) / KCHUNK;
    int max_bn = (chunks >= SINGLE_ACC_CHUNKS ? 512 : 256) / (2 + chunks) / 16 * 16;
    if (max_bn > MAX_BN) max_bn = MAX_BN;
    if (max_bn < 16) return 0;
    const int n16 = (n + 15) / 16 * 16;
    if (n16 <= max_bn) return n16;
    const int tiles = (n16 + max_bn - 1) / max_bn;
    const int bn = (n16 + tiles - 1) / tiles;
    return (bn + 15) / 16 * 16;
}

namespace {

// K blocks of the GEMM: two 32-channel taps or one 64-channel tap per block in
// conv mode, else ceil(K / 64).
int split_k_blocks(const SplitGemmParams& p) {
    if (p.conv) {
        const int taps = p.kh * p.kw, cpt = taps > 0 ? p.k / taps : 0;
        return cpt == 32 ? (taps + 1) / 2 : taps * (cpt / 64);
    }
    return (p.k + BK - 1) / BK;
}

// Accumulator buffers of (2 + chunks) BN columns each: two when both fit in
// the 512 TMEM columns of an SM, else one (the long-K tiles of
// gemm_split_tile_n, whose MMAs then wait for the previous tile's epilogue).
int split_acc_buffers(int bn, int dchunks) { return 2 * (2 + dchunks) * bn <= 512 ? 2 : 1; }

// TMEM columns of those buffers, rounded up to a power of two (0 when one
// buffer needs more than 512).
int split_tmem_cols(int bn, int dchunks) {
    int cols = 32;
    while (cols < split_acc_buffers(bn, dchunks) * (2 + dchunks) * bn) cols <<= 1;
    return cols > 512 ? 0 : cols;
}

}  // namespace

bool gemm_split_supported(const SplitGemmParams& p) {
    if (p.n <= 0 || p.k <= 0) return false;
    const int bn = gemm_split_tile_n(p.n, p.k);
    if (bn <= 0 || p.n_pad < (p.n + bn - 1) / bn * bn || p.k_pad % BK || p.k_pad < p.k) return false;
    if (p.ldc % 4 || p.coff % 4 || p.ldc < p.coff + p.n) return false;
    const int kt = split_k_blocks(p);
    if (kt <= 0 || !split_tmem_cols(bn, (kt + KCHUNK - 1) / KCHUNK)) return false;
    if (p.conv) {
        if (p.a_planes) return false;
        const int cpt = p.kh * p.kw > 0 ? p.k / (p.kh * p.kw) : 0;
        const int cin = p.cin > 0 ? p.cin : cpt;
        if (cpt <= 0 || gemm_split_conv_cpt(cin) != cpt || p.k != p.kh * p.kw * cpt || p.lda % 4 || p.lda < cin || p.gate ||
            (p.residual && (p.res_scale != 1 || p.res_gate || p.ldr < p.n)))
            return false;
        return p.n_img > 0 && p.hi > 0 && p.wi > 0 && p.ho > 0 && p.wo > 0 && (p.stride == 1 || p.stride == 2);
    }
    if (p.m <= 0 || p.k % 16) return false;
    if (!p.a_planes && (p.lda % 4 || p.lda < p.k)) return false;
    if (p.res_scale < 1 || (p.res_scale & (p.res_scale - 1))) return false;
    if ((p.gate || p.res_gate) && p.rows_per_image < 1) return false;
    return true;
}

cudaError_t launch_gemm_split(const SplitGemmParams& in, cudaStream_t stream) {
    const bool presplit = in.a_planes != nullptr;
    if (!gemm_split_supported(in) || (!presplit && !in.a) || !in.w || !in.c) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(presplit ? in.a_planes : in.a) % 16) || (reinterpret_cast<uintptr_t>(in.w) % 16))
        return cudaErrorInvalidValue;
    float* cbase = in.c + in.coff;
    if (reinterpret_cast<uintptr_t>(cbase) % 16) return cudaErrorInvalidValue;
    SplitArgs a;
    a.p = in;
    a.bn = gemm_split_tile_n(in.n, in.k);
    a.n_tiles = (in.n + a.bn - 1) / a.bn;
    a.kt = split_k_blocks(in);
    a.cpt = in.conv ? in.k / (in.kh * in.kw) : 0;
    if (in.conv) {
        a.tiles_y = (in.ho + 7) / 8;
        a.tiles_x = (in.wo + 15) / 16;
        a.m_tiles = in.n_img * a.tiles_y * a.tiles_x;
    } else {
        a.tiles_y = a.tiles_x = 0;
        a.m_tiles = (in.m + BM - 1) / BM;
    }
    a.kchunk = KCHUNK;
    a.dchunks = (a.kt + KCHUNK - 1) / KCHUNK;
    a.tmem_cols = split_tmem_cols(a.bn, a.dchunks);
    a.nacc = split_acc_buffers(a.bn, a.dchunks);
    if (!a.tmem_cols) return cudaErrorInvalidConfiguration;
    a.wait_ns = in.wait_ns ? in.wait_ns : tc::kWaitNs;
    // Shared memory: the plane ring and the staging tiles are fixed; W is
    // resident when each CTA keeps one N tile and its K blocks fit; the rest is
    // the FP32 ring, as deep as fits (deeper rings keep more loads in flight).
    const int align = 1024;
    auto up = [&](int v) { return (v + align - 1) / align * align; };
    a.w_bytes = 3 * a.bn * BK * 2;
    a.w_block = up(a.w_bytes);
    // Grid: one CTA per SM; with several N tiles, a multiple of their count
    // (dropping at most n_tiles - 1 SMs) so that each CTA keeps one N tile and
    // its W can stay in shared memory for the launch.
    const int tiles = a.m_tiles * a.n_tiles;
    const int sms = sm_count();
    int grid = tiles < sms ? tiles : sms;
    if (tiles > sms && a.n_tiles > 1 && a.n_tiles <= sms / 2) grid = sms - sms % a.n_tiles;
    const bool fixed_n = tiles <= grid || grid % a.n_tiles == 0;
    a.presplit = presplit ? 1 : 0;
    int fixed = 0;
    a.stages = 0;
    const int can_resident = (fixed_n && a.kt * a.w_block <= W_RESIDENT_MAX) ? 1 : 0;
    if (presplit) {
        // No FP32 A: the ring holds only streamed W (nothing when W is
        // resident), so the shared memory goes to a deeper plane ring.
        a.a_box_bytes = 0;
        for (int resident = can_resident; resident >= 0 && !a.stages; --resident) {
            a.w_resident = resident;
            a.w_region = resident ? a.kt * a.w_block : 0;
            a.a_stage_bytes = resident ? 0 : a.w_block;
            for (int ps = MAX_PLANE_STAGES; ps >= 2 && !a.stages; --ps)
                for (int bufs = STAGE_BUFS; bufs >= 1 && !a.stages; --bufs) {
                    const int f = align + a.w_region + ps * PLANES_STAGE + EPI_WARPS * bufs * STAGE_OUT;
                    const int avail = SMEM_MAX - 1024 - f;   // 1 KB left for the static barriers
                    if (avail < 0) continue;
                    const int st = resident ? 1 : avail / a.a_stage_bytes;
                    if (!resident && st < 2) continue;
                    a.stages = st > MAX_A ? MAX_A : st;
                    a.plane_stages = ps;
                    a.stage_bufs = bufs;
                    fixed = f;
                }
        }
        if (!a.stages) return cudaErrorInvalidConfiguration;
    } else {
        a.a_box_bytes = (in.conv || in.k > 32) ? 2 * BOX_BYTES : BOX_BYTES;
        a.plane_stages = a.kt == 1 ? SINGLE_BLOCK_PLANES : PLANE_STAGES;
        for (int resident = can_resident; resident >= 0 && a.stages < 2; --resident) {
            a.w_resident = resident;
            a.w_region = resident ? a.kt * a.w_block : 0;
            a.a_stage_bytes = a.a_box_bytes + (resident ? 0 : a.w_block);
            for (a.stage_bufs = STAGE_BUFS; a.stage_bufs >= 1; --a.stage_bufs) {
                fixed = align + a.w_region + a.plane_stages * PLANES_STAGE + EPI_WARPS * a.stage_bufs * STAGE_OUT;
                a.stages = (SMEM_MAX - 1024 - fixed) / a.a_stage_bytes;   // 1 KB left for the static barriers
                if (a.stages >= 2) break;
            }
        }
        if (a.stages > MAX_A) a.stages = MAX_A;
        if (a.stages < 2) return cudaErrorInvalidConfiguration;
    }
    const int smem = fixed + a.stages * a.a_stage_bytes;
    CUtensorMap ma, mw, mc;
    if (in.conv) {
        // The map spans the input's own channels: a tap's padding channels
        // (cpt > cin) fall outside it and load as zeros.
        if (!make_map4(&ma, in.a, (uint64_t)(in.cin > 0 ? in.cin : a.cpt), (uint64_t)in.wi, (uint64_t)in.hi, (uint64_t)in.n_img, (uint64_t)in.lda * 4, 32,
                       16 * (uint32_t)in.stride, 8 * (uint32_t)in.stride, (uint32_t)in.stride, CU_TENSOR_MAP_SWIZZLE_128B) ||
            !make_map4(&mc, cbase, (uint64_t)in.n, (uint64_t)in.wo, (uint64_t)in.ho, (uint64_t)in.n_img, (uint64_t)in.ldc * 4,
                       16, 16, 2, 1, CU_TENSOR_MAP_SWIZZLE_64B))
            return cudaErrorInvalidValue;
    } else if (!(presplit ? make_map(&ma, in.a_planes, (uint64_t)in.k_pad, (uint64_t)3 * in.m, (uint64_t)in.k_pad * 2, BK, BM,
                                     CU_TENSOR_MAP_DATA_TYPE_BFLOAT16)
                          : make_map(&ma, in.a, (uint64_t)in.k, (uint64_t)in.m, (uint64_t)in.lda * 4, 32, BM,
                                     CU_TENSOR_MAP_DATA_TYPE_FLOAT32)) ||
               !make_map(&mc, cbase, (uint64_t)in.n, (uint64_t)in.m, (uint64_t)in.ldc * 4, 16, 32,
                         CU_TENSOR_MAP_DATA_TYPE_FLOAT32, CU_TENSOR_MAP_SWIZZLE_64B)) {
        return cudaErrorInvalidValue;
    }
    if (!make_map(&mw, in.w, (uint64_t)in.k_pad, (uint64_t)3 * in.n_pad, (uint64_t)in.k_pad * 2, BK, (uint32_t)a.bn,
                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16))
        return cudaErrorInvalidValue;

    switch (in.act) {
        case ACT_NONE: return launch_act<ACT_NONE>(ma, mw, mc, a, grid, smem, stream);
        case ACT_RELU: return launch_act<ACT_RELU>(ma, mw, mc, a, grid, smem, stream);
        case ACT_SILU: return launch_act<ACT_SILU>(ma, mw, mc, a, grid, smem, stream);
        case ACT_GELU: return launch_act<ACT_GELU>(ma, mw, mc, a, grid, smem, stream);
        case ACT_HSWISH: return launch_act<ACT_HSWISH>(ma, mw, mc, a, grid, smem, stream);
        case ACT_SIGMOID: return launch_act<ACT_SIGMOID>(ma, mw, mc, a, grid, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}


namespace {

// One thread per (row, 8 columns): the gated A values split exactly as the
// converter warps split them (split8), each piece's 8 columns one 16-byte
// store into its plane.  Zeros past column k.
__global__ void __launch_bounds__(256) split_planes_kernel(SplitGemmParams p, uint4* planes) {
    const int q_row = p.k_pad / 8;
    const long long total = (long long)p.m * q_row;
    const size_t plane = (size_t)p.m * q_row;   // uint4 per plane
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / q_row), q = (int)(i - (long long)row * q_row), k0 = q * 8;
        float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (k0 < p.k) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(p.a + (size_t)row * p.lda + k0));
            const float4 v = __ldg(reinterpret_cast<const float4*>(p.a + (size_t)row * p.lda + k0 + 4));
            x[0] = u.x; x[1] = u.y; x[2] = u.z; x[3] = u.w; x[4] = v.x; x[5] = v.y; x[6] = v.z; x[7] = v.w;
            if (p.gate) {
                const float* g = p.gate + (size_t)(row / p.rows_per_image) * p.k + k0;
                const float4 g0 = __ldg(reinterpret_cast<const float4*>(g));
                const float4 g1 = __ldg(reinterpret_cast<const float4*>(g + 4));
                x[0] *= g0.x; x[1] *= g0.y; x[2] *= g0.z; x[3] *= g0.w;
                x[4] *= g1.x; x[5] *= g1.y; x[6] *= g1.z; x[7] *= g1.w;
            }
        }
        uint4 hi, mid, lo;
        split8(x, hi, mid, lo);
        planes[(size_t)i] = hi;
        planes[plane + (size_t)i] = mid;
        planes[2 * plane + (size_t)i] = lo;
    }
}

}  // namespace

cudaError_t launch_split_planes(const SplitGemmParams& p, void* planes, cudaStream_t stream) {
    if (!p.a || !planes || p.conv || p.m <= 0 || p.k <= 0 || p.k % 16 || p.lda % 4 || p.lda < p.k || p.k_pad % BK ||
        p.k_pad < p.k || (p.gate && p.rows_per_image < 1))
        return cudaErrorInvalidValue;
    if (reinterpret_cast<uintptr_t>(p.a) % 16 || reinterpret_cast<uintptr_t>(planes) % 16 ||
        (p.gate && reinterpret_cast<uintptr_t>(p.gate) % 16) || (p.gate && p.k % 4))
        return cudaErrorInvalidValue;
    const long long total = (long long)p.m * (p.k_pad / 8);
    long long blocks = (total + 255) / 256;
    if (blocks > 148LL * 32) blocks = 148LL * 32;
    split_planes_kernel<<<(unsigned)(blocks < 1 ? 1 : blocks), 256, 0, stream>>>(p, static_cast<uint4*>(planes));
    return cudaGetLastError();
}

bool gemm_split_presplit_pays(int m, int n, int k) {
    // Measured on B200: the pieces' round trip (10 bytes per element) costs
    // about as much as splitting A in shared memory for 2-3 N tiles.
    const int bn = gemm_split_tile_n(n, k);
    return m > 0 && bn > 0 && (n + bn - 1) / bn >= 4;
}

}  // namespace ppocr
