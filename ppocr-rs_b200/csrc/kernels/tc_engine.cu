// Tensor-core GEMM / implicit-GEMM convolution engine (tcgen05, BF16 operands).
//
//   C[m, n] = act(A[m, k] W[n, k]^T + bias) (+ residual), FP32 accumulation in TMEM,
//   A either dense rows (pointwise convs, with the SE gate) or the window of a
//   dense conv gathered from up to four concatenated / nearest-upsampled /
//   2x2-max-pooled NHWC sources or the NCHW F32 image.
//
// Two operand modes:
//   planes = 1   BF16 activations and weights, one MMA per K step (BF16 mode);
//   planes = 3   FP32 activations and weights split into three BF16 pieces,
//                x = x0 + x1 + x2 with x0 = bf16(x), x1 = bf16(x - x0),
//                x2 = bf16(x - x0 - x1) (24 significand bits, the FP32 value
//                for normal ranges), and the six products with i + j <= 2
//                accumulated: the dropped x1 w2 + x2 w1 + x2 w2 are ~2^-24
//                relative, so each product carries FP32-class error.
//
// Persistent CTAs walk 128 x BN output tiles.  Roles (320 threads):
//   warp 0 / lane 0   TMA: the W planes (BN x 64 BF16, 128-byte swizzle);
//   warp 1 / lane 0   MMA: planes^2-ish products x 4 K steps per stage into one
//                     of two TMEM accumulators;
//   warps 2-5         A producers: gather 128 rows x 64 K elements per stage
//                     (8 threads per row, 16-byte loads), split (planes = 3),
//                     store swizzled BF16 planes;
//   warps 6-9         epilogue: TMEM lane quarter warp % 4, bias, activation,
//                     residual, packed into a 128-byte-swizzled staging tile
//                     and written by TMA stores.
// Every mbarrier wait is bounded: on expiry the kernel records a code in
// g_tce_error, stops, frees its TMEM and returns.  No clusters, no multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace ppocr {

__device__ int g_tce_error = 0;

namespace {

constexpr int BM = 128, BK = 64, MAX_STAGES = 4, THREADS = 320;
constexpr int STAGE_OUT_BYTES = 32 * 128;
constexpr int EPI_WARPS = 4;
constexpr int SMEM_LIMIT = 227 * 1024;

struct EngArgs {
    TcEngineParams p;
    int kt, bn, stages, tmem_cols, m_tiles, n_tiles, tma_store;
    uint64_t wait_ns;
};

// Wait-expiry code into the caller's flag (null: g_tce_error).
__device__ __forceinline__ void report(const TcEngineParams& p, int code) { atomicExch(p.err ? p.err : &g_tce_error, code); }

// 8 BF16 / 4 FP32 consecutive elements as floats.
__device__ __forceinline__ void load8(const __nv_bfloat16* src, float (&v)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const float2 f = __bfloat1622float2(h[t]);
        v[2 * t] = f.x;
        v[2 * t + 1] = f.y;
    }
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Conv source pixel (iy, ix) of the logical (upsampled) input, CH consecutive
// channels starting at view channel cs of source s, as floats.
template <int CH>
__device__ __forceinline__ void gather(const TcEngineParams& p, int s, int cs, int img, int iy, int ix, float (&v)[CH]) {
    const ConvSource& src = p.conv.src[s];
    if (src.mode == SRC_NCHW_F32) {
        const float* base = static_cast<const float*>(src.ptr);
#pragma unroll
        for (int q = 0; q < CH; ++q) {
            const int c = cs + q;
            v[q] = c < src.channels ? base[((size_t)(img * src.channels + c) * p.conv.hi + iy) * p.conv.wi + ix] : 0.f;
        }
        return;
    }
    const int sh = p.conv.shift[s];
    const int hs = p.conv.hi >> sh, ws = p.conv.wi >> sh;
    const int sy = iy >> sh, sx = ix >> sh;
    const size_t off = ((size_t)(img * hs + sy) * ws + sx) * src.cstride + src.coff + cs;
    if constexpr (CH == 8) {
        const __nv_bfloat16* b = static_cast<const __nv_bfloat16*>(src.ptr);
        float t[8];
        load8(b + off, t);
        if (src.mode == SRC_NHWC_MAXPOOL) {
            // 2x2 window anchored at the pixel; positions past the bottom / right
            // edge are padding and never win (pads [0, 0, 1, 1]).
            float u[8];
            if (sx + 1 < ws) {
                load8(b + off + src.cstride, u);
#pragma unroll
                for (int q = 0; q < 8; ++q) t[q] = fmaxf(t[q], u[q]);
            }
            if (sy + 1 < hs) {
                load8(b + off + (size_t)ws * src.cstride, u);
#pragma unroll
                for (int q = 0; q < 8; ++q) t[q] = fmaxf(t[q], u[q]);
                if (sx + 1 < ws) {
                    load8(b + off + (size_t)(ws + 1) * src.cstride, u);
#pragma unroll
                    for (int q = 0; q < 8; ++q) t[q] = fmaxf(t[q], u[q]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < CH; ++q) v[q] = t[q % 8];
    } else {
        const float* b = static_cast<const float*>(src.ptr);
        float4 t = *reinterpret_cast<const float4*>(b + off);
        if (src.mode == SRC_NHWC_MAXPOOL) {
            if (sx + 1 < ws) t = f4_max(t, *reinterpret_cast<const float4*>(b + off + src.cstride));
            if (sy + 1 < hs) {
                t = f4_max(t, *reinterpret_cast<const float4*>(b + off + (size_t)ws * src.cstride));
                if (sx + 1 < ws) t = f4_max(t, *reinterpret_cast<const float4*>(b + off + (size_t)(ws + 1) * src.cstride));
            }
        }
        const float f[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
        for (int q = 0; q < CH; ++q) v[q] = f[q % 4];
    }
}

// One 128-byte column group of one row through bias / activation / residual
// into the warp's swizzled staging line (see gemm_tc.cu's epilogue).
template <bool F32>
__device__ __forceinline__ void epilogue_group(const TcEngineParams& p, uint32_t taddr, int row, int col0, uint8_t* stage,
                                               int lane) {
    constexpr int GW = F32 ? 32 : 64;
    uint32_t r[GW];
#pragma unroll
    for (int j = 0; j < GW; j += 16) tc::tmem_ld16_async(taddr + (uint32_t)j, r + j);
    const bool full = col0 + GW <= p.n;
    const bool res = p.residual != nullptr && row < p.m;
    size_t rrow = (size_t)row;
    if (res && p.res_scale > 1) {
        const int img_hw = p.out_h * p.out_w;
        const int pimg = row / img_hw, rem = row % img_hw;
        const int y = rem / p.out_w, x = rem % p.out_w;
        const int rh = p.out_h / p.res_scale, rw = p.out_w / p.res_scale;
        rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
    }
    tc::tmem_wait_ld_regs(r);
    float o[GW];
#pragma unroll
    for (int j = 0; j < GW; ++j) {
        const float b = (p.bias && col0 + j < p.n) ? __ldg(p.bias + col0 + j) : 0.f;
        o[j] = apply_act(__uint_as_float(r[j]) + b, p.act);
    }
    if (res) {
        if constexpr (F32) {
            const float* rp = static_cast<const float*>(p.residual) + rrow * p.ldr + col0;
            if (full && (p.ldr % 4) == 0) {
#pragma unroll
                for (int j = 0; j < GW; j += 4) {
                    const float4 v = __ldg(reinterpret_cast<const float4*>(rp + j));
                    o[j] += v.x; o[j + 1] += v.y; o[j + 2] += v.z; o[j + 3] += v.w;
                }
            } else {
#pragma unroll
                for (int j = 0; j < GW; ++j)
                    if (col0 + j < p.n) o[j] += rp[j];
            }
        } else {
            const __nv_bfloat16* rp = static_cast<const __nv_bfloat16*>(p.residual) + rrow * p.ldr + col0;
            if (full && (p.ldr % 8) == 0) {
#pragma unroll
                for (int j = 0; j < GW; j += 8) {
                    float t[8];
                    load8(rp + j, t);
#pragma unroll
                    for (int q = 0; q < 8; ++q) o[j + q] += t[q];
                }
            } else {
#pragma unroll
                for (int j = 0; j < GW; ++j)
                    if (col0 + j < p.n) o[j] += __bfloat162float(rp[j]);
            }
        }
    }
    uint32_t w[32];
    if constexpr (F32) {
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(o[j]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = pack_bf16(o[2 * j], o[2 * j + 1]);
    }
    if (lane == 0) tc::bulk_wait_read();
    __syncwarp();
    uint8_t* line = stage + lane * 128;
    const int swz = lane & 7;
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(line + ((c ^ swz) << 4)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
}

// Direct stores for outputs whose base or pitch is not 16-byte aligned.
template <bool F32>
__device__ __forceinline__ void epilogue_direct(const TcEngineParams& p, uint32_t taddr, int row, int col0) {
    uint32_t r[16];
    tc::tmem_ld16(taddr, r);
    if (row >= p.m) return;
    for (int j = 0; j < 16 && col0 + j < p.n; ++j) {
        float o = __uint_as_float(r[j]) + (p.bias ? p.bias[col0 + j] : 0.f);
        o = apply_act(o, p.act);
        if (p.residual) {
            size_t rrow = (size_t)row;
            if (p.res_scale > 1) {
                const int img_hw = p.out_h * p.out_w;
                const int pimg = row / img_hw, rem = row % img_hw;
                const int y = rem / p.out_w, x = rem % p.out_w;
                const int rh = p.out_h / p.res_scale, rw = p.out_w / p.res_scale;
                rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
            }
            o += F32 ? static_cast<const float*>(p.residual)[rrow * p.ldr + col0 + j]
                     : __bfloat162float(static_cast<const __nv_bfloat16*>(p.residual)[rrow * p.ldr + col0 + j]);
        }
        const size_t at = (size_t)row * p.ldc + p.coff + col0 + j;
        if (F32) static_cast<float*>(p.c)[at] = o;
        else static_cast<__nv_bfloat16*>(p.c)[at] = __float2bfloat16_rn(o);
    }
}

template <int PLANES>
__global__ void __launch_bounds__(THREADS, 1) tc_engine_kernel(const __grid_constant__ CUtensorMap tma_w,
                                                               const __grid_constant__ CUtensorMap tma_c, EngArgs args) {
    constexpr bool F32 = PLANES == 3;
    constexpr int CH = F32 ? 4 : 8;           // K elements per 16-byte A load
    constexpr int CPT = (BK / CH) / 8;        // A chunks per thread per row (8 threads per row)
    const TcEngineParams& p = args.p;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t w_full[MAX_STAGES], a_full[MAX_STAGES], empty_bar[MAX_STAGES], acc_full[2],
        acc_empty[2], drain_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    // Up to the next 1024-byte boundary by offsetting the shared pointer itself:
    // the compiler keeps its address space, so the tile reads and writes below
    // are shared-memory instructions rather than generic ones.
    uint8_t* smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
    const int a_bytes = BM * BK * 2;          // one A plane per stage
    const int b_bytes = args.bn * BK * 2;     // one W plane per stage
    const int stage_bytes = PLANES * (a_bytes + b_bytes);
    const int S = args.stages;
    uint8_t* sout = smem + (size_t)S * stage_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = args.m_tiles * args.n_tiles;
    const uint64_t wait_ns = args.wait_ns;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(&w_full[s], 1);
            tc::mbar_init(&a_full[s], 128);
            tc::mbar_init(&empty_bar[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            tc::mbar_init(&acc_full[b], 1);
            tc::mbar_init(&acc_empty[b], EPI_WARPS * 32);
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
            // last_it[s]: the last iteration whose W loads went into stage s (-1:
            // none), so an aborting CTA can wait for its copies in flight.
            int last_it[MAX_STAGES];
            for (int s = 0; s < MAX_STAGES; ++s) last_it[s] = -1;
            int it = 0;
            for (int tile = blockIdx.x; tile < total && !abort_flag; tile += gridDim.x) {
                const int n0 = (tile % args.n_tiles) * args.bn;
                for (int kt = 0; kt < args.kt; ++kt, ++it) {
                    const int s = it % S;
                    if (it >= S && !tc::mbar_wait(&empty_bar[s], ((it / S) + 1) & 1, false, wait_ns, &abort_flag)) {
                        report(p, 1);
                        abort_flag = 1;
                        break;
                    }
                    if (p.skip_load && it == 0 && blockIdx.x == 0) continue;
                    uint8_t* st = smem + (size_t)s * stage_bytes + PLANES * a_bytes;
                    tc::mbar_expect_tx(&w_full[s], (uint32_t)(PLANES * b_bytes));
#pragma unroll
                    for (int j = 0; j < PLANES; ++j)
                        tc::tma_load_2d(st + j * b_bytes, &tma_w, &w_full[s], kt * BK, j * p.n_pad + n0);
                    last_it[s] = it;
                }
            }
            if (abort_flag) {
                for (int s = 0; s < S; ++s)
                    if (last_it[s] >= 0) tc::mbar_wait(&w_full[s], (last_it[s] / S) & 1, false, wait_ns);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16(BM, args.bn);
            int it = 0, ti = 0;
            for (int tile = blockIdx.x; tile < total && !abort_flag; tile += gridDim.x, ++ti) {
                const int b = ti & 1;
                if (ti >= 2 && !tc::mbar_wait(&acc_empty[b], ((ti >> 1) + 1) & 1, false, wait_ns, &abort_flag)) {
                    report(p, 2);
                    abort_flag = 1;
                    break;
                }
                tc::fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * args.bn);
                bool ok = true;
                for (int kt = 0; kt < args.kt; ++kt, ++it) {
                    const int s = it % S;
                    const uint32_t par = (it / S) & 1;
                    if (!tc::mbar_wait(&a_full[s], par, false, wait_ns, &abort_flag) ||
                        !tc::mbar_wait(&w_full[s], par, false, wait_ns, &abort_flag)) {
                        report(p, 3);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc::fence_after();
                    uint8_t* st = smem + (size_t)s * stage_bytes;
                    const uint64_t ad = tc::sw128_desc(tc::smem_u32(st));
                    const uint64_t bd = tc::sw128_desc(tc::smem_u32(st + PLANES * a_bytes));
                    const uint64_t a_step = (uint64_t)(a_bytes >> 4), b_step = (uint64_t)(b_bytes >> 4);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {   // +32 bytes per 16-element K step
                        if constexpr (PLANES == 1) {
                            tc::mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
                        } else {
                            // Smallest products first: (2,0) (1,1) (0,2) (1,0) (0,1) (0,0).
                            const int ia[6] = {2, 1, 0, 1, 0, 0}, jw[6] = {0, 1, 2, 0, 1, 0};
#pragma unroll
                            for (int t = 0; t < 6; ++t)
                                tc::mma_bf16(acc, ad + ia[t] * a_step + 2 * kk, bd + jw[t] * b_step + 2 * kk, idesc,
                                             ((kt | kk) != 0 || t != 0) ? 1u : 0u);
                        }
                    }
                    tc::commit(&empty_bar[s]);
                }
                if (!ok) break;
                tc::commit(&acc_full[b]);
            }
            // Every MMA this thread issued completes before TMEM is freed.
            tc::commit(&drain_bar);
            tc::mbar_wait(&drain_bar, 0, false, wait_ns);
        }
    } else if (warp < 6) {
        // A producers: thread pt owns rows rb + 16 i (i < 8) and chunk(s) ch + 8 j (j < CPT).
        const int pt = threadIdx.x - 64;
        const int ch = pt & 7, rb = pt >> 3;
        const int hw_out = p.conv.ho * p.conv.wo;
        int it = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
            if (abort_flag) break;
            const int m0 = (tile / args.n_tiles) * BM;
            int rimg[8], ry[8], rx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int m = m0 + rb + 16 * i;
                rimg[i] = -1;
                ry[i] = rx[i] = 0;
                if (m < p.m) {
                    if (p.mode == 1) {
                        rimg[i] = m / hw_out;
                        const int rem = m - rimg[i] * hw_out;
                        const int oy = rem / p.conv.wo;
                        ry[i] = oy * p.conv.sh - p.conv.pt;
                        rx[i] = (rem - oy * p.conv.wo) * p.conv.sw - p.conv.pl;
                    } else {
                        rimg[i] = 0;
                    }
                }
            }
            bool ok = true;
            for (int kt = 0; kt < args.kt; ++kt, ++it) {
                const int s = it % S;
                if (it >= S && !tc::mbar_wait(&empty_bar[s], ((it / S) + 1) & 1, true, wait_ns, &abort_flag)) {
                    report(p, 4);
                    abort_flag = 1;
                    ok = false;
                    break;
                }
                uint8_t* st = smem + (size_t)s * stage_bytes;
#pragma unroll
                for (int j = 0; j < CPT; ++j) {
                    const int cidx = ch + 8 * j;                 // chunk within the 64-element K block
                    const int k0 = kt * BK + cidx * CH;
                    // Conv: tap and source channel of this chunk (uniform over the rows).
                    int ky = 0, kx = 0, src = 0, cs = k0;
                    const bool kin = k0 < p.k;
                    if (p.mode == 1 && kin) {
                        const int tap = k0 / p.conv.cin;
                        const int ci = k0 - tap * p.conv.cin;
                        ky = tap / p.conv.kw;
                        kx = tap - ky * p.conv.kw;
                        cs = ci;
                        while (src + 1 < p.conv.nsrc && cs >= p.conv.src[src].channels) { cs -= p.conv.src[src].channels; ++src; }
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const int r = rb + 16 * i;
                        float v[CH];
#pragma unroll
                        for (int q = 0; q < CH; ++q) v[q] = 0.f;
                        if (kin && rimg[i] >= 0) {
                            const int m = m0 + r;
                            if (p.mode == 0) {
                                if constexpr (F32) {
                                    const float4 t = *reinterpret_cast<const float4*>(static_cast<const float*>(p.a) + (size_t)m * p.lda + k0);
                                    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
                                } else {
                                    float t[8];
                                    load8(static_cast<const __nv_bfloat16*>(p.a) + (size_t)m * p.lda + k0, t);
#pragma unroll
                                    for (int q = 0; q < CH; ++q) v[q] = t[q % 8];
                                }
                                if (p.gate) {
                                    const float* g = p.gate + (size_t)(m / p.rows_per_image) * p.k + k0;
#pragma unroll
                                    for (int q = 0; q < CH; ++q) v[q] *= g[q];
                                }
                            } else {
                                const int iy = ry[i] + ky, ix = rx[i] + kx;
                                if (iy >= 0 && iy < p.conv.hi && ix >= 0 && ix < p.conv.wi) gather<CH>(p, src, cs, rimg[i], iy, ix, v);
                            }
                        }
                        if constexpr (PLANES == 1) {
                            const uint4 u = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]),
                                                       pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
                            *reinterpret_cast<uint4*>(st + tc::sw128_offset(r, cidx)) = u;
                        } else {
                            // Three BF16 pieces per value, 4 values = 8 bytes per plane.
                            uint32_t pk[3][2];
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const float x0 = v[2 * h], y0 = v[2 * h + 1];
                                const float xa = __bfloat162float(__float2bfloat16_rn(x0));
                                const float ya = __bfloat162float(__float2bfloat16_rn(y0));
                                const float xr = x0 - xa, yr = y0 - ya;
                                const float xb = __bfloat162float(__float2bfloat16_rn(xr));
                                const float yb = __bfloat162float(__float2bfloat16_rn(yr));
                                pk[0][h] = pack_bf16(xa, ya);
                                pk[1][h] = pack_bf16(xb, yb);
                                pk[2][h] = pack_bf16(xr - xb, yr - yb);
                            }
                            const uint32_t off = (uint32_t)(r * 128 + ((((cidx >> 1) ^ (r & 7))) << 4) + (cidx & 1) * 8);
#pragma unroll
                            for (int pl = 0; pl < 3; ++pl)
                                *reinterpret_cast<uint2*>(st + pl * a_bytes + off) = make_uint2(pk[pl][0], pk[pl][1]);
                        }
                    }
                }
                tc::fence_proxy_async();
                tc::mbar_arrive(&a_full[s]);
            }
            if (!ok) break;
        }
    } else {
        // Epilogue warps 6-9: TMEM lane quarter warp % 4, every column group of the tile.
        const int q = warp & 3;
        uint8_t* stage = sout + (warp - 6) * STAGE_OUT_BYTES;
        constexpr int GW = F32 ? 32 : 64;
        int ti = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
            if (abort_flag) break;
            const int b = ti & 1;
            const int m0 = (tile / args.n_tiles) * BM, n0 = (tile % args.n_tiles) * args.bn;
            bool got = tc::mbar_wait(&acc_full[b], (ti >> 1) & 1, true, wait_ns, &abort_flag);
            got = __all_sync(0xffffffffu, got);
            if (!got) {
                if (lane == 0) report(p, 5);
                abort_flag = 1;
                break;
            }
            tc::fence_after();
            const int row = m0 + q * 32 + lane;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * args.bn);
            if (args.tma_store) {
                for (int cb = 0; cb < args.bn && n0 + cb < p.n; cb += GW) {
                    epilogue_group<F32>(p, tbase + (uint32_t)cb, row, n0 + cb, stage, lane);
                    tc::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tc::tma_store_2d(&tma_c, stage, n0 + cb, m0 + q * 32);
                        tc::bulk_commit();
                    }
                }
            } else {
                for (int c0 = 0; c0 < args.bn; c0 += 16) epilogue_direct<F32>(p, tbase + (uint32_t)c0, row, n0 + c0);
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
              uint32_t box_outer, CUtensorMapDataType type) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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

int tc_engine_tile_n(int n, int planes) {
    // One N tile when it fits (any multiple of 16); otherwise equal tiles that
    // are whole 128-byte output groups, so no TMA store box reaches the next tile.
    const int cap = planes == 3 ? 128 : 256;
    const int n16 = (n + 15) / 16 * 16;
    if (n16 <= cap) return n16;
    const int gw = planes == 3 ? 32 : 64;
    const int tiles = (n16 + cap - 1) / cap;
    const int bn = (n16 + tiles - 1) / tiles;
    return (bn + gw - 1) / gw * gw;
}

bool tc_engine_supported(const TcEngineParams& p) {
    if (p.planes != 1 && p.planes != 3) return false;
    if (p.m <= 0 || p.n <= 0 || p.k <= 0 || p.k_pad % BK || p.k_pad < p.k || !p.w) return false;
    const int ch = p.planes == 1 ? 8 : 4;
    if (p.mode == 0) return p.k % ch == 0 && p.lda % ch == 0;
    if (p.conv.cin % ch || p.conv.nsrc < 1 || p.conv.nsrc > 4) return false;
    for (int s = 0; s < p.conv.nsrc; ++s) {
        const ConvSource& src = p.conv.src[s];
        if (src.mode == SRC_NCHW_F32) {
            if (p.conv.nsrc != 1) return false;
            continue;
        }
        if (src.channels % ch || src.cstride % ch || src.coff % ch) return false;
        if (src.scale < 1 || (src.scale & (src.scale - 1)) || p.conv.hi % src.scale || p.conv.wi % src.scale) return false;
        if (src.mode == SRC_NHWC_MAXPOOL && src.scale != 1) return false;
    }
    return true;
}

cudaError_t launch_tc_engine(const TcEngineParams& in, cudaStream_t stream) {
    if (!tc_engine_supported(in)) return cudaErrorInvalidValue;
    EngArgs a;
    a.p = in;
    for (int s = 0; s < a.p.conv.nsrc; ++s) {
        a.p.conv.shift[s] = 0;
        while ((1 << a.p.conv.shift[s]) < a.p.conv.src[s].scale) ++a.p.conv.shift[s];
    }
    const int planes = in.planes;
    a.bn = tc_engine_tile_n(in.n, planes);
    a.n_tiles = (in.n + a.bn - 1) / a.bn;
    if (a.n_tiles * a.bn > in.n_pad) return cudaErrorInvalidValue;
    a.m_tiles = (in.m + BM - 1) / BM;
    a.kt = in.k_pad / BK;
    // Two accumulators of bn columns; an epilogue group reads up to GW columns
    // from the second one's start, so the allocation covers bn + GW as well.
    const int gw = planes == 3 ? 32 : 64;
    int cols = 32;
    while (cols < 2 * a.bn || cols < a.bn + gw) cols <<= 1;
    if (cols > 512) return cudaErrorInvalidConfiguration;
    a.tmem_cols = cols;
    a.wait_ns = in.wait_ns ? in.wait_ns : tc::kWaitNs;
    const int stage_bytes = planes * (BM * BK * 2 + a.bn * BK * 2);
    const int out_bytes = EPI_WARPS * STAGE_OUT_BYTES;
    a.stages = (SMEM_LIMIT - 2048 - out_bytes) / stage_bytes;
    if (a.stages > MAX_STAGES) a.stages = MAX_STAGES;
    if (a.stages < 2) return cudaErrorInvalidConfiguration;
    const size_t smem = (size_t)a.stages * stage_bytes + out_bytes + 1024;

    CUtensorMap mw, mc;
    std::memset(&mc, 0, sizeof(mc));
    if (!make_map(&mw, in.w, (uint64_t)in.k_pad, (uint64_t)planes * in.n_pad, (uint64_t)in.k_pad * 2, BK, (uint32_t)a.bn,
                  CU_TENSOR_MAP_DATA_TYPE_BFLOAT16))
        return cudaErrorInvalidValue;
    const size_t esize = planes == 3 ? 4 : 2;
    char* cbase = static_cast<char*>(in.c) + (size_t)in.coff * esize;
    a.tma_store = ((reinterpret_cast<uintptr_t>(cbase) % 16) == 0 && ((size_t)in.ldc * esize) % 16 == 0 &&
                   make_map(&mc, cbase, (uint64_t)in.n, (uint64_t)in.m, (uint64_t)in.ldc * esize, planes == 3 ? 32 : 64, 32,
                            planes == 3 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16))
                      ? 1 : 0;
    const int tiles = a.m_tiles * a.n_tiles;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    if (planes == 1) {
        {
            cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(tc_engine_kernel<1>), SMEM_LIMIT - 1024);
            if (e != cudaSuccess) return e;
        }
        tc_engine_kernel<1><<<grid, THREADS, smem, stream>>>(mw, mc, a);
    } else {
        {
            cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(tc_engine_kernel<3>), SMEM_LIMIT - 1024);
            if (e != cudaSuccess) return e;
        }
        tc_engine_kernel<3><<<grid, THREADS, smem, stream>>>(mw, mc, a);
    }
    return cudaGetLastError();
}

int tc_engine_error_and_clear() {
    int h = 0;
    cudaMemcpyFromSymbol(&h, g_tce_error, sizeof(int));
    const int zero = 0;
    cudaMemcpyToSymbol(g_tce_error, &zero, sizeof(int));
    return h;
}

}  // namespace ppocr
