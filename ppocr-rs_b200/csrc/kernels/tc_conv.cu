// FP32-accurate tensor-core GEMM / implicit-GEMM convolution (3xTF32 on tcgen05).
//
// The FP32 mode's pointwise convs (C = act(A W^T + b) [+ residual]) and dense
// convs (stems, 3x3 / k x k, the head's 3x3 over the upsample-concat of the
// neck outputs) all run here.  FP32 operands are split into TF32 pairs,
// x = hi + lo with hi = tf32(x), lo = tf32(x - hi), and the tile product is
// A_hi W_hi + A_hi W_lo + A_lo W_hi accumulated in FP32 in TMEM: per-product
// error ~2^-22, the same class as FP32 FMA arithmetic (the dropped
// A_lo W_lo term is ~2^-22 relative).
//
// Persistent CTAs walk 128 x BN output tiles.  Roles (192 threads):
//   warp 0 / lane 0   TMA: W_hi and W_lo tiles (BN x 32 FP32, 128-byte swizzle)
//   warp 1 / lane 0   MMA: 3 x 4 tcgen05.mma.kind::tf32 (M=128, N=BN, K=8) per stage
//   warps 2-5         A producers: gather 128 rows x 32 FP32 per stage from
//                     global memory (dense rows with the SE gate, or the conv
//                     window of up to four concatenated / upsampled /
//                     max-pooled sources), split, store swizzled A_hi / A_lo;
//                     then the epilogue of the tile from TMEM.
// All waits are bounded; an expired wait records a code in g_tcc_error,
// stops the CTA's work, frees its TMEM and returns.
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

#include <cudaTypedefs.h>

namespace ppocr {

__device__ int g_tcc_error = 0;

namespace {

constexpr int BM = 128, BKF = 32, MAX_STAGES = 4, THREADS = 192;

struct TccArgs {
    TcConvParams p;
    int kt, bn, stages, tmem_cols, m_tiles, n_tiles;
};

__device__ __forceinline__ float4 f4max(float4 a, float4 b) {
    return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
}

// Four consecutive input channels (cs..cs+3 of source s) at conv input pixel (iy, ix).
__device__ __forceinline__ float4 gather4(const TcConvParams& p, int s, int cs, int img, int iy, int ix) {
    const ConvSource& src = p.conv.src[s];
    if (src.mode == SRC_NCHW_F32) {
        const float* base = static_cast<const float*>(src.ptr);
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int c = cs + q;
            v[q] = c < src.channels ? base[((size_t)(img * src.channels + c) * p.conv.hi + iy) * p.conv.wi + ix] : 0.f;
        }
        return make_float4(v[0], v[1], v[2], v[3]);
    }
    const float* base = static_cast<const float*>(src.ptr);
    const int hs = p.conv.hi / src.scale, ws = p.conv.wi / src.scale;
    if (src.mode == SRC_NHWC_MAXPOOL) {
        auto at = [&](int y, int x) {
            return *reinterpret_cast<const float4*>(base + ((size_t)(img * hs + y) * ws + x) * src.cstride + src.coff + cs);
        };
        float4 m = at(iy, ix);
        if (ix + 1 < ws) m = f4max(m, at(iy, ix + 1));
        if (iy + 1 < hs) {
            m = f4max(m, at(iy + 1, ix));
            if (ix + 1 < ws) m = f4max(m, at(iy + 1, ix + 1));
        }
        return m;
    }
    return *reinterpret_cast<const float4*>(base + ((size_t)(img * hs + iy / src.scale) * ws + ix / src.scale) * src.cstride +
                                            src.coff + cs);
}

__device__ __forceinline__ void epilogue16(const TcConvParams& p, int row, int col0, const float (&v)[16]) {
    float o[16];
    const bool full = col0 + 16 <= p.n;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        float a = v[j];
        if (p.bias && (full || col0 + j < p.n)) a += p.bias[col0 + j];
        o[j] = apply_act(a, p.act);
    }
    if (p.residual) {
        size_t rrow = (size_t)row;
        if (p.res_scale > 1) {
            const int hw = p.out_h * p.out_w;
            const int pimg = row / hw, rem = row % hw;
            const int y = rem / p.out_w, x = rem % p.out_w;
            const int rh = p.out_h / p.res_scale, rw = p.out_w / p.res_scale;
            rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
        }
        const float* r = p.residual + rrow * p.ldr + col0;
        const float* g = p.res_gate ? p.res_gate + (size_t)(row / p.rows_per_image) * p.n + col0 : nullptr;
        if (full && (p.ldr % 4) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                float4 rv = *reinterpret_cast<const float4*>(r + j);
                if (g) rv = f4_mul(rv, *reinterpret_cast<const float4*>(g + j));
                o[j] += rv.x; o[j + 1] += rv.y; o[j + 2] += rv.z; o[j + 3] += rv.w;
            }
        } else {
            for (int j = 0; j < 16 && col0 + j < p.n; ++j) o[j] += g ? r[j] * g[j] : r[j];
        }
    }
    float* c = p.c + (size_t)row * p.ldc + p.coff + col0;
    if (full && (p.ldc % 4) == 0 && (p.coff % 4) == 0) {
#pragma unroll
        for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(c + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
    } else {
        for (int j = 0; j < 16 && col0 + j < p.n; ++j) c[j] = o[j];
    }
}

__global__ void __launch_bounds__(THREADS, 1) tc_conv_kernel(const __grid_constant__ CUtensorMap tma_w, TccArgs args) {
    const TcConvParams& p = args.p;
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t a_full[MAX_STAGES], b_full[MAX_STAGES], empty[MAX_STAGES], done;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int a_bytes = BM * 128, b_bytes = args.bn * 128;
    const int stage_bytes = 2 * a_bytes + 2 * b_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = args.stages;
    const int total_tiles = args.m_tiles * args.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(&a_full[s], 128);
            tc::mbar_init(&b_full[s], 1);
            tc::mbar_init(&empty[s], 1);
        }
        tc::mbar_init(&done, 1);
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
            // W tiles by TMA: rows [n0, n0 + BN) of the hi half and of the lo half.
            int it = 0;
            for (int tile = blockIdx.x; tile < total_tiles && !abort_flag; tile += gridDim.x) {
                const int n0 = (tile % args.n_tiles) * args.bn;
                for (int kt = 0; kt < args.kt; ++kt, ++it) {
                    const int s = it % S;
                    if (it >= S && !tc::mbar_wait(&empty[s], ((it / S) + 1) & 1)) {
                        atomicExch(&g_tcc_error, 1);
                        abort_flag = 1;
                        break;
                    }
                    uint8_t* st = smem + (size_t)s * stage_bytes;
                    tc::mbar_expect_tx(&b_full[s], (uint32_t)(2 * b_bytes));
                    tc::tma_load_2d(st + 2 * a_bytes, &tma_w, &b_full[s], kt * BKF, n0);
                    tc::tma_load_2d(st + 2 * a_bytes + b_bytes, &tma_w, &b_full[s], kt * BKF, p.n_pad + n0);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_tf32(BM, args.bn);
            int it = 0;
            for (int tile = blockIdx.x; tile < total_tiles && !abort_flag; tile += gridDim.x) {
                bool ok = true;
                for (int kt = 0; kt < args.kt; ++kt, ++it) {
                    const int s = it % S;
                    const uint32_t par = (it / S) & 1;
                    if (!tc::mbar_wait(&a_full[s], par) || !tc::mbar_wait(&b_full[s], par)) {
                        atomicExch(&g_tcc_error, 2);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc::fence_after();
                    uint8_t* st = smem + (size_t)s * stage_bytes;
                    const uint64_t ahi = tc::sw128_desc(tc::smem_u32(st));
                    const uint64_t alo = tc::sw128_desc(tc::smem_u32(st + a_bytes));
                    const uint64_t bhi = tc::sw128_desc(tc::smem_u32(st + 2 * a_bytes));
                    const uint64_t blo = tc::sw128_desc(tc::smem_u32(st + 2 * a_bytes + b_bytes));
#pragma unroll
                    for (int kk = 0; kk < BKF / 8; ++kk) {   // +32 bytes per 8-element K step
                        tc::mma_tf32(tmem, ahi + 2 * kk, bhi + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
                        tc::mma_tf32(tmem, ahi + 2 * kk, blo + 2 * kk, idesc, 1u);
                        tc::mma_tf32(tmem, alo + 2 * kk, bhi + 2 * kk, idesc, 1u);
                    }
                    tc::commit(&empty[s]);
                }
                if (!ok) break;
                tc::commit(&done);
            }
        }
    } else {
        // A producers + epilogue (128 threads).
        const int pt = threadIdx.x - 64;
        const int chunk = pt & 7, rbase = pt >> 3;
        const int q = warp & 3;   // TMEM lane quarter this warp may access
        int it = 0, tile_iter = 0;
        const int hw_out = p.out_h * p.out_w;
        for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tile_iter) {
            if (abort_flag) break;
            const int m0 = (tile / args.n_tiles) * BM, n0 = (tile % args.n_tiles) * args.bn;
            // Per-row pixel coordinates of this thread's 8 rows.
            int rimg[8], ry[8], rx[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int m = m0 + rbase + 16 * i;
                if (p.mode == 1 && m < p.m) {
                    rimg[i] = m / hw_out;
                    const int rem = m - rimg[i] * hw_out;
                    ry[i] = rem / p.out_w;
                    rx[i] = rem - ry[i] * p.out_w;
                } else {
                    rimg[i] = ry[i] = rx[i] = 0;
                }
            }
            bool ok = true;
            for (int kt = 0; kt < args.kt; ++kt, ++it) {
                const int s = it % S;
                if (it >= S && !tc::mbar_wait(&empty[s], ((it / S) + 1) & 1)) {
                    atomicExch(&g_tcc_error, 3);
                    abort_flag = 1;
                    ok = false;
                    break;
                }
                uint8_t* st = smem + (size_t)s * stage_bytes;
                const int kk = kt * BKF + chunk * 4;
                // Uniform per (stage, chunk): conv tap and source of channels kk..kk+3.
                int ky = 0, kx = 0, src = 0, cs = kk;
                if (p.mode == 1 && kk < p.k) {
                    const int tap = kk / p.cin4;
                    const int ci = kk - tap * p.cin4;
                    ky = tap / p.conv.kw;
                    kx = tap - ky * p.conv.kw;
                    src = 0;
                    while (src + 1 < p.conv.nsrc && ci >= p.src_start[src + 1]) ++src;
                    cs = ci - p.src_start[src];
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int r = rbase + 16 * i;
                    const int m = m0 + r;
                    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (m < p.m && kk < p.k) {
                        if (p.mode == 0) {
                            v = *reinterpret_cast<const float4*>(p.a + (size_t)m * p.lda + kk);
                            if (p.gate) v = f4_mul(v, *reinterpret_cast<const float4*>(p.gate + (size_t)(m / p.rows_per_image) * p.k + kk));
                        } else {
                            const int iy = ry[i] * p.conv.sh - p.conv.pt + ky;
                            const int ix = rx[i] * p.conv.sw - p.conv.pl + kx;
                            if (iy >= 0 && iy < p.conv.hi && ix >= 0 && ix < p.conv.wi) v = gather4(p, src, cs, rimg[i], iy, ix);
                        }
                    }
                    const float4 hi = make_float4(tc::to_tf32(v.x), tc::to_tf32(v.y), tc::to_tf32(v.z), tc::to_tf32(v.w));
                    const float4 lo = make_float4(tc::to_tf32(v.x - hi.x), tc::to_tf32(v.y - hi.y), tc::to_tf32(v.z - hi.z),
                                                  tc::to_tf32(v.w - hi.w));
                    const uint32_t off = tc::sw128_offset(r, chunk);
                    *reinterpret_cast<float4*>(st + off) = hi;
                    *reinterpret_cast<float4*>(st + a_bytes + off) = lo;
                }
                tc::fence_proxy_async();
                tc::mbar_arrive(&a_full[s]);
            }
            if (!ok) break;
            // Epilogue: wait for the tile's MMAs, then TMEM -> registers -> global.
            bool got = tc::mbar_wait(&done, tile_iter & 1);
            got = __all_sync(0xffffffffu, got);
            if (!got) {
                if (lane == 0) atomicExch(&g_tcc_error, 4);
                abort_flag = 1;
                break;
            }
            tc::fence_after();
            const int row = m0 + q * 32 + lane;
            for (int c0 = 0; c0 < args.bn; c0 += 16) {
                uint32_t rr[16];
                tc::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, rr);
                if (row < p.m && n0 + c0 < p.n) {
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(rr[j]);
                    epilogue16(p, row, n0 + c0, v);
                }
            }
            tc::fence_before();
        }
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

int tc_conv_tile_n(int n) {
    const int n16 = (n + 15) / 16 * 16;
    const int tiles = (n16 + 255) / 256;
    int bn = (n16 + tiles - 1) / tiles;
    return (bn + 15) / 16 * 16;
}

cudaError_t launch_tc_conv(const TcConvParams& p, cudaStream_t stream) {
    if (p.k % 4 || p.k_pad % BKF || p.k_pad < p.k || p.m <= 0 || p.n <= 0) return cudaErrorInvalidValue;
    TccArgs a;
    a.p = p;
    a.bn = tc_conv_tile_n(p.n);
    if (p.n_pad % a.bn) return cudaErrorInvalidValue;
    a.kt = (p.k + BKF - 1) / BKF;
    a.n_tiles = p.n_pad / a.bn;
    a.m_tiles = (p.m + BM - 1) / BM;
    int cols = 32;
    while (cols < a.bn) cols <<= 1;
    a.tmem_cols = cols;
    const int stage_bytes = 2 * BM * 128 + 2 * a.bn * 128;
    a.stages = (200 * 1024 - 1024) / stage_bytes;
    if (a.stages > MAX_STAGES) a.stages = MAX_STAGES;
    if (a.stages < 1) return cudaErrorInvalidValue;
    const size_t smem = (size_t)a.stages * stage_bytes + 1024;

    auto fn = encode_fn();
    if (!fn) return cudaErrorInvalidValue;
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)p.k_pad, (cuuint64_t)(2 * p.n_pad)};
    cuuint64_t strides[1] = {(cuuint64_t)p.k_pad * 4};
    cuuint32_t box[2] = {BKF, (cuuint32_t)a.bn};
    cuuint32_t estr[2] = {1, 1};
    if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p.w2), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorInvalidValue;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(tc_conv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    const int tiles = a.m_tiles * a.n_tiles;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    tc_conv_kernel<<<grid, THREADS, smem, stream>>>(map, a);
    return cudaGetLastError();
}

int tc_conv_error_and_clear() {
    int h = 0;
    cudaMemcpyFromSymbol(&h, g_tcc_error, sizeof(int));
    const int zero = 0;
    cudaMemcpyToSymbol(g_tcc_error, &zero, sizeof(int));
    return h;
}

}  // namespace ppocr
