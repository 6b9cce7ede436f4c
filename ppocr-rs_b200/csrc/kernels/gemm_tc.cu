// tcgen05 BF16 GEMM for the pointwise convs and linears in BF16 mode.
//
//   C[m, n] = act(A[m, k] * W[n, k]^T + bias) (+ residual, optionally through
//   nearest upsampling of the pixel grid), FP32 accumulation in TMEM.
//
// Persistent CTAs walk 128 x BN output tiles (BN a multiple of 64, <= 256).
// Roles (576 threads):
//   warp 0 / lane 0   TMA producer: A and W tiles (128 x 64 and BN x 64 BF16,
//                     128-byte swizzled, K-major) into a SMEM ring;
//   warp 1 / lane 0   MMA issuer: 4 x tcgen05.mma (M=128, N=BN, K=16) per
//                     stage into one of two TMEM accumulators (2 x BN columns),
//                     so the next tile's MMAs run while the previous tile's
//                     epilogue drains the other accumulator;
//   warps 2-17        epilogue: tcgen05.ld of their TMEM lane quarter (warp % 4),
//                     bias, activation, residual, then release the accumulator.
//                     Four warps share a lane quarter, each owning every fourth
//                     128-byte column group of the tile (64 BF16 / 32 FP32
//                     columns), processed 32 columns at a time to stay within
//                     the register budget of 576 threads; sixteen warps give
//                     the activation math (GELU: two MUFU ops per element)
//                     enough issue slots and latency hiding to keep up with
//                     the MMAs.  A warp packs 32 rows of a group into its own
//                     4 KB 128-byte-swizzled staging tile and one lane issues
//                     a TMA store of it, so the output leaves as whole lines.
//                     Outputs whose row pitch or base is not 16-byte aligned
//                     take a direct-store epilogue instead.
// Every mbarrier wait is bounded: on expiry the kernel records an error code
// in g_tc_error, stops, frees its TMEM and returns.  No cluster launch and no
// multicast: each CTA loads its own tiles from this GPU's memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace ppocr {

__device__ int g_tc_error = 0;

namespace {

constexpr int BM = 128, BK = 64, MAX_STAGES = 4, THREADS = 576, EPI_WARPS = 16;
constexpr int STAGE_OUT_BYTES = 32 * 128;                 // one epilogue warp's staging tile
constexpr int SMEM_LIMIT = 227 * 1024;                    // opt-in shared memory per block

struct TcArgs {
    int m, n, k, kt, bn, tmem_cols, stages, m_tiles, n_tiles;
    const float* bias;
    int act;
    const void* residual;
    int ldr, res_scale, h, w_px;
    void* c;
    int ldc, coff, c_f32;
    int tma_store;
    // Implicit-GEMM conv (conv = 1): a tile is 8 x 16 output pixels of one image,
    // a K step one (tap, 64-channel block) loaded as a strided 4D TMA box.
    int conv, tiles_y, tiles_x, cblocks, kw, stride, pt, pl;
    // Wait-expiry reporting: the code lands in *err (null: g_tc_error); each
    // pipeline wait gives up after wait_ns.  skip_load (self-test only): CTA 0
    // never issues its first stage's loads, so the waits on it run out.
    int* err;
    uint64_t wait_ns;
    int skip_load;
};

__device__ __forceinline__ void report(const TcArgs& p, int code) { atomicExch(p.err ? p.err : &g_tc_error, code); }

template <typename T, int ACT>
__device__ __forceinline__ void epilogue16(const TcArgs& p, int row, int col0, const float (&v)[16]) {
    float o[16];
    const bool full = col0 + 16 <= p.n;
    if (p.bias && full) {
        // 16 consecutive biases as four 16-byte loads (col0 is a multiple of 16).
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
            const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + col0 + j));
            o[j] = v[j] + b.x; o[j + 1] = v[j + 1] + b.y; o[j + 2] = v[j + 2] + b.z; o[j + 3] = v[j + 3] + b.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = v[j] + ((p.bias && col0 + j < p.n) ? p.bias[col0 + j] : 0.f);
    }
    apply_act_fast_array<ACT>(o);
    if (p.residual) {
        size_t rrow = (size_t)row;
        if (p.res_scale > 1) {
            const int img_hw = p.h * p.w_px;
            const int pimg = row / img_hw, rem = row % img_hw;
            const int y = rem / p.w_px, x = rem % p.w_px;
            const int rh = p.h / p.res_scale, rw = p.w_px / p.res_scale;
            rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
        }
        const T* r = static_cast<const T*>(p.residual) + rrow * p.ldr + col0;
        if (full && (p.ldr % 8) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                const float4 rv = load4(r + j);
                o[j] += rv.x; o[j + 1] += rv.y; o[j + 2] += rv.z; o[j + 3] += rv.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (col0 + j < p.n) o[j] += to_f(r[j]);
        }
    }
    if (p.c_f32) {
        float* c = static_cast<float*>(p.c) + (size_t)row * p.ldc + p.coff + col0;
        if (full && (p.ldc % 4) == 0 && (p.coff % 4) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) store4(c + j, make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]));
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (col0 + j < p.n) c[j] = o[j];
        }
    } else {
        T* c = static_cast<T*>(p.c) + (size_t)row * p.ldc + p.coff + col0;
        if (full && (p.ldc % 8) == 0 && (p.coff % 8) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) store4(c + j, make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]));
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (col0 + j < p.n) c[j] = from_f<T>(o[j]);
        }
    }
}

// One 128-byte column group (64 BF16 or 32 FP32 outputs) of one row: all its
// TMEM loads, bias loads and residual loads are issued before the first wait,
// then bias, activation and residual are applied and the row's 128-byte line
// of the warp's 128-byte-swizzled staging tile is written (the swizzle XORs
// the 16-byte chunk with row % 8, so the warp's 32 row writes are free of bank
// conflicts).  Lane 0 waits for the previous TMA store to have read the tile
// only after the math, so that wait overlaps it.
template <int ACT, bool F32>
__device__ __forceinline__ void epilogue_half(const TcArgs& p, uint32_t taddr, int row, int col0, uint8_t* line, int chunk0,
                                              int swz) {
    constexpr int HW = 32;   // columns per half
    uint32_t r[HW];
#pragma unroll
    for (int j = 0; j < HW; j += 16) tc::tmem_ld16_async(taddr + (uint32_t)j, r + j);
    const bool full = col0 + HW <= p.n;
    const bool res = p.residual != nullptr && row < p.m;
    const __nv_bfloat16* rp = nullptr;
    if (res) {
        size_t rrow = (size_t)row;
        if (p.res_scale > 1) {
            const int img_hw = p.h * p.w_px;
            const int pimg = row / img_hw, rem = row % img_hw;
            const int y = rem / p.w_px, x = rem % p.w_px;
            const int rh = p.h / p.res_scale, rw = p.w_px / p.res_scale;
            rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
        }
        rp = static_cast<const __nv_bfloat16*>(p.residual) + rrow * p.ldr + col0;
    }
    const bool res_vec = res && full && (p.ldr % 8) == 0;
    uint4 rv[HW / 8];
    if (res_vec) {
#pragma unroll
        for (int j = 0; j < HW / 8; ++j) rv[j] = __ldg(reinterpret_cast<const uint4*>(rp) + j);
    }
    tc::tmem_wait_ld_regs(r);
    float o[HW];
    if (p.bias && full) {
#pragma unroll
        for (int j = 0; j < HW; j += 4) {
            const float4 b = __ldg(reinterpret_cast<const float4*>(p.bias + col0 + j));
            o[j] = __uint_as_float(r[j]) + b.x; o[j + 1] = __uint_as_float(r[j + 1]) + b.y;
            o[j + 2] = __uint_as_float(r[j + 2]) + b.z; o[j + 3] = __uint_as_float(r[j + 3]) + b.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < HW; ++j)
            o[j] = __uint_as_float(r[j]) + ((p.bias && col0 + j < p.n) ? __ldg(p.bias + col0 + j) : 0.f);
    }
    apply_act_fast_array<ACT>(o);
    if (res_vec) {
#pragma unroll
        for (int j = 0; j < HW / 8; ++j) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&rv[j]);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float2 f = __bfloat1622float2(h[t]);
                o[8 * j + 2 * t] += f.x;
                o[8 * j + 2 * t + 1] += f.y;
            }
        }
    } else if (res) {
#pragma unroll
        for (int j = 0; j < HW; ++j)
            if (col0 + j < p.n) o[j] += __bfloat162float(rp[j]);
    }
    if constexpr (F32) {
#pragma unroll
        for (int c = 0; c < 8; ++c)
            *reinterpret_cast<float4*>(line + (((chunk0 + c) ^ swz) << 4)) = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
    } else {
        uint32_t w[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(o[2 * j], o[2 * j + 1]);
            w[j] = *reinterpret_cast<const uint32_t*>(&h);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(line + (((chunk0 + c) ^ swz) << 4)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    }
}

template <int ACT, bool F32>
__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a,
                                                             const __grid_constant__ CUtensorMap tma_b,
                                                             const __grid_constant__ CUtensorMap tma_c, TcArgs p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[MAX_STAGES], empty_bar[MAX_STAGES], acc_full[2], acc_empty[2], drain_bar;
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;
    // Up to the next 1024-byte boundary by offsetting the shared pointer itself:
    // the compiler keeps its address space, so the tile reads and writes below
    // are shared-memory instructions rather than generic ones.
    uint8_t* smem = smem_raw + ((1024u - (tc::smem_u32(smem_raw) & 1023u)) & 1023u);
    const int a_bytes = BM * BK * 2;
    const int b_bytes = p.bn * BK * 2;
    const uint64_t wait_ns = p.wait_ns;
    const int S = p.stages;
    uint8_t* sa = smem;
    uint8_t* sb = smem + S * a_bytes;
    uint8_t* sout = sb + S * b_bytes;   // 8 x 4 KB staging tiles, 1024-byte aligned
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int total = p.m_tiles * p.n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            tc::mbar_init(&full_bar[s], 1);
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
    if (warp == 0) tc::tmem_alloc(&tmem_slot, (uint32_t)p.tmem_cols);
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // last_it[s]: the last iteration whose loads were issued into stage s
            // (-1: none), so an aborting CTA can wait for its copies in flight.
            int last_it[MAX_STAGES];
            for (int s = 0; s < MAX_STAGES; ++s) last_it[s] = -1;
            int it = 0;
            for (int tile = blockIdx.x; tile < total && !abort_flag; tile += gridDim.x) {
                const int mt = tile / p.n_tiles;
                const int m0 = mt * BM, n0 = (tile % p.n_tiles) * p.bn;
                int img = 0, x0 = 0, y0 = 0;
                if (p.conv) {
                    const int per = p.tiles_y * p.tiles_x;
                    img = mt / per;
                    const int r = mt - img * per;
                    y0 = (r / p.tiles_x) * 8 * p.stride - p.pt;
                    x0 = (r % p.tiles_x) * 16 * p.stride - p.pl;
                }
                for (int kt = 0; kt < p.kt; ++kt, ++it) {
                    const int s = it % S;
                    if (it >= S && !tc::mbar_wait(&empty_bar[s], ((it / S) + 1) & 1, false, wait_ns, &abort_flag)) {
                        report(p, 1);
                        abort_flag = 1;
                        break;
                    }
                    if (p.skip_load && it == 0 && blockIdx.x == 0) continue;
                    tc::mbar_expect_tx(&full_bar[s], (uint32_t)(a_bytes + b_bytes));
                    if (p.conv) {
                        const int tap = kt / p.cblocks, cb = kt - tap * p.cblocks;
                        const int ky = tap / p.kw, kx = tap - ky * p.kw;
                        tc::tma_load_4d(sa + s * a_bytes, &tma_a, &full_bar[s], cb * BK, x0 + kx, y0 + ky, img);
                    } else {
                        tc::tma_load_2d(sa + s * a_bytes, &tma_a, &full_bar[s], kt * BK, m0);
                    }
                    tc::tma_load_2d(sb + s * b_bytes, &tma_b, &full_bar[s], kt * BK, n0);
                    last_it[s] = it;
                }
            }
            if (abort_flag) {
                // Let the copies already issued land before the CTA exits.
                for (int s = 0; s < S; ++s)
                    if (last_it[s] >= 0) tc::mbar_wait(&full_bar[s], (last_it[s] / S) & 1, false, wait_ns);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = tc::idesc_bf16(BM, p.bn);
            int it = 0, ti = 0;
            for (int tile = blockIdx.x; tile < total && !abort_flag; tile += gridDim.x, ++ti) {
                const int b = ti & 1;
                if (ti >= 2 && !tc::mbar_wait(&acc_empty[b], ((ti >> 1) + 1) & 1, false, wait_ns, &abort_flag)) {
                    report(p, 2);
                    abort_flag = 1;
                    break;
                }
                tc::fence_after();
                const uint32_t acc = tmem + (uint32_t)(b * p.bn);
                bool ok = true;
                for (int kt = 0; kt < p.kt; ++kt, ++it) {
                    const int s = it % S;
                    if (!tc::mbar_wait(&full_bar[s], (it / S) & 1, false, wait_ns, &abort_flag)) {
                        report(p, 3);
                        abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc::fence_after();
                    const uint64_t ad = tc::sw128_desc(tc::smem_u32(sa + s * a_bytes));
                    const uint64_t bd = tc::sw128_desc(tc::smem_u32(sb + s * b_bytes));
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)   // +32 bytes per 16-element K step inside the swizzle atom
                        tc::mma_bf16(acc, ad + 2 * kk, bd + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
                    tc::commit(&empty_bar[s]);
                }
                if (!ok) break;
                tc::commit(&acc_full[b]);
            }
            // Every MMA this thread issued completes before the CTA goes on to
            // free TMEM (on the normal path they already have).
            tc::commit(&drain_bar);
            tc::mbar_wait(&drain_bar, 0, false, wait_ns);
        }
    } else {
        // Epilogue warps 2..17: TMEM lane quarter q = warp % 4, column slot (warp - 2) / 4.
        const int q = warp & 3, slot = (warp - 2) >> 2;
        uint8_t* stage = sout + (warp - 2) * STAGE_OUT_BYTES;
        uint8_t* line = stage + lane * 128;
        const int swz = lane & 7;
        constexpr int GW = F32 ? 32 : 64;
        int ti = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++ti) {
            if (abort_flag) break;
            const int b = ti & 1;
            const int m0 = (tile / p.n_tiles) * BM, n0 = (tile % p.n_tiles) * p.bn;
            bool got = tc::mbar_wait(&acc_full[b], (ti >> 1) & 1, true, wait_ns, &abort_flag);
            got = __all_sync(0xffffffffu, got);
            if (!got) {
                if (lane == 0) report(p, 4);
                abort_flag = 1;
                break;
            }
            tc::fence_after();
            const int row = m0 + q * 32 + lane;
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * p.bn);
            if (p.tma_store) {
                for (int cb = slot * GW; cb < p.bn && n0 + cb < p.n; cb += 4 * GW) {
                    if (lane == 0) tc::bulk_wait_read();
                    __syncwarp();
                    for (int hf = 0; hf < GW; hf += 32)
                        epilogue_half<ACT, F32>(p, tbase + (uint32_t)(cb + hf), row, n0 + cb + hf, line, hf / (F32 ? 4 : 8), swz);
                    tc::fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        if (p.conv) {
                            // The warp's 32 rows are two 16-pixel output rows of the tile.
                            const int mt = tile / p.n_tiles, per = p.tiles_y * p.tiles_x;
                            const int img = mt / per, r = mt - img * per;
                            tc::tma_store_4d(&tma_c, stage, n0 + cb, (r % p.tiles_x) * 16, (r / p.tiles_x) * 8 + q * 2, img);
                        } else {
                            tc::tma_store_2d(&tma_c, stage, n0 + cb, m0 + q * 32);
                        }
                        tc::bulk_commit();
                    }
                }
            } else {
                const int cols = p.bn / 4;   // multiple of 16, processed 16 at a time
                const int half = slot;
                const uint32_t base = tbase + (uint32_t)(half * cols);
                for (int c0 = 0; c0 < cols; c0 += 16) {
                    uint32_t r[16];
                    tc::tmem_ld16(base + (uint32_t)c0, r);
                    const int col = n0 + half * cols + c0;
                    if (row < p.m && col < p.n) {
                        float v[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
                        epilogue16<__nv_bfloat16, ACT>(p, row, col, v);
                    }
                }
            }
            tc::fence_before();
            tc::mbar_arrive(&acc_empty[b]);
        }
        if (lane == 0) tc::bulk_wait_all();
    }
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        tc::tmem_dealloc(tmem, (uint32_t)p.tmem_cols);
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
              uint32_t box_outer, CUtensorMapDataType type = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4D NHWC map: dims (channels, width, height, images) of a view with pixel
// pitch `cstride` elements, box (box_c, box_x, box_y, 1) traversed with
// element strides (1, stride, stride, 1).
bool make_map4(CUtensorMap* map, const void* base, uint64_t channels, uint64_t w, uint64_t h, uint64_t n, uint64_t cstride,
               uint32_t box_c, uint32_t box_x, uint32_t box_y, uint32_t stride) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {channels, w, h, n};
    cuuint64_t strides[3] = {cstride * 2, w * cstride * 2, h * w * cstride * 2};
    cuuint32_t box[4] = {box_c, box_x, box_y, 1};
    cuuint32_t estr[4] = {1, stride, stride, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tile width: N split into <= 256-wide tiles of equal width, a multiple of 64
// (whole 128-byte BF16 column groups for the staged epilogue).
int pick_bn(int n) {
    const int n64 = (n + 63) / 64 * 64;
    const int tiles = (n64 + 255) / 256;
    const int bn = (n64 + tiles - 1) / tiles;
    return (bn + 63) / 64 * 64;
}

template <int ACT, bool F32>
cudaError_t launch_out(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const TcArgs& a, int grid,
                       size_t smem, cudaStream_t stream) {
    {
        cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(gemm_tc_kernel<ACT, F32>), SMEM_LIMIT - 1024);
        if (e != cudaSuccess) return e;
    }
    gemm_tc_kernel<ACT, F32><<<grid, THREADS, smem, stream>>>(ma, mb, mc, a);
    return cudaGetLastError();
}

template <int ACT>
cudaError_t launch_act(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const TcArgs& a, int grid,
                       size_t smem, cudaStream_t stream) {
    return a.c_f32 ? launch_out<ACT, true>(ma, mb, mc, a, grid, smem, stream)
                   : launch_out<ACT, false>(ma, mb, mc, a, grid, smem, stream);
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

bool gemm_tc_supported(const GemmParams& p) {
    return p.dtype == DT_BF16 && p.w_tc != nullptr && p.gate == nullptr && p.res_gate == nullptr && p.k_pad % 64 == 0 &&
           p.k_pad >= p.k && p.lda % 8 == 0 && p.k % 8 == 0 && p.m > 0 && p.n > 0 &&
           (reinterpret_cast<uintptr_t>(p.a) % 16) == 0 && (reinterpret_cast<uintptr_t>(p.w_tc) % 16) == 0;
}

cudaError_t launch_gemm_tc(const GemmParams& p, cudaStream_t stream) {
    const int bn = pick_bn(p.n);
    const int n_rows = (p.n + 15) / 16 * 16;   // rows of the packed BF16 weight
    CUtensorMap ma, mb;
    if (!make_map(&ma, p.a, (uint64_t)p.k, (uint64_t)p.m, (uint64_t)p.lda * 2, BK, BM)) return cudaErrorInvalidValue;
    if (!make_map(&mb, p.w_tc, (uint64_t)p.k_pad, (uint64_t)n_rows, (uint64_t)p.k_pad * 2, BK, (uint32_t)bn))
        return cudaErrorInvalidValue;
    TcArgs a{};
    a.m = p.m; a.n = p.n; a.k = p.k; a.kt = (p.k + BK - 1) / BK; a.bn = bn;
    int cols = 32;
    while (cols < 2 * bn) cols <<= 1;
    a.tmem_cols = cols;
    const int stage_bytes = BM * BK * 2 + bn * BK * 2;
    const int out_bytes = EPI_WARPS * STAGE_OUT_BYTES;
    a.stages = (SMEM_LIMIT - 2048 - out_bytes) / stage_bytes;
    if (a.stages > MAX_STAGES) a.stages = MAX_STAGES;
    a.m_tiles = (p.m + BM - 1) / BM;
    a.n_tiles = (p.n + bn - 1) / bn;
    a.bias = p.bias; a.act = p.act;
    a.err = p.err; a.wait_ns = p.wait_ns ? p.wait_ns : tc::kWaitNs; a.skip_load = p.skip_load;
    a.residual = p.residual; a.ldr = p.ldr; a.res_scale = p.res_scale; a.h = p.h; a.w_px = p.w_px;
    a.c = p.c; a.ldc = p.ldc; a.coff = p.coff; a.c_f32 = p.c_f32;
    // TMA store: the output base and row pitch must be 16-byte aligned.
    const size_t esize = p.c_f32 ? 4 : 2;
    char* cbase = static_cast<char*>(p.c) + (size_t)p.coff * esize;
    CUtensorMap mc;
    memset(&mc, 0, sizeof(mc));
    a.tma_store = ((reinterpret_cast<uintptr_t>(cbase) % 16) == 0 && ((size_t)p.ldc * esize) % 16 == 0 &&
                   make_map(&mc, cbase, (uint64_t)p.n, (uint64_t)p.m, (uint64_t)p.ldc * esize, p.c_f32 ? 32 : 64, 32,
                            p.c_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16))
                      ? 1 : 0;
    const size_t smem = (size_t)a.stages * stage_bytes + out_bytes + 1024;
    const int tiles = a.m_tiles * a.n_tiles;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    switch (p.act) {
        case ACT_NONE: return launch_act<ACT_NONE>(ma, mb, mc, a, grid, smem, stream);
        case ACT_RELU: return launch_act<ACT_RELU>(ma, mb, mc, a, grid, smem, stream);
        case ACT_SILU: return launch_act<ACT_SILU>(ma, mb, mc, a, grid, smem, stream);
        case ACT_GELU: return launch_act<ACT_GELU>(ma, mb, mc, a, grid, smem, stream);
        case ACT_HSWISH: return launch_act<ACT_HSWISH>(ma, mb, mc, a, grid, smem, stream);
        case ACT_SIGMOID: return launch_act<ACT_SIGMOID>(ma, mb, mc, a, grid, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}

bool conv_tc_supported(const ConvParams& p) {
    if (p.dtype != DT_BF16 || p.nsrc != 1 || p.residual) return false;
    const ConvSource& s = p.src[0];
    if (s.mode != SRC_NHWC || s.scale != 1 || s.cstride % 8 || s.coff % 8) return false;
    if (p.sh != p.sw || (p.sh != 1 && p.sh != 2)) return false;
    if (p.out_cstride % 8 || p.out_coff % 8 || p.cout < 1) return false;
    return p.n > 0 && p.ho > 0 && p.wo > 0;
}

cudaError_t launch_conv_tc(const ConvParams& p, cudaStream_t stream) {
    if (!conv_tc_supported(p) || !p.w_tc) return cudaErrorInvalidValue;
    const ConvSource& src = p.src[0];
    const int cblocks = (src.channels + BK - 1) / BK;
    if (p.tc_cin_pad != cblocks * BK) return cudaErrorInvalidValue;
    const int bn = pick_bn(p.cout);
    const int taps = p.kh * p.kw;
    const int n_rows = (p.cout + 15) / 16 * 16;
    if (p.tc_n_pad != n_rows) return cudaErrorInvalidValue;
    const int s = p.sh;
    CUtensorMap ma, mb, mc;
    memset(&mc, 0, sizeof(mc));
    const char* abase = static_cast<const char*>(src.ptr) + (size_t)src.coff * 2;
    char* cbase = static_cast<char*>(p.out) + (size_t)p.out_coff * 2;
    if ((reinterpret_cast<uintptr_t>(abase) % 16) || (reinterpret_cast<uintptr_t>(cbase) % 16)) return cudaErrorInvalidValue;
    if (!make_map4(&ma, abase, (uint64_t)src.channels, (uint64_t)p.wi, (uint64_t)p.hi, (uint64_t)p.n, (uint64_t)src.cstride, BK,
                   16 * s, 8 * s, s))
        return cudaErrorInvalidValue;
    if (!make_map(&mb, p.w_tc, (uint64_t)taps * cblocks * BK, (uint64_t)n_rows, (uint64_t)taps * cblocks * BK * 2, BK,
                  (uint32_t)bn))
        return cudaErrorInvalidValue;
    if (!make_map4(&mc, cbase, (uint64_t)p.cout, (uint64_t)p.wo, (uint64_t)p.ho, (uint64_t)p.n, (uint64_t)p.out_cstride, 64,
                   16, 2, 1))
        return cudaErrorInvalidValue;
    TcArgs a{};
    a.conv = 1;
    a.tiles_y = (p.ho + 7) / 8;
    a.tiles_x = (p.wo + 15) / 16;
    a.cblocks = cblocks;
    a.kw = p.kw;
    a.stride = s;
    a.pt = p.pt;
    a.pl = p.pl;
    a.m_tiles = p.n * a.tiles_y * a.tiles_x;
    a.m = a.m_tiles * BM;
    a.n = p.cout;
    a.k = taps * cblocks * BK;
    a.kt = taps * cblocks;
    a.bn = bn;
    int cols = 32;
    while (cols < 2 * bn) cols <<= 1;
    a.tmem_cols = cols;
    const int stage_bytes = BM * BK * 2 + bn * BK * 2;
    const int out_bytes = EPI_WARPS * STAGE_OUT_BYTES;
    a.stages = (SMEM_LIMIT - 2048 - out_bytes) / stage_bytes;
    if (a.stages > MAX_STAGES) a.stages = MAX_STAGES;
    a.n_tiles = (p.cout + bn - 1) / bn;
    a.bias = p.bias;
    a.act = p.act;
    a.c = p.out;
    a.ldc = p.out_cstride;
    a.coff = p.out_coff;
    a.tma_store = 1;
    a.err = p.err;
    a.wait_ns = p.wait_ns ? p.wait_ns : tc::kWaitNs;
    const size_t smem = (size_t)a.stages * stage_bytes + out_bytes + 1024;
    const int tiles = a.m_tiles * a.n_tiles;
    const int grid = tiles < sm_count() ? tiles : sm_count();
    switch (p.act) {
        case ACT_NONE: return launch_act<ACT_NONE>(ma, mb, mc, a, grid, smem, stream);
        case ACT_RELU: return launch_act<ACT_RELU>(ma, mb, mc, a, grid, smem, stream);
        case ACT_SILU: return launch_act<ACT_SILU>(ma, mb, mc, a, grid, smem, stream);
        case ACT_GELU: return launch_act<ACT_GELU>(ma, mb, mc, a, grid, smem, stream);
        case ACT_HSWISH: return launch_act<ACT_HSWISH>(ma, mb, mc, a, grid, smem, stream);
        case ACT_SIGMOID: return launch_act<ACT_SIGMOID>(ma, mb, mc, a, grid, smem, stream);
        default: return cudaErrorInvalidValue;
    }
}

int gemm_tc_error_and_clear() {
    int h = 0;
    cudaMemcpyFromSymbol(&h, g_tc_error, sizeof(int));
    const int zero = 0;
    cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
    return h;
}

}  // namespace ppocr
