// tcgen05 BF16 GEMM for the pointwise convs and linears in BF16 mode.
//
//   C[m, n] = act(A[m, k] * W[n, k]^T + bias) (+ residual, optionally through
//   nearest upsampling of the pixel grid), FP32 accumulation in TMEM.
//
// One CTA computes a 128 x BN output tile (BN a multiple of 16, <= 256):
//   warp 0 / lane 0   TMA producer: A and W tiles (128 x 64 and BN x 64 BF16,
//                     128-byte swizzled, K-major) into a 4-stage SMEM ring;
//   warp 1 / lane 0   MMA issuer: 4 x tcgen05.mma (M=128, N=BN, K=16) per
//                     stage, accumulating in TMEM; tcgen05.commit frees the stage;
//   warps 0-3         epilogue: tcgen05.ld of the warp's 32 TMEM lanes, bias,
//                     activation, residual, BF16/FP32 store.
// Every mbarrier wait is bounded: on expiry the kernel records an error code
// in g_tc_error, skips the rest of the tile, frees its TMEM and returns.
// No cluster launch and no multicast: each CTA loads its own tiles from this
// GPU's memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"

namespace ppocr {

__device__ int g_tc_error = 0;

namespace {

constexpr int BM = 128, BK = 64, STAGES = 4, THREADS = 128;
constexpr uint32_t kWaitLimit = 1u << 22;

struct TcArgs {
    int m, n, k, kt, bn, tmem_cols;
    const float* bias;
    int act;
    const void* residual;
    int ldr, res_scale, h, w_px;
    void* c;
    int ldc, coff, c_f32;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Bounded parity wait: true when the phase completed, false on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if (i > 32) __nanosleep(128);
    }
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor: K-major tile, 128-byte swizzle, 8-row
// groups 1024 bytes apart (SBO), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

template <typename T>
__device__ __forceinline__ void epilogue16(const TcArgs& p, int row, int col0, const float (&v)[16]) {
    float o[16];
    const int img_hw = p.h * p.w_px;
    size_t rrow = (size_t)row;
    if (p.residual && p.res_scale > 1) {
        const int pimg = row / img_hw, rem = row % img_hw;
        const int y = rem / p.w_px, x = rem % p.w_px;
        const int rh = p.h / p.res_scale, rw = p.w_px / p.res_scale;
        rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
    }
    const bool full = col0 + 16 <= p.n;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int col = col0 + j;
        float a = v[j];
        if (p.bias && (full || col < p.n)) a += p.bias[col];
        o[j] = apply_act(a, p.act);
    }
    if (p.residual) {
        const T* r = static_cast<const T*>(p.residual) + rrow * p.ldr + col0;
        if (full && (p.ldr % 8) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) {
                const float4 rv = load4(r + j);
                o[j] += rv.x; o[j + 1] += rv.y; o[j + 2] += rv.z; o[j + 3] += rv.w;
            }
        } else {
            for (int j = 0; j < 16 && col0 + j < p.n; ++j) o[j] += to_f(r[j]);
        }
    }
    if (p.c_f32) {
        float* c = static_cast<float*>(p.c) + (size_t)row * p.ldc + p.coff + col0;
        if (full && (p.ldc % 4) == 0 && (p.coff % 4) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) store4(c + j, make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]));
        } else {
            for (int j = 0; j < 16 && col0 + j < p.n; ++j) c[j] = o[j];
        }
    } else {
        T* c = static_cast<T*>(p.c) + (size_t)row * p.ldc + p.coff + col0;
        if (full && (p.ldc % 8) == 0 && (p.coff % 8) == 0) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) store4(c + j, make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]));
        } else {
            for (int j = 0; j < 16 && col0 + j < p.n; ++j) c[j] = from_f<T>(o[j]);
        }
    }
}

__global__ void __launch_bounds__(THREADS, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a,
                                                             const __grid_constant__ CUtensorMap tma_b, TcArgs p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], done_bar;
    __shared__ uint32_t tmem_slot;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int a_bytes = BM * BK * 2;
    const int b_bytes = p.bn * BK * 2;
    uint8_t* sa = smem;
    uint8_t* sb = smem + STAGES * a_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * p.bn;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&done_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"((uint32_t)p.tmem_cols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = tmem_slot;
    // kind::f16 instruction descriptor: FP32 accumulate, BF16 A and B, both K-major, N >> 3, M >> 4.
    const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.bn >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

    if (warp == 0 && lane == 0) {
        for (int kt = 0; kt < p.kt; ++kt) {
            const int s = kt % STAGES;
            if (kt >= STAGES && !mbar_wait(&empty_bar[s], ((kt / STAGES) + 1) & 1)) {
                atomicExch(&g_tc_error, 1);
                break;
            }
            mbar_expect_tx(&full_bar[s], (uint32_t)(a_bytes + b_bytes));
            tma_load_2d(sa + s * a_bytes, &tma_a, &full_bar[s], kt * BK, m0);
            tma_load_2d(sb + s * b_bytes, &tma_b, &full_bar[s], kt * BK, n0);
        }
    } else if (warp == 1 && lane == 0) {
        bool ok = true;
        for (int kt = 0; kt < p.kt; ++kt) {
            const int s = kt % STAGES;
            if (!mbar_wait(&full_bar[s], (kt / STAGES) & 1)) {
                atomicExch(&g_tc_error, 2);
                ok = false;
                break;
            }
            fence_after();
            const uint64_t ad = sw128_desc(smem_u32(sa + s * a_bytes));
            const uint64_t bd = sw128_desc(smem_u32(sb + s * b_bytes));
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)   // +32 bytes per 16-element K step inside the swizzle atom
                umma_bf16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
            umma_commit(&empty_bar[s]);
        }
        if (ok) umma_commit(&done_bar);
    }
    __syncwarp();

    bool ok = mbar_wait(&done_bar, 0);
    ok = __all_sync(0xffffffffu, ok);
    fence_after();
    if (ok) {
        const int row = m0 + warp * 32 + lane;
        for (int c0 = 0; c0 < p.bn; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, r);
            if (row < p.m && n0 + c0 < p.n) {
                float v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
                epilogue16<__nv_bfloat16>(p, row, n0 + c0, v);
            }
        }
    } else if (threadIdx.x == 0) {
        atomicExch(&g_tc_error, 3);
    }
    fence_before();
    __syncthreads();
    if (warp == 0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)p.tmem_cols));
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
              uint32_t box_outer) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int pick_bn(int n_pad) {
    const int tiles = (n_pad + 255) / 256;
    int bn = (n_pad + tiles - 1) / tiles;
    return (bn + 15) / 16 * 16;
}

}  // namespace

bool gemm_tc_supported(const GemmParams& p) {
    return p.dtype == DT_BF16 && p.w_tc != nullptr && p.gate == nullptr && p.res_gate == nullptr && p.k_pad % 64 == 0 &&
           p.k_pad >= p.k && p.lda % 8 == 0 && p.k % 8 == 0 && p.m > 0 && p.n > 0 &&
           (reinterpret_cast<uintptr_t>(p.a) % 16) == 0 && (reinterpret_cast<uintptr_t>(p.w_tc) % 16) == 0;
}

cudaError_t launch_gemm_tc(const GemmParams& p, cudaStream_t stream) {
    const int n_pad16 = (p.n + 15) / 16 * 16;
    const int bn = pick_bn(n_pad16);
    CUtensorMap ma, mb;
    if (!make_map(&ma, p.a, (uint64_t)p.k, (uint64_t)p.m, (uint64_t)p.lda * 2, BK, BM)) return cudaErrorInvalidValue;
    if (!make_map(&mb, p.w_tc, (uint64_t)p.k_pad, (uint64_t)n_pad16, (uint64_t)p.k_pad * 2, BK, (uint32_t)bn))
        return cudaErrorInvalidValue;
    TcArgs a;
    a.m = p.m; a.n = p.n; a.k = p.k; a.kt = (p.k + BK - 1) / BK; a.bn = bn;
    int cols = 32;
    while (cols < bn) cols <<= 1;
    a.tmem_cols = cols;
    a.bias = p.bias; a.act = p.act;
    a.residual = p.residual; a.ldr = p.ldr; a.res_scale = p.res_scale; a.h = p.h; a.w_px = p.w_px;
    a.c = p.c; a.ldc = p.ldc; a.coff = p.coff; a.c_f32 = p.c_f32;
    const size_t smem = (size_t)STAGES * (BM * BK * 2 + bn * BK * 2) + 1024;
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    dim3 grid((p.m + BM - 1) / BM, (p.n + bn - 1) / bn);
    gemm_tc_kernel<<<grid, THREADS, smem, stream>>>(ma, mb, a);
    return cudaGetLastError();
}

int gemm_tc_error_and_clear() {
    int h = 0;
    cudaMemcpyFromSymbol(&h, g_tc_error, sizeof(int));
    const int zero = 0;
    cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int));
    return h;
}

}  // namespace ppocr
