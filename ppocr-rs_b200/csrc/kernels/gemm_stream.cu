// Streaming FP32 pointwise GEMM for the thin layers of the FP32 mode
// (K <= 128, N <= 128: the detector's 1x1 convs and the tiny recognizer's).
//
// C[m, n] = act(A[m, k] * W[k, n] + bias) (+ residual), with the optional SE
// gate on A and on the residual and the nearest-upsampled residual, exactly as
// gemm_simt.cu computes them: per output the FMAs run in k order, then the
// bias is added, then the activation, then the residual.  Only the schedule
// differs.
//
// These layers read K and write N floats per row and do 2 K N flops, so they
// are close to both the HBM and the FP32 roofline; the row-tiled kernels ran
// them latency-bound (load, barrier, compute, store per tile).  Here:
//   * W (K x BN) and the bias stay in shared memory for the whole launch;
//   * blocks are persistent and walk BM-row tiles of A, double-buffering them
//     in shared memory with 16-byte cp.async copies, so the next tile streams
//     in while the current one is multiplied;
//   * each thread owns TM x TN outputs (rows ty + i * TY, columns tx * TN + j)
//     and issues the products as packed two-lane FMAs (fma.rn.f32x2, each lane
//     rounded as fmaf), halving the arithmetic issue slots.
// The A tile rows are padded to ld = K + pad floats with ld = 4 (mod 32), so
// the up to eight distinct rows a warp reads at one k fall in distinct banks.
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int kThreads = 256;
constexpr size_t kSmemLimit = 200 * 1024;
constexpr int kMaxK = 128;

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

inline int a_ld(int k) { return k + ((4 - k) % 32 + 32) % 32; }

template <int BN, int TN, int TM>
struct StreamCfg {
    static constexpr int TX = BN / TN;          // threads along N
    static constexpr int TY = kThreads / TX;    // threads along M
    static constexpr int BM = TY * TM;          // rows per tile
    static_assert(TX * TY == kThreads && TN % 4 == 0, "tile shape");
};

template <int BN, int TN, int TM>
__global__ void __launch_bounds__(kThreads, 2) gemm_stream_kernel(GemmParams p, int ld, int tiles) {
    using G = StreamCfg<BN, TN, TM>;
    constexpr int TX = G::TX, TY = G::TY, BM = G::BM;
    extern __shared__ float4 gsm[];
    float* ws = reinterpret_cast<float*>(gsm);       // [K][BN]
    float* abuf = ws + (size_t)p.k * BN;              // [2][BM][ld]
    const int tile_floats = BM * ld;
    const int t = threadIdx.x, tx = t % TX, ty = t / TX;
    const int kq = p.k / 4;                           // 16-byte chunks per A row

    for (int i = t; i < p.k * (BN / 4); i += kThreads) {
        const int kr = i / (BN / 4), nq = (i % (BN / 4)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (nq < p.n_pad) v = *reinterpret_cast<const float4*>(p.w + (size_t)kr * p.n_pad + nq);
        *reinterpret_cast<float4*>(ws + kr * BN + nq) = v;
    }
    const int col0 = tx * TN;
    float bias[TN];
#pragma unroll
    for (int j = 0; j < TN; ++j) bias[j] = (p.bias && col0 + j < p.n) ? p.bias[col0 + j] : 0.f;

    const float* A = static_cast<const float*>(p.a);
    auto issue = [&](int tile, float* dst) {
        const int m0 = tile * BM;
        for (int i = t; i < BM * kq; i += kThreads) {
            const int r = i / kq, q = i - r * kq;
            const int row = m0 + r;
            const bool ok = row < p.m;
            cp_async16(dst + r * ld + q * 4, ok ? A + (size_t)row * p.lda + q * 4 : A, ok);
        }
        cp_async_commit();
    };
    // The SE gate scales A once per element: each thread rescales the chunks
    // it copied itself, after its own copies have landed.
    auto gate = [&](int tile, float* dst) {
        const int m0 = tile * BM;
        for (int i = t; i < BM * kq; i += kThreads) {
            const int r = i / kq, q = i - r * kq;
            const int row = m0 + r;
            if (row >= p.m) continue;
            float4* v = reinterpret_cast<float4*>(dst + r * ld + q * 4);
            *v = f4_mul(*v, *reinterpret_cast<const float4*>(p.gate + (size_t)(row / p.rows_per_image) * p.k + q * 4));
        }
    };

    int tile = blockIdx.x;
    if (tile < tiles) issue(tile, abuf);
    int parity = 0;
    const int hw = p.h * p.w_px;
    for (; tile < tiles; tile += gridDim.x, parity ^= 1) {
        const int next = tile + gridDim.x;
        if (next < tiles) issue(next, abuf + (parity ^ 1) * tile_floats);
        else cp_async_commit();
        cp_async_wait<1>();
        float* at = abuf + parity * tile_floats;
        if (p.gate) gate(tile, at);
        __syncthreads();

        float acc[TM][TN];
#pragma unroll
        for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
        const float* arow = at + ty * ld;
#pragma unroll 1
        for (int k = 0; k < p.k; k += 4) {
            float4 a[TM];
#pragma unroll
            for (int i = 0; i < TM; ++i) a[i] = *reinterpret_cast<const float4*>(arow + i * TY * ld + k);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                float b[TN];
#pragma unroll
                for (int j = 0; j < TN; j += 4) {
                    const float4 v = *reinterpret_cast<const float4*>(ws + (k + kk) * BN + col0 + j);
                    b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
                }
#pragma unroll
                for (int i = 0; i < TM; ++i) {
                    const float av = kk == 0 ? a[i].x : kk == 1 ? a[i].y : kk == 2 ? a[i].z : a[i].w;
#pragma unroll
                    for (int j = 0; j < TN; j += 2) fma2(acc[i][j], acc[i][j + 1], av, av, b[j], b[j + 1]);
                }
            }
        }

        const int m0 = tile * BM;
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int row = m0 + ty + i * TY;
            if (row >= p.m || col0 >= p.n) continue;
            float o[TN];
#pragma unroll
            for (int j = 0; j < TN; ++j) o[j] = apply_act(acc[i][j] + bias[j], p.act);
            if (p.residual) {
                size_t rrow = (size_t)row;
                if (p.res_scale > 1) {
                    const int pimg = row / hw, rem = row % hw;
                    const int y = rem / p.w_px, x = rem % p.w_px;
                    const int rh = p.h / p.res_scale, rw = p.w_px / p.res_scale;
                    rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
                }
                const float* r = static_cast<const float*>(p.residual) + rrow * p.ldr + col0;
                const float* g = p.res_gate ? p.res_gate + (size_t)(row / p.rows_per_image) * p.n + col0 : nullptr;
#pragma unroll
                for (int j = 0; j < TN; j += 4) {
                    if (col0 + j >= p.n) break;
                    if (col0 + j + 4 <= p.n && (p.ldr % 4) == 0) {
                        float4 rv = *reinterpret_cast<const float4*>(r + j);
                        if (g) rv = f4_mul(rv, *reinterpret_cast<const float4*>(g + j));
                        o[j] += rv.x; o[j + 1] += rv.y; o[j + 2] += rv.z; o[j + 3] += rv.w;
                    } else {
                        for (int jj = j; jj < j + 4 && col0 + jj < p.n; ++jj) o[jj] += g ? r[jj] * g[jj] : r[jj];
                    }
                }
            }
            float* c = static_cast<float*>(p.c) + (size_t)row * p.ldc + p.coff + col0;
#pragma unroll
            for (int j = 0; j < TN; j += 4) {
                if (col0 + j >= p.n) break;
                if (col0 + j + 4 <= p.n && (p.ldc % 4) == 0 && (p.coff % 4) == 0)
                    *reinterpret_cast<float4*>(c + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
                else
                    for (int jj = j; jj < j + 4 && col0 + jj < p.n; ++jj) c[jj] = o[jj];
            }
        }
        __syncthreads();   // the buffer is free for the copies two tiles ahead
    }
    cp_async_wait<0>();
}

template <int BN, int TN, int TM>
size_t stream_smem(int k) {
    return ((size_t)k * BN + 2 * (size_t)StreamCfg<BN, TN, TM>::BM * a_ld(k)) * sizeof(float);
}

template <int BN, int TN, int TM>
cudaError_t launch_cfg(const GemmParams& p, cudaStream_t stream) {
    using G = StreamCfg<BN, TN, TM>;
    const size_t smem = stream_smem<BN, TN, TM>(p.k);
    if (smem > kSmemLimit) return cudaErrorInvalidConfiguration;
    const long long tiles = ((long long)p.m + G::BM - 1) / G::BM;
    if (tiles > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    if (tiles == 0) return cudaSuccess;
    auto kernel = gemm_stream_kernel<BN, TN, TM>;
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
    int dev = 0, sms = 148, smem_sm = 0, reserved = 0, regs_sm = 65536, threads_sm = 2048;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    const int warp_regs = (nregs + 7) / 8 * 8 * 32;
    int per_sm = threads_sm / kThreads;
    per_sm = std::min(per_sm, regs_sm / (warp_regs * (kThreads / 32)));
    per_sm = std::min(per_sm, (int)(smem_sm / (smem + (size_t)reserved)));
    if (per_sm < 1) per_sm = 1;
    const long long cap = (long long)sms * per_sm;
    const int grid = (int)(tiles < cap ? tiles : cap);
    kernel<<<grid, kThreads, smem, stream>>>(p, a_ld(p.k), (int)tiles);
    return cudaGetLastError();
}

}  // namespace

bool gemm_stream_supported(const GemmParams& p) {
    if (p.dtype != DT_F32 || p.n > 128 || p.n < 1 || p.k < 4 || p.k > kMaxK || p.k % 4 || p.lda % 4 ||
        p.n_pad % 4 || p.n_pad < p.n || (reinterpret_cast<uintptr_t>(p.a) & 15))
        return false;
    if (p.res_gate && p.n % 4) return false;
    const size_t smem = p.n <= 16 ? stream_smem<16, 4, 4>(p.k) : p.n <= 32 ? stream_smem<32, 4, 4>(p.k)
                      : p.n <= 64 ? stream_smem<64, 8, 4>(p.k) : stream_smem<128, 8, 8>(p.k);
    return smem <= kSmemLimit;
}

cudaError_t launch_gemm_stream(const GemmParams& p, cudaStream_t stream) {
    if (!gemm_stream_supported(p)) return cudaErrorInvalidValue;
    if (p.n <= 16) return launch_cfg<16, 4, 4>(p, stream);
    if (p.n <= 32) return launch_cfg<32, 4, 4>(p, stream);
    if (p.n <= 64) return launch_cfg<64, 8, 4>(p, stream);
    return launch_cfg<128, 8, 8>(p, stream);
}

}  // namespace ppocr
