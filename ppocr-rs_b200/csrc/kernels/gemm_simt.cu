// FP32 pointwise GEMM on the CUDA cores (the FP32 mode's 1x1 convs and linears).
//
// C[m, n] = act(A[m, k] * W[k, n] + bias) (+ residual), with the optional SE
// gate on A and on the residual, and a nearest-upsampled residual for the
// medium neck's top-down adds (src/cpu/model.rs:1022-1066).  Exact FP32
// products and sums (FMA), as the reference's packed CPU GEMMs compute them;
// only the summation order differs.
//
// Register-tiled: 256 threads compute a BM x BN tile, each thread TM x TN = 8 x 4
// outputs, K staged through shared memory 16 at a time (A transposed so a
// thread's 8 rows are one 32-byte shared load).  The tile shape follows N:
// 128 x 64 for wide outputs, 256 x 32 and 512 x 16 for the thin pointwise
// layers of the detector, so no thread computes padding columns.
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int BK = 16, TM = 8, TN = 4, THREADS = 256;

template <typename T>
__device__ __forceinline__ float load1(const T* p) { return to_f(*p); }

template <typename T, int BM, int BN>
__global__ void __launch_bounds__(THREADS) gemm_simt_kernel(GemmParams p) {
    static_assert((BM / TM) * (BN / TN) == THREADS, "tile shape");
    constexpr int TX = BN / TN;   // threads along N
    __shared__ __align__(16) float As[BK][BM];
    __shared__ __align__(16) float Bs[BK][BN];
    const int t = threadIdx.x;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int tx = t % TX, ty = t / TX;
    const T* A = static_cast<const T*>(p.a);
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

    // A tile: BM rows x BK columns = BM * 4 float4; each thread loads A_LOADS of them.
    constexpr int A_LOADS = BM * (BK / 4) / THREADS;
    constexpr int B_LOADS = BK * (BN / 4) / THREADS;   // may be 0 for BN < 64 -> handled below
    for (int k0 = 0; k0 < p.k; k0 += BK) {
#pragma unroll
        for (int l = 0; l < A_LOADS; ++l) {
            const int idx = t + l * THREADS;
            const int r = idx % BM, kq = idx / BM;   // consecutive threads -> consecutive rows
            const int row = m0 + r, kk = k0 + kq * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (row < p.m && kk < p.k) {
                v = load4(A + (size_t)row * p.lda + kk);
                if (p.gate) v = f4_mul(v, *reinterpret_cast<const float4*>(p.gate + (size_t)(row / p.rows_per_image) * p.k + kk));
            }
            As[kq * 4 + 0][r] = v.x;
            As[kq * 4 + 1][r] = v.y;
            As[kq * 4 + 2][r] = v.z;
            As[kq * 4 + 3][r] = v.w;
        }
        if (B_LOADS >= 1) {
#pragma unroll
            for (int l = 0; l < (B_LOADS >= 1 ? B_LOADS : 1); ++l) {
                const int idx = t + l * THREADS;
                const int kr = idx / (BN / 4), nq = (idx % (BN / 4)) * 4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (k0 + kr < p.k && n0 + nq < p.n_pad)
                    v = *reinterpret_cast<const float4*>(p.w + (size_t)(k0 + kr) * p.n_pad + n0 + nq);
                *reinterpret_cast<float4*>(&Bs[kr][nq]) = v;
            }
        } else if (t < BK * (BN / 4)) {
            const int kr = t / (BN / 4), nq = (t % (BN / 4)) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (k0 + kr < p.k && n0 + nq < p.n_pad)
                v = *reinterpret_cast<const float4*>(p.w + (size_t)(k0 + kr) * p.n_pad + n0 + nq);
            *reinterpret_cast<float4*>(&Bs[kr][nq]) = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * TM]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ty * TM + 4]);
            const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * TN]);
            const float ar[TM] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float br[TN] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
        }
        __syncthreads();
    }

    const int hw = p.h * p.w_px;
    const int col0 = n0 + tx * TN;
    if (col0 >= p.n) return;
    const bool full = col0 + TN <= p.n;
    float bias[TN];
#pragma unroll
    for (int j = 0; j < TN; ++j) bias[j] = (p.bias && (full || col0 + j < p.n)) ? p.bias[col0 + j] : 0.f;
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int row = m0 + ty * TM + i;
        if (row >= p.m) break;
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
            const T* r = static_cast<const T*>(p.residual) + rrow * p.ldr + col0;
            const float* g = p.res_gate ? p.res_gate + (size_t)(row / p.rows_per_image) * p.n + col0 : nullptr;
            if (full && (p.ldr % 4) == 0) {
                float4 rv = load4(r);
                if (g) rv = f4_mul(rv, *reinterpret_cast<const float4*>(g));
                o[0] += rv.x; o[1] += rv.y; o[2] += rv.z; o[3] += rv.w;
            } else {
                for (int j = 0; j < TN && col0 + j < p.n; ++j) o[j] += g ? load1(r + j) * g[j] : load1(r + j);
            }
        }
        const size_t off = (size_t)row * p.ldc + p.coff + col0;
        if (p.c_f32) {
            float* c = static_cast<float*>(p.c) + off;
            if (full && (p.ldc % 4) == 0 && (p.coff % 4) == 0) *reinterpret_cast<float4*>(c) = make_float4(o[0], o[1], o[2], o[3]);
            else for (int j = 0; j < TN && col0 + j < p.n; ++j) c[j] = o[j];
        } else {
            T* c = static_cast<T*>(p.c) + off;
            if (full && (p.ldc % 4) == 0 && (p.coff % 4) == 0) store4(c, make_float4(o[0], o[1], o[2], o[3]));
            else for (int j = 0; j < TN && col0 + j < p.n; ++j) c[j] = from_f<T>(o[j]);
        }
    }
}

template <typename T, int BM, int BN>
cudaError_t launch_cfg(const GemmParams& p, cudaStream_t stream) {
    dim3 grid((p.m + BM - 1) / BM, (p.n + BN - 1) / BN);
    gemm_simt_kernel<T, BM, BN><<<grid, THREADS, 0, stream>>>(p);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const GemmParams& p, cudaStream_t stream) {
    if (p.n <= 16) return launch_cfg<T, 512, 16>(p, stream);
    if (p.n <= 32) return launch_cfg<T, 256, 32>(p, stream);
    return launch_cfg<T, 128, 64>(p, stream);
}

}  // namespace

cudaError_t launch_gemm_simt(const GemmParams& p, cudaStream_t stream) {
    if (p.k % 4 || p.lda % 4 || p.n_pad % 4 || p.n_pad < p.n) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_t<float>(p, stream) : launch_t<__nv_bfloat16>(p, stream);
}

}  // namespace ppocr
