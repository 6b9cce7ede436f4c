// FP32 pointwise GEMM (the FP32-mode path for 1x1 convs and linears).
//
// C[m, n] = act(A[m, k] * W[k, n] + bias) (+ residual), with the optional SE
// gate on A and on the residual, and a nearest-upsampled residual for the
// medium neck's top-down adds (src/cpu/model.rs:1022-1066).  64x64 output
// tile per 256-thread block, 4x4 outputs per thread, K in steps of 16 staged
// through shared memory.  Exact FP32 products and sums, as the reference's
// packed CPU GEMMs compute them (only the summation order differs).
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int BM = 64, BN = 64, BK = 16;

template <typename T>
__device__ __forceinline__ float load1(const T* p) { return to_f(*p); }

template <typename T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(GemmParams p) {
    __shared__ __align__(16) float As[BK][BM];
    __shared__ __align__(16) float Bs[BK][BN];
    const int t = threadIdx.x;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int ty = t / 16, tx = t % 16;
    const T* A = static_cast<const T*>(p.a);
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

    const int a_row = t / 4, a_k = (t % 4) * 4;
    const int b_k = t / 16, b_n = (t % 16) * 4;
    const int grow = m0 + a_row;
    const float* grow_gate = nullptr;
    if (p.gate && grow < p.m) grow_gate = p.gate + (size_t)(grow / p.rows_per_image) * p.k;

    for (int k0 = 0; k0 < p.k; k0 += BK) {
        float4 av = make_float4(0.f, 0.f, 0.f, 0.f);
        if (grow < p.m && k0 + a_k < p.k) {
            av = load4(A + (size_t)grow * p.lda + k0 + a_k);
            if (grow_gate) av = f4_mul(av, *reinterpret_cast<const float4*>(grow_gate + k0 + a_k));
        }
        As[a_k + 0][a_row] = av.x;
        As[a_k + 1][a_row] = av.y;
        As[a_k + 2][a_row] = av.z;
        As[a_k + 3][a_row] = av.w;
        float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (k0 + b_k < p.k && n0 + b_n < p.n_pad)
            bv = *reinterpret_cast<const float4*>(p.w + (size_t)(k0 + b_k) * p.n_pad + n0 + b_n);
        *reinterpret_cast<float4*>(&Bs[b_k][b_n]) = bv;
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
            const float ar[4] = {a.x, a.y, a.z, a.w};
            const float br[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
        }
        __syncthreads();
    }

    const int hw = p.h * p.w_px;
    for (int i = 0; i < 4; ++i) {
        const int row = m0 + ty * 4 + i;
        if (row >= p.m) break;
        const int img = row / p.rows_per_image;
        size_t rrow = (size_t)row;
        if (p.residual && p.res_scale > 1) {
            const int pimg = row / hw, rem = row % hw;
            const int y = rem / p.w_px, x = rem % p.w_px;
            const int rh = p.h / p.res_scale, rw = p.w_px / p.res_scale;
            rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
        }
        for (int j = 0; j < 4; ++j) {
            const int col = n0 + tx * 4 + j;
            if (col >= p.n) break;
            float v = acc[i][j];
            if (p.bias) v += p.bias[col];
            v = apply_act(v, p.act);
            if (p.residual) {
                float r = load1(static_cast<const T*>(p.residual) + rrow * p.ldr + col);
                if (p.res_gate) r *= p.res_gate[(size_t)img * p.n + col];
                v += r;
            }
            const size_t o = (size_t)row * p.ldc + p.coff + col;
            if (p.c_f32) static_cast<float*>(p.c)[o] = v;
            else static_cast<T*>(p.c)[o] = from_f<T>(v);
        }
    }
}

}  // namespace

cudaError_t launch_gemm_simt(const GemmParams& p, cudaStream_t stream) {
    if (p.k % 4 || p.lda % 4 || p.n_pad % 4 || p.n_pad < p.n) return cudaErrorInvalidValue;
    dim3 grid((p.m + BM - 1) / BM, (p.n + BN - 1) / BN);
    if (p.dtype == DT_F32) gemm_simt_kernel<float><<<grid, 256, 0, stream>>>(p);
    else gemm_simt_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace ppocr
