// Row-per-thread pointwise kernels for the thin 1x1 convs of the detector and
// the tiny recognizer (K, N <= a few hundred).
//
// pair_rows: the LCNet channel pair (src/cpu/model.rs:591-602,
//   src/cpu/backend.rs:443-695) fused:
//     out = W2 GELU(W1 (a * gate) + b1) + b2 (+ a * gate)
//   One thread owns one pixel row: its C inputs live in registers, each of
//   the 2C hidden units is formed, activated and immediately folded into the
//   C' output accumulators, so the hidden tensor never leaves the SM (the
//   unfused form writes and re-reads 2C values per pixel).  The residual is
//   the gated input row itself (already in registers).
// rows_gemm: C = act(A W + b) (+ residual) with N <= 128 accumulators per
//   thread, K streamed in float4 steps.
// Weights sit in shared memory and are read by broadcast (all lanes of a
// warp read the same address), 4 weights per 16-byte load.  Summation is
// in k order with FMA, as the tiled kernel does.
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int kRows = 128;   // threads (= rows) per block

// R pixel rows per thread: every shared-memory weight load feeds R rows.
template <typename T, int C, int CO, int R>
__global__ void __launch_bounds__(kRows) pair_rows_kernel(PairRowsParams p) {
    constexpr int H = 2 * C;
    extern __shared__ float4 psm[];
    float* w1p = reinterpret_cast<float*>(psm);          // [H / 2][C][2]: hidden units 2jp, 2jp + 1 side by side
    float* w2 = w1p + H * C;                             // [H][CO]
    float* b1 = w2 + H * CO;                             // [H]
    float* b2 = b1 + H;                                  // [CO]
    for (int i = threadIdx.x; i < H * C / 2; i += kRows) {   // i = jp * C + k
        const int jp = i / C, k = i - jp * C;
        *reinterpret_cast<float2*>(w1p + 2 * i) = make_float2(p.w1t[(2 * jp) * C + k], p.w1t[(2 * jp + 1) * C + k]);
    }
    for (int i = threadIdx.x * 4; i < H * CO; i += kRows * 4)
        *reinterpret_cast<float4*>(w2 + i) = *reinterpret_cast<const float4*>(p.w2 + i);
    for (int i = threadIdx.x; i < H; i += kRows) b1[i] = p.b1[i];
    for (int i = threadIdx.x; i < CO; i += kRows) b2[i] = p.b2[i];
    __syncthreads();
    const long long row0 = (long long)blockIdx.x * kRows * R + threadIdx.x;   // rows row0 + r * kRows
    if (row0 >= p.m) return;
    float a[R][C];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const long long row = row0 + (long long)r * kRows < p.m ? row0 + (long long)r * kRows : row0;
        const T* src = static_cast<const T*>(p.a) + (size_t)row * C;
        const float* g = p.gate ? p.gate + (size_t)(row / p.rows_per_image) * C : nullptr;
#pragma unroll
        for (int k = 0; k < C; k += 4) {
            float4 v = load4(src + k);
            if (g) v = f4_mul(v, *reinterpret_cast<const float4*>(g + k));
            a[r][k] = v.x; a[r][k + 1] = v.y; a[r][k + 2] = v.z; a[r][k + 3] = v.w;
        }
    }
    float out[R][CO];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int o = 0; o < CO; ++o) out[r][o] = 0.f;
    // Hidden units in pairs: each packed FMA advances the k-ordered sums of two
    // hidden units (each lane rounded as fmaf), so every hidden value is the
    // same chain of FMAs as one scalar sum.
#pragma unroll 2
    for (int jp = 0; jp < H / 2; ++jp) {
        const float* wj = w1p + jp * C * 2;
        float h0[R], h1[R];
#pragma unroll
        for (int r = 0; r < R; ++r) h0[r] = h1[r] = 0.f;
#pragma unroll
        for (int k = 0; k < C; k += 2) {
            const float4 w = *reinterpret_cast<const float4*>(wj + 2 * k);   // (j, k) (j + 1, k) (j, k + 1) (j + 1, k + 1)
#pragma unroll
            for (int r = 0; r < R; ++r) {
                fma2(h0[r], h1[r], a[r][k], a[r][k], w.x, w.y);
                fma2(h0[r], h1[r], a[r][k + 1], a[r][k + 1], w.z, w.w);
            }
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const int j = 2 * jp + half;
            float h[R];
#pragma unroll
            for (int r = 0; r < R; ++r) h[r] = apply_act((half ? h1[r] : h0[r]) + b1[j], ACT_GELU);
            const float* w2j = w2 + j * CO;
#pragma unroll
            for (int o = 0; o < CO; o += 4) {
                const float4 w = *reinterpret_cast<const float4*>(w2j + o);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    fma2(out[r][o], out[r][o + 1], h[r], h[r], w.x, w.y);
                    fma2(out[r][o + 2], out[r][o + 3], h[r], h[r], w.z, w.w);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
        const long long row = row0 + (long long)r * kRows;
        if (row >= p.m) break;
        T* dst = static_cast<T*>(p.c) + (size_t)row * CO;
#pragma unroll
        for (int o = 0; o < CO; o += 4) {
            float4 v = make_float4(out[r][o] + b2[o], out[r][o + 1] + b2[o + 1], out[r][o + 2] + b2[o + 2],
                                   out[r][o + 3] + b2[o + 3]);
            if (p.residual) {
                // CO == C: the residual is the gated input row (src/cpu/backend.rs:504-521).
                v.x += a[r][o % C]; v.y += a[r][(o + 1) % C]; v.z += a[r][(o + 2) % C]; v.w += a[r][(o + 3) % C];
            }
            store4(dst + o, v);
        }
    }
}

template <typename T, int N>
__global__ void __launch_bounds__(kRows) rows_gemm_kernel(GemmParams p) {
    extern __shared__ float4 rsm[];
    float* w = reinterpret_cast<float*>(rsm);   // [K][N]
    float* bias = w + (size_t)p.k * N;          // [N]
    for (int i = threadIdx.x; i < p.k * (N / 4); i += kRows) {
        const int kk = i / (N / 4), q = (i % (N / 4)) * 4;
        *reinterpret_cast<float4*>(w + kk * N + q) = q < p.n_pad
            ? *reinterpret_cast<const float4*>(p.w + (size_t)kk * p.n_pad + q)
            : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int i = threadIdx.x; i < N; i += kRows) bias[i] = (p.bias && i < p.n) ? p.bias[i] : 0.f;
    __syncthreads();
    const long long row = (long long)blockIdx.x * kRows + threadIdx.x;
    if (row >= p.m) return;
    const T* src = static_cast<const T*>(p.a) + (size_t)row * p.lda;
    const float* g = p.gate ? p.gate + (size_t)(row / p.rows_per_image) * p.k : nullptr;
    float acc[N];
#pragma unroll
    for (int o = 0; o < N; ++o) acc[o] = 0.f;
    for (int kk = 0; kk < p.k; kk += 4) {
        float4 v = load4(src + kk);
        if (g) v = f4_mul(v, *reinterpret_cast<const float4*>(g + kk));
        const float av[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float* wk = w + (kk + q) * N;
#pragma unroll
            for (int o = 0; o < N; o += 4) {
                const float4 ww = *reinterpret_cast<const float4*>(wk + o);
                fma2(acc[o], acc[o + 1], av[q], av[q], ww.x, ww.y);
                fma2(acc[o + 2], acc[o + 3], av[q], av[q], ww.z, ww.w);
            }
        }
    }
    size_t rrow = (size_t)row;
    if (p.residual && p.res_scale > 1) {
        const int hw = p.h * p.w_px;
        const int pimg = (int)(row / hw), rem = (int)(row % hw);
        const int y = rem / p.w_px, x = rem % p.w_px;
        const int rh = p.h / p.res_scale, rw = p.w_px / p.res_scale;
        rrow = ((size_t)pimg * rh + y / p.res_scale) * rw + x / p.res_scale;
    }
    const T* res = p.residual ? static_cast<const T*>(p.residual) + rrow * p.ldr : nullptr;
    const float* rg = p.res_gate ? p.res_gate + (size_t)(row / p.rows_per_image) * p.n : nullptr;
    T* dst = static_cast<T*>(p.c) + (size_t)row * p.ldc + p.coff;
#pragma unroll
    for (int o = 0; o < N; o += 4) {
        if (o >= p.n) break;
        float4 v = make_float4(acc[o] + bias[o], acc[o + 1] + bias[o + 1], acc[o + 2] + bias[o + 2], acc[o + 3] + bias[o + 3]);
        v = f4_act(v, p.act);
        if (res) {
            float4 r = load4(res + o);
            if (rg) r = f4_mul(r, *reinterpret_cast<const float4*>(rg + o));
            v = f4_add(v, r);
        }
        store4(dst + o, v);
    }
}

template <typename T, int C, int CO>
cudaError_t launch_pair(const PairRowsParams& p, cudaStream_t stream) {
    // One row per thread and four hidden units in flight: measured faster than
    // two rows per thread (fewer registers, more resident warps to cover the
    // dependent FMA chains of each hidden unit).
    constexpr int R = 1;
    const size_t smem = ((size_t)2 * C * C + (size_t)2 * C * CO + 2 * C + CO) * sizeof(float);
    {
        cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(pair_rows_kernel<T, C, CO, R>), 200 * 1024);
        if (e != cudaSuccess) return e;
    }
    pair_rows_kernel<T, C, CO, R><<<(unsigned)((p.m + kRows * R - 1) / (kRows * R)), kRows, smem, stream>>>(p);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_pair_t(const PairRowsParams& p, cudaStream_t stream) {
#define PAIR_CASE(C_, CO_) \
    if (p.c_in == C_ && p.c_out == CO_) return launch_pair<T, C_, CO_>(p, stream);
    PAIR_CASE(16, 16) PAIR_CASE(16, 32) PAIR_CASE(24, 24) PAIR_CASE(24, 48) PAIR_CASE(32, 32) PAIR_CASE(32, 48)
    PAIR_CASE(32, 64) PAIR_CASE(48, 48) PAIR_CASE(48, 64) PAIR_CASE(48, 96) PAIR_CASE(64, 64) PAIR_CASE(64, 96)
#undef PAIR_CASE
    return cudaErrorInvalidValue;
}

template <typename T, int N>
cudaError_t launch_rows(const GemmParams& p, cudaStream_t stream) {
    const size_t smem = ((size_t)p.k * N + N) * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidConfiguration;
    {
        cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(rows_gemm_kernel<T, N>), 200 * 1024);
        if (e != cudaSuccess) return e;
    }
    rows_gemm_kernel<T, N><<<(unsigned)((p.m + kRows - 1) / kRows), kRows, smem, stream>>>(p);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_rows_t(const GemmParams& p, cudaStream_t stream) {
    const int n4 = (p.n + 3) / 4 * 4;
    if (n4 <= 16) return launch_rows<T, 16>(p, stream);
    if (n4 <= 32) return launch_rows<T, 32>(p, stream);
    if (n4 <= 48) return launch_rows<T, 48>(p, stream);
    if (n4 <= 64) return launch_rows<T, 64>(p, stream);
    if (n4 <= 96) return launch_rows<T, 96>(p, stream);
    return launch_rows<T, 128>(p, stream);
}

}  // namespace

bool pair_rows_supported(int c_in, int c_out) {
    static const int cases[][2] = {{16, 16}, {16, 32}, {24, 24}, {24, 48}, {32, 32}, {32, 48},
                                   {32, 64}, {48, 48}, {48, 64}, {48, 96}, {64, 64}, {64, 96}};
    for (auto& c : cases)
        if (c[0] == c_in && c[1] == c_out) return true;
    return false;
}

cudaError_t launch_pair_rows(const PairRowsParams& p, cudaStream_t stream) {
    if (!pair_rows_supported(p.c_in, p.c_out) || (p.residual && p.c_in != p.c_out)) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_pair_t<float>(p, stream) : launch_pair_t<__nv_bfloat16>(p, stream);
}

bool rows_gemm_supported(const GemmParams& p) {
    return p.n <= 128 && p.k % 4 == 0 && p.lda % 4 == 0 && p.ldc % 4 == 0 && p.coff % 4 == 0 && p.n % 4 == 0 &&
           !p.c_f32 && (size_t)p.k * 128 * 4 <= 200 * 1024 && (!p.residual || p.ldr % 4 == 0);
}

cudaError_t launch_rows_gemm(const GemmParams& p, cudaStream_t stream) {
    if (!rows_gemm_supported(p)) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_rows_t<float>(p, stream) : launch_rows_t<__nv_bfloat16>(p, stream);
}

}  // namespace ppocr
