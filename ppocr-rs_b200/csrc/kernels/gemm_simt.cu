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
//
// A is loaded with four consecutive threads per row (64 contiguous bytes of
// FP32), and stored transposed with the row index XOR-swizzled by the K
// quad, so both the shared stores and the 16-byte shared reads are free of
// bank conflicts.
//
// The same kernel runs dense convolutions as implicit GEMMs (CONV = true):
// row = output pixel, k = (ky, kx, c) over the virtual concatenation of NHWC
// sources (nearest-upsampled or 2x2 max-pooled views), gathered while A is
// staged; out-of-image taps contribute zeros.  Per output the FMAs run in k
// order, i.e. (ky, kx, channel), as in the direct convolution.
#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int BK = 16, TM = 8, TN = 4, THREADS = 256;

template <typename T>
__device__ __forceinline__ float load1(const T* p) { return to_f(*p); }

// Row index of A element (k, r) in the transposed shared tile: r XOR 8 * (k / 4 % 4).
__device__ __forceinline__ int a_swz(int k, int r) { return r ^ (((k >> 2) & 3) << 3); }

template <typename T, int BM, int BN, bool CONV>
__global__ void __launch_bounds__(THREADS) gemm_simt_kernel(GemmParams p, ConvGather g) {
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

    // A tile: BM rows x BK columns = BM * 4 float4; thread t loads quad t % 4 of
    // rows t / 4 + 64 l (four threads per row: 64 contiguous bytes).
    constexpr int A_LOADS = BM * (BK / 4) / THREADS;
    constexpr int B_LOADS = BK * (BN / 4) / THREADS;   // may be 0 for BN < 64 -> handled below
    const int kq = t & 3;
    // Implicit GEMM: each loaded row's output pixel, as (oy * sh - pt, ox * sw - pl, image).
    int iyb[CONV ? A_LOADS : 1], ixb[CONV ? A_LOADS : 1], pim[CONV ? A_LOADS : 1];
    int ky = 0, kx = 0, c = kq * 4;   // this thread's quad position in k = (ky, kx, c)
    if (CONV) {
#pragma unroll
        for (int l = 0; l < A_LOADS; ++l) {
            const int row = m0 + (t >> 2) + l * (THREADS / 4);
            const int rr = row < p.m ? row : 0;
            const int ox = rr % g.wo, rest = rr / g.wo;
            iyb[l] = (rest % g.ho) * g.sh - g.pt;
            ixb[l] = ox * g.sw - g.pl;
            pim[l] = row < p.m ? rest / g.ho : -1;
        }
        while (c >= g.cin) { c -= g.cin; if (++kx == g.kw) { kx = 0; ++ky; } }
    }
    for (int k0 = 0; k0 < p.k; k0 += BK) {
        if (CONV) {
            // The source view holding channel c (NHWC sources hold whole quads).
            int s = 0, cs = c;
            while (s + 1 < g.nsrc && cs >= g.src[s].channels) { cs -= g.src[s].channels; ++s; }
            const ConvSource& src = g.src[s];
            const T* base = static_cast<const T*>(src.ptr);
            const int shift = g.shift[s];
            const int hs = g.hi >> shift, ws = g.wi >> shift;
            const bool kin = ky < g.kh;
#pragma unroll
            for (int l = 0; l < A_LOADS; ++l) {
                const int r = (t >> 2) + l * (THREADS / 4);
                const int iy = iyb[l] + ky, ix = ixb[l] + kx;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (kin && pim[l] >= 0 && iy >= 0 && iy < g.hi && ix >= 0 && ix < g.wi) {
                    const int sy = iy >> shift, sx = ix >> shift;
                    const T* px = base + ((size_t)(pim[l] * hs + sy) * ws + sx) * src.cstride + src.coff + cs;
                    v = load4(px);
                    if (src.mode == SRC_NHWC_MAXPOOL) {
                        // 2x2 window anchored at the pixel; positions past the bottom /
                        // right edge are padding and never win (pads [0, 0, 1, 1]).
                        const bool right = sx + 1 < ws, down = sy + 1 < hs;
                        if (right) v = f4_max(v, load4(px + src.cstride));
                        if (down) {
                            v = f4_max(v, load4(px + (size_t)ws * src.cstride));
                            if (right) v = f4_max(v, load4(px + (size_t)(ws + 1) * src.cstride));
                        }
                    }
                }
                As[kq * 4 + 0][a_swz(kq * 4, r)] = v.x;
                As[kq * 4 + 1][a_swz(kq * 4, r)] = v.y;
                As[kq * 4 + 2][a_swz(kq * 4, r)] = v.z;
                As[kq * 4 + 3][a_swz(kq * 4, r)] = v.w;
            }
            // Advance this thread's quad by BK channels of k.
            c += BK;
            while (c >= g.cin && ky < g.kh) { c -= g.cin; if (++kx == g.kw) { kx = 0; ++ky; } }
        } else {
#pragma unroll
            for (int l = 0; l < A_LOADS; ++l) {
                const int r = (t >> 2) + l * (THREADS / 4);
                const int row = m0 + r, kk = k0 + kq * 4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (row < p.m && kk < p.k) {
                    v = load4(A + (size_t)row * p.lda + kk);
                    if (p.gate) v = f4_mul(v, *reinterpret_cast<const float4*>(p.gate + (size_t)(row / p.rows_per_image) * p.k + kk));
                }
                As[kq * 4 + 0][a_swz(kq * 4, r)] = v.x;
                As[kq * 4 + 1][a_swz(kq * 4, r)] = v.y;
                As[kq * 4 + 2][a_swz(kq * 4, r)] = v.z;
                As[kq * 4 + 3][a_swz(kq * 4, r)] = v.w;
            }
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
            const int ar0 = a_swz(kk, ty * TM);   // TM = 8: the swizzle keeps the 8 rows contiguous
            const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ar0]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][ar0 + 4]);
            const float4 b = *reinterpret_cast<const float4*>(&Bs[kk][tx * TN]);
            const float ar[TM] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float br[TN] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < TM; i += 2)
#pragma unroll
                for (int j = 0; j < TN; ++j) fma2(acc[i][j], acc[i + 1][j], ar[i], ar[i + 1], br[j], br[j]);
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

template <typename T, int BM, int BN, bool CONV>
cudaError_t launch_cfg(const GemmParams& p, const ConvGather& g, cudaStream_t stream) {
    const long long mt = ((long long)p.m + BM - 1) / BM;
    if (mt > 0x7fffffffLL || (p.n + BN - 1) / BN > 65535) return cudaErrorInvalidConfiguration;
    dim3 grid((unsigned)mt, (p.n + BN - 1) / BN);
    gemm_simt_kernel<T, BM, BN, CONV><<<grid, THREADS, 0, stream>>>(p, g);
    return cudaGetLastError();
}

template <typename T, bool CONV>
cudaError_t launch_t(const GemmParams& p, const ConvGather& g, cudaStream_t stream) {
    if (p.n <= 16) return launch_cfg<T, 512, 16, CONV>(p, g, stream);
    if (p.n <= 32) return launch_cfg<T, 256, 32, CONV>(p, g, stream);
    return launch_cfg<T, 128, 64, CONV>(p, g, stream);
}

}  // namespace

cudaError_t launch_gemm_simt(const GemmParams& p, cudaStream_t stream) {
    if (p.k % 4 || p.lda % 4 || p.n_pad % 4 || p.n_pad < p.n) return cudaErrorInvalidValue;
    const ConvGather g{};
    return p.dtype == DT_F32 ? launch_t<float, false>(p, g, stream) : launch_t<__nv_bfloat16, false>(p, g, stream);
}

bool conv_gemm_supported(const ConvParams& p) {
    if (p.cin % 4 || p.cout < 16 || p.nsrc < 1 || p.nsrc > 4) return false;
    for (int s = 0; s < p.nsrc; ++s) {
        const ConvSource& src = p.src[s];
        if (src.mode == SRC_NCHW_F32 || src.channels % 4 || src.cstride % 4 || src.coff % 4) return false;
        if (src.scale < 1 || (src.scale & (src.scale - 1)) || p.hi % src.scale || p.wi % src.scale) return false;
        if (src.mode == SRC_NHWC_MAXPOOL && src.scale != 1) return false;
    }
    return true;
}

cudaError_t launch_conv_gemm(const ConvParams& p, cudaStream_t stream) {
    if (!conv_gemm_supported(p) || !p.weight_kn || p.n_pad % 4 || p.n_pad < p.cout) return cudaErrorInvalidValue;
    ConvGather g{};
    g.hi = p.hi; g.wi = p.wi; g.ho = p.ho; g.wo = p.wo; g.cin = p.cin; g.kh = p.kh; g.kw = p.kw;
    g.sh = p.sh; g.sw = p.sw; g.pt = p.pt; g.pl = p.pl; g.nsrc = p.nsrc;
    for (int s = 0; s < p.nsrc; ++s) {
        g.src[s] = p.src[s];
        while ((1 << g.shift[s]) < p.src[s].scale) ++g.shift[s];
    }
    GemmParams q;
    const long long m = (long long)p.n * p.ho * p.wo;
    if (m > 0x7fffffffLL) return cudaErrorInvalidValue;
    q.m = (int)m; q.n = p.cout; q.k = p.kh * p.kw * p.cin;
    q.w = p.weight_kn; q.n_pad = p.n_pad;
    q.bias = p.bias; q.act = p.act;
    q.residual = p.residual; q.ldr = p.cout;
    q.res_scale = p.res_scale; q.h = p.ho; q.w_px = p.wo;
    q.c = p.out; q.ldc = p.out_cstride; q.coff = p.out_coff; q.dtype = p.dtype;
    q.k_pad = q.k; q.lda = 4;   // unused in CONV mode (A is gathered)
    return p.dtype == DT_F32 ? launch_t<float, true>(q, g, stream) : launch_t<__nv_bfloat16, true>(q, g, stream);
}

}  // namespace ppocr
