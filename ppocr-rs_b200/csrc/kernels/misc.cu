// Squeeze-excitation, detector-head tail, recognizer ops, preprocessing and
// small conversion kernels.  Reference semantics are cited per kernel.
#include "common.cuh"
#include "kernels.h"

#include <cfloat>

namespace ppocr {
namespace {

// ---------------------------------------------------------------------------
// SE: per-(image, channel) sums over pixels (global_avg_pool2d numerator,
// src/cpu/model.rs:488).  grid = (chunks, images); each thread owns 4
// channels of a strided pixel slice of its chunk; the slices are reduced in
// shared memory in a fixed order and the block writes its chunk partial (no
// atomics, so every run produces the same bits).
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) channel_sum_kernel(PoolParams p) {
    __shared__ float4 part[256];
    const int cg = p.c / 4;
    const int rows = blockDim.x / cg;          // pixel lanes per block
    const int g = threadIdx.x % cg, r = threadIdx.x / cg;
    const int img = blockIdx.y, chunk = blockIdx.x;
    const int per = (p.hw + p.chunks - 1) / p.chunks;
    const int px0 = chunk * per, px1 = min(p.hw, px0 + per);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows) {
        const T* base = static_cast<const T*>(p.in) + (size_t)img * p.hw * p.in_cstride + g * 4;
        // Unrolled so several loads are in flight; the adds stay in pixel order.
#pragma unroll 4
        for (int px = px0 + r; px < px1; px += rows) acc = f4_add(acc, load4(base + (size_t)px * p.in_cstride));
    }
    part[threadIdx.x] = acc;
    __syncthreads();
    if (r == 0) {
        for (int i = 1; i < rows; ++i) acc = f4_add(acc, part[i * cg + g]);
        *reinterpret_cast<float4*>(p.sum + ((size_t)img * p.chunks + chunk) * p.c + g * 4) = acc;
    }
}

// gate = hard_sigmoid(W2 relu(W1 mean + b1) + b2; alpha, 0.5)
// (SqueezeExcitation src/cpu/model.rs:486-492, VariantSqueezeExcitation 1098-1104)
// A block serves IMG images so every weight row it streams feeds IMG dot
// products.  Each output unit is one thread's sequential FMA chain over its
// weight row, starting from the bias, in input order; rows are streamed with
// 16-byte loads.  ACC is the accumulation type: double for the FP32 mode
// (where a gate's pre-activation can be a near-cancelling sum of large terms,
// so its rounding is amplified into the gated channel), float for BF16.
// GATE = false: hid = relu(.); GATE = true: gate = hard_sigmoid(.; alpha, 0.5).
template <typename ACC, int IMG, bool GATE, typename OUT>
__device__ __forceinline__ void se_dot_rows(const float* __restrict__ w, const float* __restrict__ bias, const ACC* in,
                                            int in_len, int out_len, float alpha, OUT* out, size_t out_stride, int nimg) {
    const bool vec = (in_len % 4) == 0;
    for (int j = threadIdx.x; j < out_len; j += blockDim.x) {
        ACC a[IMG];
#pragma unroll
        for (int k = 0; k < IMG; ++k) a[k] = (ACC)bias[j];
        const float* row = w + (size_t)j * in_len;
        if (vec) {
            const float4* row4 = reinterpret_cast<const float4*>(row);
#pragma unroll 8
            for (int i4 = 0; i4 < in_len / 4; ++i4) {
                const float4 wv = __ldg(row4 + i4);
#pragma unroll
                for (int k = 0; k < IMG; ++k) {
                    const ACC* x = in + k * in_len + 4 * i4;
                    a[k] = fma((ACC)wv.x, x[0], a[k]);
                    a[k] = fma((ACC)wv.y, x[1], a[k]);
                    a[k] = fma((ACC)wv.z, x[2], a[k]);
                    a[k] = fma((ACC)wv.w, x[3], a[k]);
                }
            }
        } else {
#pragma unroll 4
            for (int i = 0; i < in_len; ++i) {
                const ACC wv = (ACC)__ldg(row + i);
#pragma unroll
                for (int k = 0; k < IMG; ++k) a[k] = fma(wv, in[k * in_len + i], a[k]);
            }
        }
        for (int k = 0; k < nimg; ++k) {
            if (GATE) {
                const float v = (float)a[k];
                out[k * out_stride + j] = (OUT)fminf(fmaxf(fmaf(v, alpha, 0.5f), 0.f), 1.f);
            } else {
                out[k * out_stride + j] = (OUT)(a[k] > (ACC)0 ? a[k] : (ACC)0);
            }
        }
    }
}

// Sum of `count` chunk partials at `stride`, in chunk order, with the loads
// issued sixteen at a time (the same sums as one load-add chain, without a
// cache round trip per partial).  L2: read through to L2, for partials other
// blocks of the same launch have just written.
template <typename ACC, bool L2>
__device__ __forceinline__ ACC ordered_chunk_sum(const float* src, int count, size_t stride) {
    ACC s = 0;
    for (int ch = 0; ch < count; ch += 16) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float* q = src + (size_t)(ch + j) * stride;
            v[j] = ch + j < count ? (L2 ? __ldcg(q) : __ldg(q)) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) s += (ACC)v[j];   // adding a zero past the end is exact
    }
    return s;
}

template <typename ACC, int IMG>
__global__ void __launch_bounds__(256) se_mlp_kernel(SeMlpParams p) {
    extern __shared__ float4 sm4[];
    ACC* mean = reinterpret_cast<ACC*>(sm4);   // [IMG][c]
    ACC* hid = mean + IMG * p.c;               // [IMG][r]
    const int img0 = blockIdx.x * IMG;
    const int nimg = min(IMG, p.n - img0);
    const ACC inv = (ACC)1 / (ACC)p.hw;
    for (int t = threadIdx.x; t < IMG * p.c; t += blockDim.x) {
        const int k = t / p.c, i = t % p.c;
        ACC s = 0;
        if (k < nimg) s = ordered_chunk_sum<ACC, false>(p.sum + (size_t)(img0 + k) * p.chunks * p.c + i, p.chunks, (size_t)p.c);
        mean[t] = s * inv;
    }
    for (int t = threadIdx.x; t < IMG * p.r; t += blockDim.x) hid[t] = 0;
    __syncthreads();
    se_dot_rows<ACC, IMG, false, ACC>(p.w1, p.b1, mean, p.c, p.r, 0.f, hid, (size_t)p.r, nimg);
    __syncthreads();
    se_dot_rows<ACC, IMG, true, float>(p.w2, p.b2, hid, p.r, p.c, p.alpha, p.gate + (size_t)img0 * p.c, (size_t)p.c, nimg);
}

// channel_sum_kernel's chunk sums, then, in the last block to finish an
// image, se_mlp_kernel's arithmetic for that image (IMG = 1).
template <typename T, typename ACC>
__global__ void __launch_bounds__(256) se_pool_mlp_kernel(SePoolParams sp) {
    const PoolParams& p = sp.pool;
    __shared__ float4 part[256];
    __shared__ int last;
    const int cg = p.c / 4;
    const int rows = blockDim.x / cg;
    const int g = threadIdx.x % cg, r = threadIdx.x / cg;
    const int img = blockIdx.y, chunk = blockIdx.x;
    const int per = (p.hw + p.chunks - 1) / p.chunks;
    const int px0 = chunk * per, px1 = min(p.hw, px0 + per);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows) {
        const T* base = static_cast<const T*>(p.in) + (size_t)img * p.hw * p.in_cstride + g * 4;
#pragma unroll 4
        for (int px = px0 + r; px < px1; px += rows) acc = f4_add(acc, load4(base + (size_t)px * p.in_cstride));
    }
    part[threadIdx.x] = acc;
    __syncthreads();
    if (r == 0) {
        for (int i = 1; i < rows; ++i) acc = f4_add(acc, part[i * cg + g]);
        *reinterpret_cast<float4*>(p.sum + ((size_t)img * p.chunks + chunk) * p.c + g * 4) = acc;
    }
    // Publish this block's sums, then count it in; the image's last block
    // (whichever it is) computes the gate from all chunk sums.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(sp.counters + img, 1) == p.chunks - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    extern __shared__ float4 sm4[];
    const SeMlpParams& m = sp.mlp;
    ACC* mean = reinterpret_cast<ACC*>(sm4);   // [c]
    ACC* hid = mean + m.c;                     // [r]
    const ACC inv = (ACC)1 / (ACC)m.hw;
    for (int i = threadIdx.x; i < m.c; i += blockDim.x) {
        const ACC s = ordered_chunk_sum<ACC, true>(p.sum + (size_t)img * p.chunks * p.c + i, p.chunks, (size_t)p.c);
        mean[i] = s * inv;
    }
    for (int i = threadIdx.x; i < m.r; i += blockDim.x) hid[i] = 0;
    __syncthreads();
    se_dot_rows<ACC, 1, false, ACC>(m.w1, m.b1, mean, m.c, m.r, 0.f, hid, (size_t)m.r, 1);
    __syncthreads();
    se_dot_rows<ACC, 1, true, float>(m.w2, m.b2, hid, m.r, m.c, m.alpha, m.gate + (size_t)img * m.c, (size_t)m.c, 1);
    if (threadIdx.x == 0) sp.counters[img] = 0;   // ready for the next launch
}

// out = x*g or x + x*g (residual_mul_in_place, src/cpu/kernels/mod.rs:777-796),
// then + nearest-upsampled addend (upsample_add_nchw, src/cpu/model.rs:1265-1320).
// I: the index type, 32-bit when the element count fits (64-bit division
// costs several times the arithmetic of this bandwidth-bound loop).
template <typename T, typename I>
__global__ void __launch_bounds__(256) gate_apply_kernel(GateApplyParams p) {
    const I cg = (I)(p.c / 4);
    const I total = (I)p.n * (I)p.h * (I)p.w * cg;
    const I hw = (I)p.h * (I)p.w;
    for (I idx = (I)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (I)gridDim.x * blockDim.x) {
        const int c = (int)(idx % cg) * 4;
        const I pix = idx / cg;
        const int img = (int)(pix / hw);
        float4 v = load4(static_cast<const T*>(p.x) + (size_t)pix * p.c + c);
        if (p.gate) {
            const float4 g = *reinterpret_cast<const float4*>(p.gate + (size_t)img * p.c + c);
            const float4 s = f4_mul(v, g);
            v = p.mode ? f4_add(s, v) : s;
        }
        if (p.addend) {
            const int x = (int)(pix % (I)p.w), y = (int)((pix / (I)p.w) % (I)p.h);
            const int ah = p.h / p.add_scale, aw = p.w / p.add_scale;
            const size_t ai = ((size_t)(img * ah + y / p.add_scale) * aw + x / p.add_scale) * p.c + c;
            v = f4_add(v, load4(static_cast<const T*>(p.addend) + ai));
        }
        store4(static_cast<T*>(p.out) + (size_t)pix * p.out_cstride + p.out_coff + c, v);
    }
}

// ---------------------------------------------------------------------------
// Detector head tail (DetectorHead::forward after conv_down,
// src/cpu/model.rs:1516-1520; ConvTranspose 2x2 s2 IOHW, backend.rs:996-1181):
// each thread takes one conv_down pixel, expands it through both transposed
// convs to its 4x4 output patch, applies the sigmoid and the DB threshold.
// ---------------------------------------------------------------------------
template <typename T, int CH>
__global__ void __launch_bounds__(128) det_head_kernel(HeadParams p) {
    extern __shared__ float hsm[];
    float* wup = hsm;                  // [4][CH][CH]
    float* bup = wup + 4 * CH * CH;    // [CH]
    float* wfin = bup + CH;            // [4][CH]
    for (int i = threadIdx.x; i < 4 * CH * CH; i += blockDim.x) wup[i] = p.w_up[i];
    for (int i = threadIdx.x; i < CH; i += blockDim.x) bup[i] = p.b_up[i];
    for (int i = threadIdx.x; i < 4 * CH; i += blockDim.x) wfin[i] = p.w_fin[i];
    __syncthreads();
    const long long total = (long long)p.n * p.h * p.w;
    const long long pix = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (pix >= total) return;
    const int x = (int)(pix % p.w), y = (int)((pix / p.w) % p.h);
    const int img = (int)(pix / ((long long)p.w * p.h));
    float in[CH];
    const T* src = static_cast<const T*>(p.in) + (size_t)pix * CH;
#pragma unroll
    for (int c = 0; c < CH; c += 4) {
        const float4 v = load4(src + c);
        in[c] = v.x; in[c + 1] = v.y; in[c + 2] = v.z; in[c + 3] = v.w;
    }
    const int W = p.w * 4;
    // First transposed conv tap (a, b) puts hidden pixel (2y + a, 2x + b);
    // the second tap (c, d) of that pixel lands at (4y + 2a + c, 4x + 2b + d).
    // Hidden units of tap (a, b): bias, then the inputs in ci order (packed
    // pairs of output channels, each lane rounded as fmaf), then ReLU.
    auto hidden = [&](int a, int b, float (&h)[CH]) {
#pragma unroll
        for (int co = 0; co < CH; ++co) h[co] = bup[co];
        const float* w0 = wup + (a * 2 + b) * CH * CH;
        // Fully unrolled for the narrow heads so the input row stays in
        // registers; the weights come four per 16-byte shared load (every
        // thread reads the same address: a broadcast), not two per packed FMA.
#pragma unroll (CH <= 24 ? CH : 2)
        for (int ci = 0; ci < CH; ++ci) {
            const float v = in[ci];
            const float4* wr = reinterpret_cast<const float4*>(w0 + ci * CH);
#pragma unroll
            for (int q = 0; q < CH / 4; ++q) {
                const float4 w4 = wr[q];
                fma2(h[4 * q], h[4 * q + 1], v, v, w4.x, w4.y);
                fma2(h[4 * q + 2], h[4 * q + 3], v, v, w4.z, w4.w);
            }
        }
#pragma unroll
        for (int co = 0; co < CH; ++co) h[co] = fmaxf(h[co], 0.f);
    };
    // Output columns 2b, 2b + 1 of row c from hidden tap b: the two d as one
    // packed pair of co-ordered sums.
    auto final_pair = [&](const float (&h)[CH], int c, float& l0, float& l1) {
        l0 = p.b_fin;
        l1 = p.b_fin;
        const float4* wf0 = reinterpret_cast<const float4*>(wfin + (c * 2) * CH);
        const float4* wf1 = reinterpret_cast<const float4*>(wfin + (c * 2 + 1) * CH);
#pragma unroll
        for (int q = 0; q < CH / 4; ++q) {
            const float4 a4 = wf0[q], b4 = wf1[q];
            fma2(l0, l1, h[4 * q], h[4 * q], a4.x, b4.x);
            fma2(l0, l1, h[4 * q + 1], h[4 * q + 1], a4.y, b4.y);
            fma2(l0, l1, h[4 * q + 2], h[4 * q + 2], a4.z, b4.z);
            fma2(l0, l1, h[4 * q + 3], h[4 * q + 3], a4.w, b4.w);
        }
    };
    if constexpr (CH <= 24) {
        // Both hidden taps of a row pair in registers: each output row of the
        // 4 x 4 patch leaves as one 16-byte probability store and one 4-byte
        // mask store (a warp's stores are contiguous).
        for (int a = 0; a < 2; ++a) {
            float h0[CH], h1[CH];
            hidden(a, 0, h0);
            hidden(a, 1, h1);
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float l[4];
                final_pair(h0, c, l[0], l[1]);
                final_pair(h1, c, l[2], l[3]);
                const size_t o = ((size_t)img * p.h * 4 + (size_t)(4 * y + 2 * a + c)) * W + 4 * x;
                if (p.logits) *reinterpret_cast<float4*>(p.logits + o) = make_float4(l[0], l[1], l[2], l[3]);
                float4 pr;
                pr.x = 1.f / (1.f + expf(-l[0]));
                pr.y = 1.f / (1.f + expf(-l[1]));
                pr.z = 1.f / (1.f + expf(-l[2]));
                pr.w = 1.f / (1.f + expf(-l[3]));
                if (p.prob) *reinterpret_cast<float4*>(p.prob + o) = pr;
                if (p.mask) {
                    uchar4 m;
                    m.x = pr.x >= p.threshold;
                    m.y = pr.y >= p.threshold;
                    m.z = pr.z >= p.threshold;
                    m.w = pr.w >= p.threshold;
                    *reinterpret_cast<uchar4*>(p.mask + o) = m;
                }
            }
        }
    } else {
        for (int a = 0; a < 2; ++a) {
            for (int b = 0; b < 2; ++b) {
                float h[CH];
                hidden(a, b, h);
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    float l0, l1;
                    final_pair(h, c, l0, l1);
                    const size_t o = ((size_t)img * p.h * 4 + (size_t)(4 * y + 2 * a + c)) * W + 4 * x + 2 * b;
                    if (p.logits) *reinterpret_cast<float2*>(p.logits + o) = make_float2(l0, l1);
                    const float2 pr = make_float2(1.f / (1.f + expf(-l0)), 1.f / (1.f + expf(-l1)));
                    if (p.prob) *reinterpret_cast<float2*>(p.prob + o) = pr;
                    if (p.mask) {
                        uchar2 m;
                        m.x = pr.x >= p.threshold;
                        m.y = pr.y >= p.threshold;
                        *reinterpret_cast<uchar2*>(p.mask + o) = m;
                    }
                }
            }
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(256) maxpool_su_kernel(MaxPoolParams p) {
    const int cg = p.c / 4;
    const long long total = (long long)p.n * p.h * p.w * cg;
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(idx % cg) * 4;
        const long long pix = idx / cg;
        const int x = (int)(pix % p.w), y = (int)((pix / p.w) % p.h);
        const T* in = static_cast<const T*>(p.in);
        const size_t base = (size_t)pix * p.c + c;
        float4 m = load4(in + base);
        auto mx = [](float4 a, float4 b) {
            return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
        };
        if (x + 1 < p.w) m = mx(m, load4(in + base + p.c));
        if (y + 1 < p.h) {
            m = mx(m, load4(in + base + (size_t)p.w * p.c));
            if (x + 1 < p.w) m = mx(m, load4(in + base + (size_t)p.w * p.c + p.c));
        }
        store4(static_cast<T*>(p.out) + (size_t)pix * p.out_cstride + p.out_coff + c, m);
    }
}

// ---------------------------------------------------------------------------
// Recognizer ops
// ---------------------------------------------------------------------------
template <typename T>
__global__ void avgpool_3x2_kernel(AvgPoolParams p) {
    const int oh = p.h / 3, ow = p.w / 2, cg = p.c / 4;
    const long long total = (long long)p.n * oh * ow * cg;
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(idx % cg) * 4;
        const long long pix = idx / cg;
        const int ox = (int)(pix % ow), oy = (int)((pix / ow) % oh);
        const int img = (int)(pix / ((long long)ow * oh));
        const T* in = static_cast<const T*>(p.in);
        auto at = [&](int yy, int xx) { return load4(in + ((size_t)(img * p.h + yy) * p.w + xx) * p.c + c); };
        // (row0[x] + row0[x+1] + row1[x] + row1[x+1] + row2[x] + row2[x+1]) / 6, left to right.
        float4 s = at(oy * 3, ox * 2);
        s = f4_add(s, at(oy * 3, ox * 2 + 1));
        s = f4_add(s, at(oy * 3 + 1, ox * 2));
        s = f4_add(s, at(oy * 3 + 1, ox * 2 + 1));
        s = f4_add(s, at(oy * 3 + 2, ox * 2));
        s = f4_add(s, at(oy * 3 + 2, ox * 2 + 1));
        s = make_float4(s.x / 6.f, s.y / 6.f, s.z / 6.f, s.w / 6.f);
        store4(static_cast<T*>(p.out) + (size_t)pix * p.c + c, s);
    }
}

template <typename T>
__global__ void __launch_bounds__(256) layernorm_kernel(LayerNormParams p) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= p.rows) return;
    const T* in = static_cast<const T*>(p.in) + (size_t)warp * p.c;
    float s = 0.f;
    for (int i = lane; i < p.c; i += 32) s += to_f(in[i]);
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)p.c;
    float v = 0.f;
    for (int i = lane; i < p.c; i += 32) { const float d = to_f(in[i]) - mean; v = fmaf(d, d, v); }
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const float inv = 1.f / sqrtf(v / (float)p.c + p.eps);
    T* out = static_cast<T*>(p.out) + (size_t)warp * p.c;
    const T* res = p.residual ? static_cast<const T*>(p.residual) + (size_t)warp * p.c : nullptr;
    for (int i = lane; i < p.c; i += 32) {
        float y = fmaf(to_f(in[i]) - mean, inv * p.weight[i], p.bias[i]);
        if (res) y += to_f(res[i]);
        out[i] = from_f<T>(y);
    }
}

// One block per (image, head).  K and V of the head in shared memory; each
// warp takes query rows, holds its score row in shared memory, softmaxes it
// (src/cpu/kernels/mod.rs:2218-2243) and accumulates P V with lanes over d.
template <typename T>
__global__ void __launch_bounds__(128) attention_kernel(AttentionParams p) {
    extern __shared__ float sm[];
    const int img = blockIdx.x / p.heads, head = blockIdx.x % p.heads;
    const int hidden = p.heads * p.d;
    const int warps = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* ks = sm;
    float* vs = ks + p.t * p.d;
    float* qs = vs + p.t * p.d;              // [warps][d]
    float* sc = qs + warps * p.d;            // [warps][t]
    const T* base = static_cast<const T*>(p.qkv) + (size_t)img * p.t * 3 * hidden;
    for (int i = threadIdx.x; i < p.t * p.d; i += blockDim.x) {
        const int r = i / p.d, j = i % p.d;
        ks[i] = to_f(base[(size_t)r * 3 * hidden + hidden + head * p.d + j]);
        vs[i] = to_f(base[(size_t)r * 3 * hidden + 2 * hidden + head * p.d + j]);
    }
    __syncthreads();
    float* q = qs + warp * p.d;
    float* s = sc + warp * p.t;
    for (int row = warp; row < p.t; row += warps) {
        for (int j = lane; j < p.d; j += 32) q[j] = to_f(base[(size_t)row * 3 * hidden + head * p.d + j]);
        __syncwarp();
        float mx = -FLT_MAX;
        for (int key = lane; key < p.t; key += 32) {
            float a = 0.f;
            for (int j = 0; j < p.d; ++j) a = fmaf(q[j], ks[key * p.d + j], a);
            a = a * p.scale;
            s[key] = a;
            mx = fmaxf(mx, a);
        }
        for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
        for (int key = lane; key < p.t; key += 32) {
            const float e = expf(s[key] - mx);
            s[key] = e;
            sum += e;
        }
        for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        const float rcp = 1.f / sum;
        __syncwarp();
        T* out = static_cast<T*>(p.out) + ((size_t)img * p.t + row) * hidden + head * p.d;
        for (int j = lane; j < p.d; j += 32) {
            float a = 0.f;
            for (int key = 0; key < p.t; ++key) a = fmaf(s[key] * rcp, vs[key * p.d + j], a);
            out[j] = from_f<T>(a);
        }
        __syncwarp();
    }
}

// Row softmax + greedy-CTC statistics.  Pass 1: max logit, runner-up logit;
// pass 2: sum of exp; pass 3: probabilities and their arg-max with the last
// index winning ties (Rust Iterator::max_by, src/ocr.rs:1171-1177).
struct ArgMax {
    float v;
    int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
    return (b.v > a.v || (b.v == a.v && b.i > a.i)) ? b : a;
}

__global__ void __launch_bounds__(256) softmax_ctc_kernel(SoftmaxParams p) {
    __shared__ float r1[8], r2[8];
    __shared__ ArgMax ra[8];
    const int row = blockIdx.x;
    const float* x = p.logits + (size_t)row * p.ld;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float m1 = -FLT_MAX, m2 = -FLT_MAX;   // top-2 logits
    for (int i = threadIdx.x; i < p.classes; i += blockDim.x) {
        const float v = x[i];
        if (v > m1) { m2 = m1; m1 = v; } else if (v > m2) { m2 = v; }
    }
    for (int o = 16; o; o >>= 1) {
        const float a1 = __shfl_xor_sync(0xffffffffu, m1, o), a2 = __shfl_xor_sync(0xffffffffu, m2, o);
        const float n1 = fmaxf(m1, a1);
        const float n2 = fmaxf(fminf(m1, a1), fmaxf(m2, a2));
        m1 = n1; m2 = n2;
    }
    if (lane == 0) { r1[warp] = m1; r2[warp] = m2; }
    __syncthreads();
    m1 = r1[0]; m2 = r2[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
        const float a1 = r1[w], a2 = r2[w];
        const float n2 = fmaxf(fminf(m1, a1), fmaxf(m2, a2));
        m1 = fmaxf(m1, a1); m2 = n2;
    }
    __syncthreads();
    float sum = 0.f;
    for (int i = threadIdx.x; i < p.classes; i += blockDim.x) sum += expf(x[i] - m1);
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) r1[warp] = sum;
    __syncthreads();
    sum = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) sum += r1[w];
    const float rcp = 1.f / sum;
    ArgMax best{-FLT_MAX, -1};
    float* prob = p.prob ? p.prob + (size_t)row * p.classes : nullptr;
    for (int i = threadIdx.x; i < p.classes; i += blockDim.x) {
        const float pr = expf(x[i] - m1) * rcp;
        if (prob) prob[i] = pr;
        best = better(best, ArgMax{pr, i});
    }
    for (int o = 16; o; o >>= 1) {
        ArgMax other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
        best = better(best, other);
    }
    if (lane == 0) ra[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        ArgMax b = ra[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) b = better(b, ra[w]);
        if (p.index) p.index[row] = b.i;
        if (p.max_prob) p.max_prob[row] = b.v;
        if (p.margin) p.margin[row] = m1 - m2;
    }
}

__device__ __forceinline__ void top2_push(float v, float& m1, float& m2) {
    if (v > m1) { m2 = m1; m1 = v; } else if (v > m2) { m2 = v; }
}

// The same statistics with the row staged in shared memory: the logits are
// read from HBM once (16-byte loads) and the probabilities written once; the
// exponentials are kept in the staged row between the sum and the write.
__global__ void __launch_bounds__(512) softmax_ctc_staged_kernel(SoftmaxParams p) {
    extern __shared__ float4 srow4[];
    float* srow = reinterpret_cast<float*>(srow4);
    __shared__ float r1[16], r2[16];
    __shared__ ArgMax ra[16];
    const int row = blockIdx.x;
    const float* x = p.logits + (size_t)row * p.ld;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    float m1 = -FLT_MAX, m2 = -FLT_MAX;
    int head = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        head = p.classes & ~3;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        for (int i = threadIdx.x; i < (head >> 2); i += blockDim.x) {
            const float4 v = __ldcs(x4 + i);
            srow4[i] = v;
            top2_push(v.x, m1, m2); top2_push(v.y, m1, m2); top2_push(v.z, m1, m2); top2_push(v.w, m1, m2);
        }
    }
    for (int i = head + threadIdx.x; i < p.classes; i += blockDim.x) {
        const float v = x[i];
        srow[i] = v;
        top2_push(v, m1, m2);
    }
    for (int o = 16; o; o >>= 1) {
        const float a1 = __shfl_xor_sync(0xffffffffu, m1, o), a2 = __shfl_xor_sync(0xffffffffu, m2, o);
        const float n1 = fmaxf(m1, a1);
        const float n2 = fmaxf(fminf(m1, a1), fmaxf(m2, a2));
        m1 = n1; m2 = n2;
    }
    if (lane == 0) { r1[warp] = m1; r2[warp] = m2; }
    __syncthreads();
    m1 = r1[0]; m2 = r2[0];
    for (int w = 1; w < nw; ++w) {
        const float a1 = r1[w], a2 = r2[w];
        const float n2 = fmaxf(fminf(m1, a1), fmaxf(m2, a2));
        m1 = fmaxf(m1, a1); m2 = n2;
    }
    __syncthreads();
    float sum = 0.f;
    for (int i = threadIdx.x; i < p.classes; i += blockDim.x) {
        const float e = expf(srow[i] - m1);
        srow[i] = e;
        sum += e;
    }
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) r1[warp] = sum;
    __syncthreads();
    sum = 0.f;
    for (int w = 0; w < nw; ++w) sum += r1[w];
    const float rcp = 1.f / sum;
    ArgMax best{-FLT_MAX, -1};
    float* prob = p.prob ? p.prob + (size_t)row * p.classes : nullptr;
    for (int i = threadIdx.x; i < p.classes; i += blockDim.x) {
        const float pr = srow[i] * rcp;
        if (prob) __stcs(prob + i, pr);
        best = better(best, ArgMax{pr, i});
    }
    for (int o = 16; o; o >>= 1) {
        ArgMax other{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
        best = better(best, other);
    }
    if (lane == 0) ra[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        ArgMax b = ra[0];
        for (int w = 1; w < nw; ++w) b = better(b, ra[w]);
        if (p.index) p.index[row] = b.i;
        if (p.max_prob) p.max_prob[row] = b.v;
        if (p.margin) p.margin[row] = m1 - m2;
    }
}

// Quad -> rectangle bilinear resample with integer rounding, BGR order and
// per-channel affine normalisation, zero past content_w
// (src/preprocess/kernels.rs:94-165, the scalar row kernel).  Explicit
// round-to-nearest intrinsics keep every product and sum separately rounded,
// as the reference's scalar code computes them (no FMA contraction).
__global__ void __launch_bounds__(256) preprocess_kernel(PreprocessParams p) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    if (x >= p.out_w || y >= p.out_h) return;
    const size_t plane = (size_t)p.out_h * p.out_w;
    const size_t o = (size_t)y * p.out_w + x;
    if (x >= p.content_w) {
        p.out[o] = 0.f;
        p.out[plane + o] = 0.f;
        p.out[2 * plane + o] = 0.f;
        return;
    }
    const float v = __fdiv_rn(__fadd_rn((float)y, 0.5f), (float)p.out_h);
    const float omv = __fsub_rn(1.f, v);
    const float u = __fdiv_rn(__fadd_rn((float)x, 0.5f), (float)p.content_w);
    const float omu = __fsub_rn(1.f, u);
    const float* c = p.corners;
    float sx = __fadd_rn(__fmul_rn(__fadd_rn(__fmul_rn(c[0], omu), __fmul_rn(c[2], u)), omv),
                         __fmul_rn(__fadd_rn(__fmul_rn(c[6], omu), __fmul_rn(c[4], u)), v));
    float sy = __fadd_rn(__fmul_rn(__fadd_rn(__fmul_rn(c[1], omu), __fmul_rn(c[3], u)), omv),
                         __fmul_rn(__fadd_rn(__fmul_rn(c[7], omu), __fmul_rn(c[5], u)), v));
    sx = fminf(fmaxf(__fsub_rn(sx, 0.5f), 0.f), (float)(p.src_w - 1));
    sy = fminf(fmaxf(__fsub_rn(sy, 0.5f), 0.f), (float)(p.src_h - 1));
    const int x0 = (int)floorf(sx), y0 = (int)floorf(sy);
    const int x1 = min(x0 + 1, p.src_w - 1), y1 = min(y0 + 1, p.src_h - 1);
    const float tx = __fsub_rn(sx, (float)x0), ty = __fsub_rn(sy, (float)y0);
    const float omtx = __fsub_rn(1.f, tx), omty = __fsub_rn(1.f, ty);
    const uint8_t* r0 = p.rgb + ((size_t)y0 * p.src_w) * 3;
    const uint8_t* r1 = p.rgb + ((size_t)y1 * p.src_w) * 3;
    float rgb[3];
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
        const float tl = r0[x0 * 3 + ch], tr = r0[x1 * 3 + ch];
        const float bl = r1[x0 * 3 + ch], br = r1[x1 * 3 + ch];
        const float top = __fadd_rn(__fmul_rn(tl, omtx), __fmul_rn(tr, tx));
        const float bottom = __fadd_rn(__fmul_rn(bl, omtx), __fmul_rn(br, tx));
        const float val = __fadd_rn(__fmul_rn(top, omty), __fmul_rn(bottom, ty));
        rgb[ch] = fminf(fmaxf(roundf(val), 0.f), 255.f);
    }
    // plane 0 = blue (rgb[2]), 1 = green, 2 = red
    p.out[o] = __fadd_rn(__fmul_rn(rgb[2], p.scale[0]), p.bias[0]);
    p.out[plane + o] = __fadd_rn(__fmul_rn(rgb[1], p.scale[1]), p.bias[1]);
    p.out[2 * plane + o] = __fadd_rn(__fmul_rn(rgb[0], p.scale[2]), p.bias[2]);
}

template <typename T>
__global__ void nchw_to_nhwc_kernel(const float* in, T* out, int n, int c, int h, int w) {
    const long long total = (long long)n * c * h * w;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int ch = (int)(i % c);
        const long long pix = i / c;
        const int x = (int)(pix % w), y = (int)((pix / w) % h), img = (int)(pix / ((long long)w * h));
        out[i] = from_f<T>(in[(((size_t)img * c + ch) * h + y) * w + x]);
    }
}

template <typename T>
__global__ void to_f32_kernel(const T* in, float* out, size_t count) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
        out[i] = to_f(in[i]);
}

__global__ void check_finite_kernel(const float* in, size_t rows, size_t cols, size_t ld, int* flag) {
    const size_t count = rows * cols;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x)
        if (!isfinite(in[(i / cols) * ld + i % cols])) { *flag = 1; return; }
}

// Copies `count` floats and raises *flag if any is not finite: the staging
// copy of the pipelined host-buffer forward, done by the SMs so it never
// queues behind the other chunks' host copies on a copy engine.
__global__ void copy_check_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t count, int* flag) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    const size_t n4 = count / 4;
    bool bad = false;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        const float4 v = __ldcs(reinterpret_cast<const float4*>(src) + i);
        bad |= !isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w);
        reinterpret_cast<float4*>(dst)[i] = v;
    }
    for (size_t i = n4 * 4 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
        const float v = src[i];
        bad |= !isfinite(v);
        dst[i] = v;
    }
    if (bad) *flag = 1;
}

__global__ void copy_words_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst, size_t count) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) dst[i] = src[i];
}

inline unsigned grid_for(long long total, int threads) {
    long long b = (total + threads - 1) / threads;
    if (b > 148LL * 32) b = 148LL * 32;
    return (unsigned)(b < 1 ? 1 : b);
}

}  // namespace

int channel_sum_chunks(int hw, int c) {
    // Pixel chunks of one image: each thread sums at least 8 pixel rows.  The
    // count depends on the image's shape only, so an image's pooled sums (and
    // everything after them) are the same bits whatever batch it runs in.
    const int cg = c / 4 > 0 ? c / 4 : 1;
    const int rows = 256 / cg > 0 ? 256 / cg : 1;
    int chunks = (hw + rows * 8 - 1) / (rows * 8);
    if (chunks > 64) chunks = 64;
    if (chunks < 1) chunks = 1;
    return chunks;
}

cudaError_t launch_channel_sum(const PoolParams& p, cudaStream_t stream) {
    if (p.c % 4 || p.c / 4 > 256 || p.chunks < 1) return cudaErrorInvalidValue;
    dim3 grid(p.chunks, p.n);
    if (p.dtype == DT_F32) channel_sum_kernel<float><<<grid, 256, 0, stream>>>(p);
    else channel_sum_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_se_mlp(const SeMlpParams& p, cudaStream_t stream) {
    if (p.c % 4 || p.n <= 0 || p.r <= 0) return cudaErrorInvalidValue;
    // Images per block: enough blocks to cover the SMs, each weight row reused IMG
    // times.  (Eight images per block, to share the recognizer's large weight
    // reads, measured twice as slow: the blocks' serial FMA chains dominate.)
    const int img = p.n <= 148 ? 1 : (p.n <= 296 ? 2 : 4);
    const size_t smem = (size_t)img * (p.c + p.r) * (p.f64 ? sizeof(double) : sizeof(float));
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    const unsigned grid = (unsigned)((p.n + img - 1) / img);
    if (p.f64) {
        if (img == 1) se_mlp_kernel<double, 1><<<grid, 256, smem, stream>>>(p);
        else if (img == 2) se_mlp_kernel<double, 2><<<grid, 256, smem, stream>>>(p);
        else se_mlp_kernel<double, 4><<<grid, 256, smem, stream>>>(p);
    } else {
        if (img == 1) se_mlp_kernel<float, 1><<<grid, 256, smem, stream>>>(p);
        else if (img == 2) se_mlp_kernel<float, 2><<<grid, 256, smem, stream>>>(p);
        else se_mlp_kernel<float, 4><<<grid, 256, smem, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_se_pool_mlp(const SePoolParams& p, cudaStream_t stream) {
    const PoolParams& q = p.pool;
    if (q.c % 4 || q.c / 4 > 256 || q.n <= 0 || q.chunks < 1 || p.mlp.r <= 0 || !p.counters) return cudaErrorInvalidValue;
    const size_t smem = (size_t)(p.mlp.c + p.mlp.r) * (p.mlp.f64 ? sizeof(double) : sizeof(float));
    if (smem > 48 * 1024) return cudaErrorInvalidValue;
    dim3 grid((unsigned)q.chunks, (unsigned)q.n);
    if (q.dtype == DT_F32) {
        if (p.mlp.f64) se_pool_mlp_kernel<float, double><<<grid, 256, smem, stream>>>(p);
        else se_pool_mlp_kernel<float, float><<<grid, 256, smem, stream>>>(p);
    } else {
        if (p.mlp.f64) se_pool_mlp_kernel<__nv_bfloat16, double><<<grid, 256, smem, stream>>>(p);
        else se_pool_mlp_kernel<__nv_bfloat16, float><<<grid, 256, smem, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_gate_apply(const GateApplyParams& p, cudaStream_t stream) {
    if (p.c % 4 || p.out_cstride % 4 || p.out_coff % 4) return cudaErrorInvalidValue;
    const long long total = (long long)p.n * p.h * p.w * (p.c / 4);
    const unsigned g = grid_for(total, 256);
    const bool narrow = total + (long long)g * 256 < 0x7fffffffLL;
    if (p.dtype == DT_F32) {
        if (narrow) gate_apply_kernel<float, uint32_t><<<g, 256, 0, stream>>>(p);
        else gate_apply_kernel<float, unsigned long long><<<g, 256, 0, stream>>>(p);
    } else {
        if (narrow) gate_apply_kernel<__nv_bfloat16, uint32_t><<<g, 256, 0, stream>>>(p);
        else gate_apply_kernel<__nv_bfloat16, unsigned long long><<<g, 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_head_t(const HeadParams& p, cudaStream_t stream) {
    const long long total = (long long)p.n * p.h * p.w;
    const unsigned g = (unsigned)((total + 127) / 128);
    const size_t smem = (size_t)(4 * p.ch * p.ch + p.ch + 4 * p.ch) * sizeof(float);
    switch (p.ch) {
        case 16: det_head_kernel<T, 16><<<g, 128, smem, stream>>>(p); break;
        case 24: det_head_kernel<T, 24><<<g, 128, smem, stream>>>(p); break;
        case 64: {
            {
                cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(det_head_kernel<T, 64>), (int)smem);
                if (e != cudaSuccess) return e;
            }
            det_head_kernel<T, 64><<<g, 128, smem, stream>>>(p);
            break;
        }
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_det_head(const HeadParams& p, cudaStream_t stream) {
    return p.dtype == DT_F32 ? launch_head_t<float>(p, stream) : launch_head_t<__nv_bfloat16>(p, stream);
}

cudaError_t launch_maxpool_same_upper(const MaxPoolParams& p, cudaStream_t stream) {
    if (p.c % 4 || p.out_cstride % 4 || p.out_coff % 4) return cudaErrorInvalidValue;
    const unsigned g = grid_for((long long)p.n * p.h * p.w * (p.c / 4), 256);
    if (p.dtype == DT_F32) maxpool_su_kernel<float><<<g, 256, 0, stream>>>(p);
    else maxpool_su_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_avgpool_3x2(const AvgPoolParams& p, cudaStream_t stream) {
    if (p.c % 4) return cudaErrorInvalidValue;
    const unsigned g = grid_for((long long)p.n * (p.h / 3) * (p.w / 2) * (p.c / 4), 256);
    if (p.dtype == DT_F32) avgpool_3x2_kernel<float><<<g, 256, 0, stream>>>(p);
    else avgpool_3x2_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_layernorm(const LayerNormParams& p, cudaStream_t stream) {
    const unsigned g = (unsigned)(((long long)p.rows * 32 + 255) / 256);
    if (p.dtype == DT_F32) layernorm_kernel<float><<<g, 256, 0, stream>>>(p);
    else layernorm_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_attention(const AttentionParams& p, cudaStream_t stream) {
    const int warps = 4;
    const size_t smem = (size_t)(2 * p.t * p.d + warps * p.d + warps * p.t) * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    {
        cudaError_t e = p.dtype == DT_F32
            ? allow_dynamic_smem(reinterpret_cast<const void*>(attention_kernel<float>), 200 * 1024)
            : allow_dynamic_smem(reinterpret_cast<const void*>(attention_kernel<__nv_bfloat16>), 200 * 1024);
        if (e != cudaSuccess) return e;
    }
    if (p.dtype == DT_F32) attention_kernel<float><<<p.n * p.heads, warps * 32, smem, stream>>>(p);
    else attention_kernel<__nv_bfloat16><<<p.n * p.heads, warps * 32, smem, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_softmax_ctc(const SoftmaxParams& in, cudaStream_t stream) {
    SoftmaxParams p = in;
    if (p.ld == 0) p.ld = p.classes;
    if (p.ld < p.classes || p.rows <= 0 || p.classes <= 0) return cudaErrorInvalidValue;
    const size_t smem = ((size_t)p.classes * sizeof(float) + 15) / 16 * 16;
    constexpr size_t kStagedMax = 200 * 1024;
    if (smem <= kStagedMax) {
        {
            cudaError_t e = allow_dynamic_smem(reinterpret_cast<const void*>(softmax_ctc_staged_kernel), (int)kStagedMax);
            if (e != cudaSuccess) return e;
        }
        softmax_ctc_staged_kernel<<<p.rows, 512, smem, stream>>>(p);
    } else {
        softmax_ctc_kernel<<<p.rows, 256, 0, stream>>>(p);
    }
    return cudaGetLastError();
}

cudaError_t launch_preprocess(const PreprocessParams& p, cudaStream_t stream) {
    dim3 grid((p.out_w + 255) / 256, p.out_h);
    preprocess_kernel<<<grid, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_nchw_to_nhwc(const float* in, void* out, int n, int c, int h, int w, DType dt, cudaStream_t stream) {
    const unsigned g = grid_for((long long)n * c * h * w, 256);
    if (dt == DT_F32) nchw_to_nhwc_kernel<float><<<g, 256, 0, stream>>>(in, static_cast<float*>(out), n, c, h, w);
    else nchw_to_nhwc_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(in, static_cast<__nv_bfloat16*>(out), n, c, h, w);
    return cudaGetLastError();
}

cudaError_t launch_to_f32(const void* in, float* out, size_t count, DType dt, cudaStream_t stream) {
    const unsigned g = grid_for((long long)count, 256);
    if (dt == DT_F32) to_f32_kernel<float><<<g, 256, 0, stream>>>(static_cast<const float*>(in), out, count);
    else to_f32_kernel<__nv_bfloat16><<<g, 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(in), out, count);
    return cudaGetLastError();
}

cudaError_t launch_check_finite_rows(const float* in, size_t rows, size_t cols, size_t ld, int* flag, cudaStream_t stream) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    const unsigned g = grid_for((long long)(rows * cols), 256);
    check_finite_kernel<<<g, 256, 0, stream>>>(in, rows, cols, ld, flag);
    return cudaGetLastError();
}

cudaError_t launch_copy_check(const float* src, float* dst, size_t count, int* flag, cudaStream_t stream) {
    if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) return cudaErrorInvalidValue;
    if (count == 0) return cudaSuccess;
    copy_check_kernel<<<grid_for((long long)(count / 4 + 1), 256), 256, 0, stream>>>(src, dst, count, flag);
    return cudaGetLastError();
}

cudaError_t launch_copy_words(const void* src, void* dst, size_t count, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    copy_words_kernel<<<grid_for((long long)count, 256), 256, 0, stream>>>(static_cast<const uint32_t*>(src),
                                                                          static_cast<uint32_t*>(dst), count);
    return cudaGetLastError();
}

cudaError_t launch_check_finite(const float* in, size_t count, int* flag, cudaStream_t stream) {
    return launch_check_finite_rows(in, 1, count, count, flag, stream);
}

}  // namespace ppocr
