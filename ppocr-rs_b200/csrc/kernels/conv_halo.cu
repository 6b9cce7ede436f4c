// Halo-tiled dense convolution on the CUDA cores: the FP32 mode's stem and
// head convs (LargeStem stem1 / stem2a / stem2b / stem3, src/cpu/model.rs:
// 626-693; the DB head's 3x3 conv_down over the upsampled neck features,
// src/cpu/model.rs:1479-1521), and the BF16 mode's where the tensor-core conv
// does not apply.
//
// out[p, o] = act(sum_{q, ky, kx, c} in[p + (ky, kx), 4q + c] * w[o, 4q + c, ky, kx] + b[o]) (+ residual)
//
// A block owns TY output rows x TW = 32 TM output columns of one image and
// G * TN output channels; a warp is 32 adjacent output columns of one row and
// one channel group, each thread TM pixels (columns lane + 32 i) x TN
// channels.  The input channels stream through shared memory one quad (four
// channels) at a time: a stage holds the quad's input tile plus halo
// (IH x IW pixels, 16 bytes per FP32 pixel quad, zero outside the image) and
// the quad's weights [tap][4][BN].  Stages are filled with cp.async NST - 1
// steps ahead (a step is one quad of one tile; blocks are persistent and the
// pipeline runs across tile boundaries), so loads overlap the arithmetic.
// Per tap a thread loads its TM pixel quads (one 16-byte load each; a warp's
// 32 loads are contiguous) and, per channel, TN weights by broadcast, and
// issues TM * TN packed two-lane FMAs (fma.rn.f32x2, each lane rounded as
// fmaf).
//
// Two summation orders.  Blocked (the default): per output the products of
// one input quad are summed in (ky, kx, channel)
// order into a fresh partial sum, each with one FMA, and the quads' partial
// sums are added in quad order (a blocked summation: its rounding error grows
// with the number of quads plus the products per quad, not with their
// product); then the bias, activation and residual are applied.  With one
// input quad (the 3-channel image) this is the plain (ky, kx, channel) sum.
// Plain (halo_order = 2): one running sum in (quad, ky, kx, channel) order,
// for convs whose rounding is not amplified downstream (fewer registers than
// blocked, so more pixels per thread).
// Tap-major (ConvParams::halo_order = 1): a stage holds the tile's input for
// every quad and each output is one running sum in (ky, kx, channel) order,
// exactly the direct kernel's, for convs whose rounding must not change.
// At stride 2 the halo tile keeps even and odd columns in separate halves, so
// the 32 lanes of a warp, reading every second input column, still read 32
// consecutive pixel quads.
// Sources: up to four NHWC views (nearest-upsampled by a power of two),
// concatenated along channels, or the NCHW FP32 image (three channel planes,
// copied row by row in 16-byte chunks into a planar tile).
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ppocr {
namespace {

constexpr int kThreads = 256;
// Summation orders (ConvParams::halo_order): per-quad partial sums, the direct
// kernel's tap-major order, or one running sum quad by quad.
constexpr int kBlocked = 0, kTapMajor = 1, kPlain = 2;
// The sums stay in registers: one running sum holds up to 48 per thread (64
// spilled under the two-blocks-per-SM register cap), partial plus running
// sums 2 x 32.
constexpr bool halo_fits(bool single, int tm, int tn) { return single ? tm * tn <= 48 : 2 * tm * tn <= 64; }
constexpr size_t kSmemLimit = 200 * 1024;

struct HaloArgs {
    int groups, ty, tw;              // channel groups, tile rows, tile columns
    int ih, iw;                      // input tile (pixels)
    int iwp;                         // NCHW image: planar row pitch in floats (iw + 3 rounded up to 4)
    int tiles_x, tiles_y, total;     // tiles per image row / column, all tiles
    int quads;                       // input channel quads (steps per tile)
    int bn;                          // padded output channels (groups * TN)
    int halo_bytes, stage_bytes;     // per stage
    int qstart[5];                   // first quad of each source
    int shift[4];                    // log2 upsampling of each source
    float inv_iw;
};

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(valid ? 8 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float4 quad_at(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 quad_at(const __nv_bfloat16* p) { return load4(p); }

template <typename T, int KH, int KW, int SH, int SW, int TN, int TM, int NST, bool NCHW, int MODE>
__global__ void __launch_bounds__(kThreads, 2) conv_halo_kernel(ConvParams p, HaloArgs a) {
    constexpr int TAPS = KH * KW;
    extern __shared__ float4 hsm[];
    char* smem = reinterpret_cast<char*>(hsm);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int wy = warp % a.ty, g = warp / a.ty;
    // Blocked mode: one step per input quad.  Tap-major mode: one step per tile,
    // every quad of the tile resident in the stage.
    constexpr bool TAPQ = MODE == kTapMajor;
    const int steps_per_tile = TAPQ ? 1 : a.quads;
    int my_tiles = 0;
    if ((int)blockIdx.x < a.total) my_tiles = (a.total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1;
    const int steps = my_tiles * steps_per_tile;
    const int per_img = a.tiles_x * a.tiles_y;

    // Shared-memory pixel slot of input tile pixel (ry, rx): row-major, with
    // the even columns of a row before its odd ones at stride 2.
    const int half_w = (a.iw + 1) / 2;
    auto slot = [&](int ry, int rx) { return SW == 2 ? ry * a.iw + (rx & 1) * half_w + (rx >> 1) : ry * a.iw + rx; };
    auto issue = [&](int step) {
        char* st = smem + (size_t)(step % NST) * a.stage_bytes;
        const int tile = (int)blockIdx.x + (step / steps_per_tile) * (int)gridDim.x;
        const int q = step % steps_per_tile;
        const int img = tile / per_img, rem = tile - img * per_img;
        const int tyi = rem / a.tiles_x, txi = rem - tyi * a.tiles_x;
        const int iy0 = tyi * a.ty * SH - p.pt, ix0 = txi * a.tw * SW - p.pl;
        const int npx = a.ih * a.iw;
        if constexpr (NCHW) {
            // Planar [3][ih][iwp]: each tile row of each channel plane is copied as
            // 16-byte chunks starting at the 4-aligned column xa <= ix0 (the image
            // width is a multiple of 4, so no chunk straddles an image edge).
            const float* base = static_cast<const float*>(p.src[0].ptr) + (size_t)img * 3 * p.hi * p.wi;
            const size_t plane = (size_t)p.hi * p.wi;
            float* dst = reinterpret_cast<float*>(st);
            const int xa = ix0 >= 0 ? ix0 & ~3 : -((-ix0 + 3) & ~3);
            const int nch = a.iwp / 4;                 // chunks per row
            const int rows = 3 * a.ih;
            for (int i = t; i < rows * nch; i += kThreads) {
                const int row = i / nch, ch = i - row * nch;
                const int c = row / a.ih, ry = row - c * a.ih;
                const int y = iy0 + ry, x = xa + ch * 4;
                const bool ok = y >= 0 && y < p.hi && x >= 0 && x < p.wi;
                const float* src = ok ? base + c * plane + (size_t)y * p.wi + x : base;
                cp_async16(dst + (size_t)row * a.iwp + ch * 4, src, ok);
            }
        } else {
            auto copy_quad = [&](int qq, T* dst) {
                // The source holding quad qq (unrolled selects keep the parameter
                // block out of local memory).
                const void* sptr = p.src[0].ptr;
                int cstride = p.src[0].cstride, coff = p.src[0].coff, q0 = a.qstart[0], sh = a.shift[0];
#pragma unroll
                for (int k = 1; k < 4; ++k)
                    if (k < p.nsrc && qq >= a.qstart[k]) {
                        sptr = p.src[k].ptr; cstride = p.src[k].cstride; coff = p.src[k].coff; q0 = a.qstart[k]; sh = a.shift[k];
                    }
                const int hs = p.hi >> sh, ws = p.wi >> sh;
                const T* base = static_cast<const T*>(sptr) + (size_t)img * hs * ws * cstride + coff + (qq - q0) * 4;
                for (int i = t; i < npx; i += kThreads) {
                    const int ry = (int)(((float)i + 0.5f) * a.inv_iw), rx = i - ry * a.iw;
                    const int y = iy0 + ry, x = ix0 + rx;
                    const bool ok = y >= 0 && y < p.hi && x >= 0 && x < p.wi;
                    const T* px = ok ? base + ((size_t)(y >> sh) * ws + (x >> sh)) * cstride : base;
                    const int d = slot(ry, rx);
                    if constexpr (sizeof(T) == 4) cp_async16(dst + d * 4, px, ok);
                    else cp_async8(dst + d * 4, px, ok);
                }
            };
            T* dst = reinterpret_cast<T*>(st);
            if constexpr (TAPQ) {
                for (int qq = 0; qq < a.quads; ++qq) copy_quad(qq, dst + (size_t)qq * npx * 4);
            } else {
                copy_quad(q, dst);
            }
        }
        const float* wsrc = p.weight + (TAPQ ? 0 : (size_t)q * TAPS * 4 * a.bn);
        float* wdst = reinterpret_cast<float*>(st + a.halo_bytes);
        const int wq = (TAPQ ? a.quads : 1) * TAPS * a.bn;   // 16-byte chunks of [quads][TAPS][4][bn] floats
        for (int i = t; i < wq; i += kThreads) cp_async16(wdst + i * 4, wsrc + i * 4, true);
    };

#pragma unroll
    for (int s = 0; s < NST - 1; ++s) {
        if (s < steps) issue(s);
        cp_async_commit();
    }
    float acc[TM][TN];
    for (int step = 0; step < steps; ++step) {
        if (step + NST - 1 < steps) issue(step + NST - 1);
        cp_async_commit();
        cp_async_wait<NST - 1>();
        __syncthreads();
        const int q = step % steps_per_tile;
        const char* st = smem + (size_t)(step % NST) * a.stage_bytes;
        const T* halo = reinterpret_cast<const T*>(st);
        const float* wt = reinterpret_cast<const float*>(st + a.halo_bytes) + g * TN;
        if constexpr (NCHW) {
            // Planar image tile: per tap, channel by channel, (ky, kx, channel) order.
            const float* pl = reinterpret_cast<const float*>(st);
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
            const int tile = (int)blockIdx.x + (step / steps_per_tile) * (int)gridDim.x;
            const int rem = tile % per_img;
            const int txi = rem % a.tiles_x;
            const int ix0 = txi * a.tw * SW - p.pl;
            const int xoff = ix0 - (ix0 >= 0 ? ix0 & ~3 : -((-ix0 + 3) & ~3));
#pragma unroll
            for (int ky = 0; ky < KH; ++ky) {
#pragma unroll
                for (int kx = 0; kx < KW; ++kx) {
                    const float* wk = wt + (size_t)((ky * KW + kx) * 4) * a.bn;
#pragma unroll
                    for (int c = 0; c < 3; ++c) {
                        const float* prow = pl + (size_t)(c * a.ih + wy * SH + ky) * a.iwp + xoff + kx + lane * SW;
                        float b[TN];
#pragma unroll
                        for (int j = 0; j < TN; j += 4) {
                            const float4 v = *reinterpret_cast<const float4*>(wk + c * a.bn + j);
                            b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
                        }
#pragma unroll
                        for (int i = 0; i < TM; ++i) {
                            const float x = prow[i * 32 * SW];
#pragma unroll
                            for (int j = 0; j < TN; j += 2) fma2(acc[i][j], acc[i][j + 1], x, x, b[j], b[j + 1]);
                        }
                    }
                }
            }
        } else if constexpr (TAPQ) {
            // The direct kernel's order: per output, taps outer, every input
            // channel (quad by quad) inner, one running sum.
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
            const int plane = a.ih * a.iw * 4;
#pragma unroll
            for (int ky = 0; ky < KH; ++ky) {
#pragma unroll
                for (int kx = 0; kx < KW; ++kx) {
                    const int col = SW == 2 ? (kx & 1) * half_w + lane + (kx >> 1) : lane + kx;
                    const T* hx0 = halo + (size_t)((wy * SH + ky) * a.iw + col) * 4;
                    for (int qq = 0; qq < a.quads; ++qq) {
                        const T* hx = hx0 + (size_t)qq * plane;
                        float4 av[TM];
#pragma unroll
                        for (int i = 0; i < TM; ++i) av[i] = quad_at(hx + (size_t)(i * 32) * 4);
                        const float* wk = wt + (size_t)((qq * TAPS + ky * KW + kx) * 4) * a.bn;
#pragma unroll
                        for (int c = 0; c < 4; ++c) {
                            float b[TN];
#pragma unroll
                            for (int j = 0; j < TN; j += 4) {
                                const float4 v = *reinterpret_cast<const float4*>(wk + c * a.bn + j);
                                b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
                            }
#pragma unroll
                            for (int i = 0; i < TM; ++i) {
                                const float x = c == 0 ? av[i].x : c == 1 ? av[i].y : c == 2 ? av[i].z : av[i].w;
#pragma unroll
                                for (int j = 0; j < TN; j += 2) fma2(acc[i][j], acc[i][j + 1], x, x, b[j], b[j + 1]);
                            }
                        }
                    }
                }
            }
        } else {
        // Blocked: this quad's products go to a fresh partial sum, added to the
        // running sum below.  Plain: straight into the running sum.
        constexpr int PM = MODE == kBlocked ? TM : 1, PN = MODE == kBlocked ? TN : 2;
        float part[PM][PN];
        if constexpr (MODE == kBlocked) {
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) part[i][j] = 0.f;
        } else if (q == 0) {
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
        }
#pragma unroll
        for (int ky = 0; ky < KH; ++ky) {
            const T* hrow = halo + (size_t)((wy * SH + ky) * a.iw) * 4;
#pragma unroll
            for (int kx = 0; kx < KW; ++kx) {
                // Column lane * SW + kx + 32 SW i of the tile row; at stride 2 its
                // slot is in the half of kx's parity.
                const T* hx = SW == 2 ? hrow + (size_t)((kx & 1) * half_w + lane + (kx >> 1)) * 4
                                      : hrow + (size_t)(lane + kx) * 4;
                float4 av[TM];
#pragma unroll
                for (int i = 0; i < TM; ++i) av[i] = quad_at(hx + (size_t)(i * 32) * 4);
                const float* wk = wt + (size_t)((ky * KW + kx) * 4) * a.bn;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float b[TN];
#pragma unroll
                    for (int j = 0; j < TN; j += 4) {
                        const float4 v = *reinterpret_cast<const float4*>(wk + c * a.bn + j);
                        b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
                    }
#pragma unroll
                    for (int i = 0; i < TM; ++i) {
                        const float x = c == 0 ? av[i].x : c == 1 ? av[i].y : c == 2 ? av[i].z : av[i].w;
                        float* d;
                        if constexpr (MODE == kBlocked) d = part[i];
                        else d = acc[i];
#pragma unroll
                        for (int j = 0; j < TN; j += 2) fma2(d[j], d[j + 1], x, x, b[j], b[j + 1]);
                    }
                }
            }
        }
        if constexpr (MODE == kBlocked) {
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = q == 0 ? part[i][j] : acc[i][j] + part[i][j];
        }
        }
        if (q == steps_per_tile - 1) {
            const int tile = (int)blockIdx.x + (step / steps_per_tile) * (int)gridDim.x;
            const int img = tile / per_img, rem = tile - img * per_img;
            const int tyi = rem / a.tiles_x, txi = rem - tyi * a.tiles_x;
            const int oy = tyi * a.ty + wy;
            const int co0 = g * TN;
            if (oy < p.ho) {
#pragma unroll
                for (int i = 0; i < TM; ++i) {
                    const int ox = txi * a.tw + lane + i * 32;
                    if (ox >= p.wo) continue;
                    T* out = static_cast<T*>(p.out) + ((size_t)(img * p.ho + oy) * p.wo + ox) * p.out_cstride + p.out_coff + co0;
                    const T* res = nullptr;
                    if (p.residual) {
                        const int rh = p.ho / p.res_scale, rw = p.wo / p.res_scale;
                        res = static_cast<const T*>(p.residual) +
                              ((size_t)(img * rh + oy / p.res_scale) * rw + ox / p.res_scale) * p.cout + co0;
                    }
#pragma unroll
                    for (int j = 0; j < TN; j += 4) {
                        if (co0 + j >= p.cout) break;
                        float4 v = make_float4(acc[i][j], acc[i][j + 1], acc[i][j + 2], acc[i][j + 3]);
                        if (p.bias) v = f4_add(v, *reinterpret_cast<const float4*>(p.bias + co0 + j));
                        v = f4_act(v, p.act);
                        if (res) v = f4_add(v, load4(res + j));
                        store4(out + j, v);
                    }
                }
            }
        }
        __syncthreads();   // the stage is refilled NST - 1 steps later
    }
    cp_async_wait<0>();
}

// Tile columns per thread (TM) and pipeline depth for one launch: the TM in
// {2, 3, 4} whose tiles waste the fewest columns, among those whose stages
// leave room for two resident blocks per SM.
struct HaloPlan {
    int tm = 0, tn = 0, nst = 0;
    HaloArgs a{};
    size_t smem = 0;
};

// Tap-major mode (the direct kernel's summation order) when the conv asks for
// it and has more than one input quad: every quad of a tile shares one stage.
inline bool halo_tapq(const ConvParams& p) { return p.halo_order == 1 && p.src[0].mode != SRC_NCHW_F32 && p.cin > 4; }

// Output channels the packed weights and the bias are padded to.  Up to 32
// channels: 8, 16 or 32, so that the channel groups of TN = 8 or 16 divide the
// block's eight warps (24 output channels run as 32, the last 8 computed and
// not stored: the small detector's head conv_down 1.35 -> 0.87 ms).  Above,
// multiples of 8 (48 channels padded to 64 measured slower than the direct
// kernel: the small recognizer's stem2b 405 -> 528 us).
inline int halo_bn(int cout) { return cout <= 8 ? 8 : cout <= 16 ? 16 : cout <= 32 ? 32 : (cout + 7) / 8 * 8; }

// Tile shape and pipeline depth for one launch.  Candidates: TN in {16, 8}
// channels per thread (G = bn / TN channel groups, TY = 8 / G rows), TM in
// {4, 3, 2, 1} pixels per thread, 3 or 2 stages.  Preferred: stages that
// leave room for two resident blocks per SM, then the least tile padding,
// then the most outputs per thread, then the deeper pipeline.
inline HaloPlan plan_halo(const ConvParams& p, int elem_bytes) {
    const bool tapq = halo_tapq(p);
    const bool nchw = p.src[0].mode == SRC_NCHW_F32;
    const int stage_quads = tapq ? p.cin / 4 : 1;
    const bool single = tapq || nchw || p.halo_order == kPlain;   // one running sum, no partial sums
    const int bn = halo_bn(p.cout);
    HaloPlan best;
    long long best_key[4] = {0, 0, 0, 0};
    for (int tn : {16, 8}) {
        if (bn % tn) continue;
        const int groups = bn / tn;
        if (groups > 8 || 8 % groups) continue;
        const int ty = 8 / groups;
        for (int tm = 4; tm >= 1; --tm) {
            if (!halo_fits(single, tm, tn)) continue;
            HaloArgs a{};
            a.groups = groups; a.ty = ty; a.tw = 32 * tm;
            a.ih = (ty - 1) * p.sh + p.kh;
            a.iw = (a.tw - 1) * p.sw + p.kw;
            a.bn = bn;
            if (nchw) {
                a.iwp = (a.iw + 3 + 3) / 4 * 4;          // room for the 0..3-column alignment offset
                a.halo_bytes = 3 * a.ih * a.iwp * 4;
            } else {
                a.halo_bytes = (stage_quads * a.ih * a.iw * 4 * elem_bytes + 15) / 16 * 16;
            }
            a.stage_bytes = a.halo_bytes + stage_quads * p.kh * p.kw * 4 * a.bn * 4;
            a.tiles_x = (p.wo + a.tw - 1) / a.tw;
            a.tiles_y = (p.ho + ty - 1) / ty;
            for (int nst = 3; nst >= 2; --nst) {
                const size_t smem = (size_t)nst * a.stage_bytes;
                if (smem > kSmemLimit) continue;
                // Tap-major with one resident block per SM measured slower than the
                // direct kernel (stem3: 384 vs 343 us): it must keep two.
                if (tapq && smem > 110 * 1024) continue;
                const long long covered = (long long)a.tiles_x * a.tw * a.tiles_y * ty;
                const long long waste_pct = (covered * 50 / ((long long)p.wo * p.ho) - 50);   // 2 % buckets
                const long long key[4] = {smem <= 110 * 1024 ? 1 : 0, -waste_pct, (long long)tm * tn, nst};
                bool better = best.tm == 0;
                for (int k = 0; k < 4 && !better; ++k) {
                    if (key[k] != best_key[k]) { better = key[k] > best_key[k]; break; }
                }
                if (!better) continue;
                for (int k = 0; k < 4; ++k) best_key[k] = key[k];
                best.tm = tm; best.tn = tn; best.nst = nst; best.a = a; best.smem = smem;
            }
        }
    }
    return best;
}

template <typename T, int KH, int KW, int SH, int SW, int TN, int TM, int NST, bool NCHW, int MODE>
cudaError_t launch_halo(const ConvParams& p, HaloArgs a, size_t smem, cudaStream_t stream) {
    auto kernel = conv_halo_kernel<T, KH, KW, SH, SW, TN, TM, NST, NCHW, MODE>;
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
    const int grid = (int)(a.total < cap ? a.total : cap);
    kernel<<<grid, kThreads, smem, stream>>>(p, a);
    return cudaGetLastError();
}

template <typename T, int KH, int KW, int SH, int SW, int TN, bool NCHW, int MODE>
cudaError_t launch_tm(const ConvParams& p, const HaloPlan& pl, cudaStream_t stream) {
#define HALO_TM(TM_, NST_)                                                                                   \
    if constexpr (halo_fits(MODE != kBlocked || NCHW, TM_, TN))                                                 \
        if (pl.tm == TM_ && pl.nst == NST_) return launch_halo<T, KH, KW, SH, SW, TN, TM_, NST_, NCHW, MODE>(p, pl.a, pl.smem, stream);
    HALO_TM(4, 3) HALO_TM(4, 2) HALO_TM(3, 3) HALO_TM(3, 2) HALO_TM(2, 3) HALO_TM(2, 2) HALO_TM(1, 3) HALO_TM(1, 2)
#undef HALO_TM
    return cudaErrorInvalidConfiguration;
}

template <typename T, int KH, int KW, int SH, int SW, bool NCHW>
cudaError_t launch_tn(const ConvParams& p, cudaStream_t stream) {
    HaloPlan pl = plan_halo(p, NCHW ? 4 : (int)sizeof(T));
    if (!pl.tm) return cudaErrorInvalidConfiguration;
    const int tn = pl.tn;
    HaloArgs& a = pl.a;
    a.quads = NCHW ? 1 : p.cin / 4;
    int q = 0;
    for (int s = 0; s < 4; ++s) {
        a.qstart[s] = q;
        a.shift[s] = 0;
        if (s < p.nsrc) {
            q += p.src[s].channels / 4;
            while ((1 << a.shift[s]) < p.src[s].scale) ++a.shift[s];
        }
    }
    a.qstart[4] = q;
    const long long total = (long long)p.n * a.tiles_x * a.tiles_y;
    if (total > 0x7fffffffLL || (long long)total * a.quads > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
    a.total = (int)total;
    a.inv_iw = 1.0f / (float)a.iw;
    if (a.total == 0) return cudaSuccess;
    if constexpr (!NCHW) {
        if (halo_tapq(p))
            return tn == 16 ? launch_tm<T, KH, KW, SH, SW, 16, NCHW, kTapMajor>(p, pl, stream)
                            : launch_tm<T, KH, KW, SH, SW, 8, NCHW, kTapMajor>(p, pl, stream);
        if (p.halo_order == kPlain)
            return tn == 16 ? launch_tm<T, KH, KW, SH, SW, 16, NCHW, kPlain>(p, pl, stream)
                            : launch_tm<T, KH, KW, SH, SW, 8, NCHW, kPlain>(p, pl, stream);
    }
    return tn == 16 ? launch_tm<T, KH, KW, SH, SW, 16, NCHW, kBlocked>(p, pl, stream)
                    : launch_tm<T, KH, KW, SH, SW, 8, NCHW, kBlocked>(p, pl, stream);
}

template <typename T>
cudaError_t launch_geom(const ConvParams& p, cudaStream_t stream) {
    const bool nchw = p.src[0].mode == SRC_NCHW_F32;
    if (p.kh == 3 && p.kw == 3 && p.sh == 1 && p.sw == 1) return launch_tn<T, 3, 3, 1, 1, false>(p, stream);
    if (p.kh == 3 && p.kw == 3 && p.sh == 2 && p.sw == 2) {
        if (nchw) {
            if constexpr (sizeof(T) == 4) return launch_tn<T, 3, 3, 2, 2, true>(p, stream);
            return cudaErrorInvalidValue;
        }
        return launch_tn<T, 3, 3, 2, 2, false>(p, stream);
    }
    if (p.kh == 2 && p.kw == 2 && p.sh == 1 && p.sw == 1) return launch_tn<T, 2, 2, 1, 1, false>(p, stream);
    return cudaErrorInvalidValue;
}

}  // namespace

int conv_halo_bn(int cout) { return halo_bn(cout); }

bool conv_halo_supported(const ConvParams& p) {
    // Output channels in whole quads (the store loop writes quads up to cout).
    if (p.cout < 4 || p.cout % 4 || p.cout > 64 || p.nsrc < 1 || p.nsrc > 4) return false;
    const bool geom = (p.kh == 3 && p.kw == 3 && ((p.sh == 1 && p.sw == 1) || (p.sh == 2 && p.sw == 2))) ||
                      (p.kh == 2 && p.kw == 2 && p.sh == 1 && p.sw == 1);
    if (!geom) return false;
    if (p.out_cstride % 4 || p.out_coff % 4) return false;
    if (p.dtype == DT_BF16 && (p.out_cstride % 4 || p.out_coff % 4)) return false;
    if (p.src[0].mode == SRC_NCHW_F32) {
        // 16-byte row chunks: the image width must keep every row 16-byte aligned.
        if (!(p.nsrc == 1 && p.cin == 3 && p.src[0].channels == 3 && p.sh == 2 && p.dtype == DT_F32 && p.wi % 4 == 0))
            return false;
        HaloPlan pl = plan_halo(p, 4);
        return pl.tm != 0;
    }
    int cin = 0;
    for (int s = 0; s < p.nsrc; ++s) {
        const ConvSource& src = p.src[s];
        if (src.mode != SRC_NHWC || src.channels % 4 || src.cstride % 4 || src.coff % 4) return false;
        if (p.dtype == DT_BF16 && (src.cstride % 4 || src.coff % 4)) return false;
        if (src.scale < 1 || (src.scale & (src.scale - 1)) || p.hi % src.scale || p.wi % src.scale) return false;
        cin += src.channels;
    }
    if (cin != p.cin) return false;
    HaloPlan pl = plan_halo(p, p.dtype == DT_F32 ? 4 : 2);
    // The float-reciprocal row division in the tile loader is exact below these.
    return pl.tm != 0 && pl.a.ih * pl.a.iw < (1 << 14) && pl.a.iw < (1 << 10);
}

cudaError_t launch_conv_halo(const ConvParams& p, cudaStream_t stream) {
    if (!conv_halo_supported(p) || !p.weight) return cudaErrorInvalidValue;
    return p.dtype == DT_F32 ? launch_geom<float>(p, stream) : launch_geom<__nv_bfloat16>(p, stream);
}

}  // namespace ppocr
