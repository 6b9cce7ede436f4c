// Graph construction.  Each builder follows the structure of the reference
// model (ppocr-rs src/cpu/model.rs, the arithmetic definition) and emits
// fused B200 kernels: BN folded into conv weights, activations / residuals /
// SE gates / nearest upsampling in kernel prologues and epilogues, and the
// neck concatenations read in place by the head conv.
#include "models.hpp"

#include <algorithm>
#include <memory>
#include <sstream>

#include "common.hpp"

namespace ppocr {

const char* size_name(int size) {
    switch (size) {
        case PPOCR_MEDIUM: return "medium";
        case PPOCR_SMALL: return "small";
        case PPOCR_TINY: return "tiny";
        default: return "unknown";
    }
}

namespace {

struct Blk {
    int cin, cout, sh, sw;
    bool se;
    bool residual() const { return cin == cout && sh == 1 && sw == 1; }   // src/cpu/model.rs:528
};

std::vector<std::vector<Blk>> detector_stages(int s1, int s2, int s3, int s4) {
    // src/cpu/model.rs:1648-1680
    return {
        {{s1, s1, 1, 1, true}, {s1, s1, 1, 1, false}},
        {{s1, s2, 2, 2, false}, {s2, s2, 1, 1, true}, {s2, s2, 1, 1, false}},
        {{s2, s3, 2, 2, false}, {s3, s3, 1, 1, true}, {s3, s3, 1, 1, false}, {s3, s3, 1, 1, true}, {s3, s3, 1, 1, false}},
        {{s3, s4, 2, 2, false}, {s4, s4, 1, 1, true}, {s4, s4, 1, 1, false}},
    };
}

std::vector<std::vector<Blk>> recognizer_stages(int size) {
    // src/cpu/model.rs:2057-2122
    if (size == PPOCR_MEDIUM || size == PPOCR_SMALL) {
        const bool med = size == PPOCR_MEDIUM;
        const int a = med ? 128 : 96, b = med ? 256 : 96, c = med ? 512 : 192, d = med ? 768 : 384;
        std::vector<Blk> st3 = {{b, c, 2, 1, false}};
        for (int i = 0; i < 6; ++i) st3.push_back({c, c, 1, 1, i % 2 == 0});
        return {
            {{a, a, 1, 1, true}},
            med ? std::vector<Blk>{{a, b, 1, 1, false}, {b, b, 1, 1, false}, {b, b, 1, 1, true}}
                : std::vector<Blk>{{a, b, 1, 1, false}, {b, b, 1, 1, false}},
            st3,
            {{c, d, 2, 1, false}, {d, d, 1, 1, true}, {d, d, 1, 1, false}},
        };
    }
    return {
        {{48, 48, 1, 1, true}},
        {{48, 48, 1, 1, false}},
        {{48, 96, 2, 1, false}, {96, 96, 1, 1, true}, {96, 96, 1, 1, false}},
        {{96, 160, 2, 1, false}, {160, 160, 1, 1, true}, {160, 160, 1, 1, false}, {160, 160, 1, 1, false}},
    };
}

inline int out_size(int in, int k, int s, int pa, int pb) { return (in + pa + pb - k) / s + 1; }

struct Src {
    int tid;
    int channels, cstride, coff, scale, mode;
};

// Activation: tensor id + NHWC shape (tight).
struct Act4 {
    int tid = -1;
    int n = 0, h = 0, w = 0, c = 0;
};

struct GemmOpts {
    int act = ACT_NONE;
    int gate = -1;            // SE gate on A: FP32 [images][k]
    int res_gate = -1;        // SE gate on the residual: FP32 [images][n]
    int rows_per_image = 1;
    int residual = -1;
    int res_scale = 1, h = 1, w = 1;
    bool c_f32 = false;
    bool has_bias = true;
    int ldc = 0;              // output row stride (0: cout)
};

class Builder {
public:
    Builder(BuiltModel& m, const WeightReader& r, int tc_mode) : m_(m), r_(r), tc_(tc_mode != TC_NONE), all_(tc_mode == TC_ALL) {}
    const WeightReader& reader() const { return r_; }
    // BF16 storage with tcgen05 GEMMs: SE gates are applied by a gate kernel
    // instead of in the GEMM's A load (the tensor-core path reads A by TMA).
    bool tensor_core_gemms() const { return tc_ && m_.dtype == DT_BF16; }
    // FP32 storage, pointwise convs on tcgen05 as split GEMMs (three-piece
    // BF16 operands, gemm_split.cu).
    bool split_gemms() const { return tc_ && m_.dtype == DT_F32; }
    // FP32 storage with the dense convs (and GEMMs the split kernel does not
    // cover) on the tensor-core engine (tc_engine.cu, planes 3).
    bool tensor_core_f32() const { return all_ && m_.dtype == DT_F32; }
    int engine_planes() const { return m_.dtype == DT_BF16 ? 1 : 3; }

    // Emits a tc_engine op.  srcs empty: dense rows of `a_tid` (mode 0);
    // otherwise the conv window over the sources (mode 1, geometry in `g`).
    void engine_op(const std::string& name, const ConvWeight& cw, TcEngineParams p, const std::vector<Src>& srcs,
                   int a_tid, int gate, int residual, int out_tid, double flops) {
        const int planes = engine_planes();
        const int bn = tc_engine_tile_n(cw.cout, planes);
        p.planes = planes;
        p.n = cw.cout;
        p.k = cw.kh * cw.kw * cw.cin;
        p.n_pad = (cw.cout + bn - 1) / bn * bn;
        p.k_pad = (p.k + 63) / 64 * 64;
        const size_t woff = m_.blob.add_bf16(pack_engine_kn(cw, planes, p.n_pad, p.k_pad));
        const size_t boff = m_.blob.add_f32(cw.b);
        std::vector<int> reads = {a_tid, gate, residual};
        for (auto& s : srcs) reads.push_back(s.tid);
        std::vector<Src> s2 = srcs;
        m_.plan.add_op(name, reads, {out_tid},
                       [p, s2, woff, boff, a_tid, gate, residual, out_tid](const Ctx& c, cudaStream_t st) mutable {
                           for (size_t i = 0; i < s2.size(); ++i) p.conv.src[i].ptr = c.act(s2[i].tid);
                           p.w = c.wb(woff);
                           p.bias = c.wf(boff);
                           p.a = c.act(a_tid);
                           p.gate = gate >= 0 ? static_cast<const float*>(c.act(gate)) : nullptr;
                           p.residual = c.act(residual);
                           p.c = c.act(out_tid);
                           p.err = c.err;
                           return launch_tc_engine(p, st);
                       },
                       srcs.empty() ? "gemm" : "conv", (double)planes * p.n_pad * p.k_pad * 2, flops);
    }

    // Concurrent regions of the plan (graph.hpp): ops added in lane 1 between
    // begin_region and end_region run on the side stream beside the lane-0 ops.
    void begin_region() { m_.plan.begin_region(); }
    void lane(int l) { m_.plan.set_lane(l); }
    void end_region() { m_.plan.end_region(); }

    Act4 tensor(const std::string& name, int n, int h, int w, int c) {
        Act4 a;
        a.tid = m_.plan.add_tensor(name, n, h, w, c, m_.dtype);
        a.n = n; a.h = h; a.w = w; a.c = c;
        return a;
    }

    // Dense conv over up to four concatenated sources (conv.cu).
    // `into` (optional): write into channels [into_coff, into_coff + cout) of an
    // existing wider tensor instead of a new one (a concatenation slice).
    // `any_order`: the conv may sum its products input quad by quad (the
    // halo-tiled kernel) rather than tap by tap.  Kept to convs whose rounding
    // differences reach the output unamplified (the detector head).
    Act4 conv(const std::string& name, const ConvWeight& cw, const std::vector<Src>& srcs, int n, int hi, int wi, int sh,
              int sw, int pt, int pl, int pb, int pr, int act, int residual = -1, int res_scale = 1,
              const Act4* into = nullptr, int into_coff = 0, bool any_order = false) {
        int cin = 0;
        for (auto& s : srcs) cin += s.channels;
        if (cin != cw.cin) fail(PPOCR_ERR_INVALID_MODEL, name + ": conv input channels do not match the weight");
        const int ho = out_size(hi, cw.kh, sh, pt, pb), wo = out_size(wi, cw.kw, sw, pl, pr);
        if (into && (into->n != n || into->h != ho || into->w != wo || into_coff % 4 || into_coff + cw.cout > into->c))
            fail(PPOCR_ERR_INVALID_MODEL, name + ": concatenation slice does not fit");
        Act4 out = into ? *into : tensor(name, n, ho, wo, cw.cout);
        const int out_cstride = into ? into->c : cw.cout, out_coff = into ? into_coff : 0;
        if (split_gemms() && srcs.size() == 1 && srcs[0].mode == SRC_NHWC && srcs[0].scale == 1 && srcs[0].coff == 0 &&
            (residual < 0 || res_scale == 1) && sh == sw) {
            // FP32 mode: a dense conv over one plain NHWC source as an implicit
            // split GEMM on tcgen05 (strided TMA boxes per tap; each tap's
            // channels padded with zeros to 32 or a multiple of 64).
            const int cpt = gemm_split_conv_cpt(cin);
            SplitGemmParams sp;
            sp.conv = 1;
            sp.n_img = n; sp.hi = hi; sp.wi = wi; sp.ho = ho; sp.wo = wo; sp.kh = cw.kh; sp.kw = cw.kw;
            sp.stride = sh; sp.pt = pt; sp.pl = pl;
            sp.k = cw.kh * cw.kw * cpt; sp.cin = cin; sp.n = cw.cout; sp.lda = srcs[0].cstride;
            sp.ldc = out_cstride; sp.coff = out_coff; sp.act = act;
            if (residual >= 0) {
                sp.residual = reinterpret_cast<const float*>(1);   // placeholder for the support check
                sp.ldr = cw.cout;
            }
            const int bn = gemm_split_tile_n(cw.cout, sp.k);
            sp.n_pad = bn > 0 ? (cw.cout + bn - 1) / bn * bn : 0;
            sp.k_pad = (sp.k + 63) / 64 * 64;
            sp.m = n * ((ho + 7) / 8) * ((wo + 15) / 16) * 128;
            if (cpt > 0 && gemm_split_supported(sp)) {
                const size_t woff = m_.blob.add_bf16(pack_engine_kn(cw, 3, sp.n_pad, sp.k_pad, cpt));
                const size_t boff = m_.blob.add_f32(cw.b);
                const int stid = srcs[0].tid, otid = out.tid;
                m_.plan.add_op(name, {stid, residual}, {otid}, [sp, woff, boff, stid, otid, residual](const Ctx& c, cudaStream_t st) mutable {
                    sp.a = static_cast<const float*>(c.act(stid));
                    sp.residual = residual >= 0 ? static_cast<const float*>(c.act(residual)) : nullptr;
                    sp.w = c.wb(woff);
                    sp.bias = c.wf(boff);
                    sp.c = static_cast<float*>(c.act(otid));
                    sp.err = c.err;
                    return launch_gemm_split(sp, st);
                }, "conv", (double)3 * sp.n_pad * sp.k_pad * 2, 2.0 * n * ho * wo * cw.cout * cin * cw.kh * cw.kw);
                return out;
            }
        }
        if (tensor_core_f32()) {
            // FP32_TC: the tensor-core engine for NHWC sources whose channels split
            // into 16-byte chunks.  (BF16 convs stay on the register-tiled SIMT
            // implicit GEMM, which measured faster than the engine's gather.)
            TcEngineParams tp;
            tp.mode = 1;
            tp.planes = engine_planes();
            tp.m = n * ho * wo;
            ConvGather& g = tp.conv;
            g.hi = hi; g.wi = wi; g.ho = ho; g.wo = wo; g.cin = cin; g.kh = cw.kh; g.kw = cw.kw;
            g.sh = sh; g.sw = sw; g.pt = pt; g.pl = pl; g.nsrc = (int)srcs.size();
            for (size_t i = 0; i < srcs.size(); ++i) {
                g.src[i].channels = srcs[i].channels; g.src[i].cstride = srcs[i].cstride; g.src[i].coff = srcs[i].coff;
                g.src[i].scale = srcs[i].scale; g.src[i].mode = srcs[i].mode;
            }
            tp.act = act;
            tp.ldr = cw.cout;
            tp.res_scale = res_scale;
            tp.out_h = ho; tp.out_w = wo;
            tp.ldc = out_cstride;
            tp.coff = out_coff;
            tp.k = cw.kh * cw.kw * cin;
            tp.k_pad = (tp.k + 63) / 64 * 64;
            tp.n = cw.cout;
            tp.w = tp.c = reinterpret_cast<void*>(1);   // placeholders for the support check
            if (tc_engine_supported(tp)) {
                engine_op(name, cw, tp, srcs, -1, -1, residual, out.tid, 2.0 * n * ho * wo * cw.cout * cin * cw.kh * cw.kw);
                return out;
            }
        }
        ConvParams p;
        p.n = n; p.hi = hi; p.wi = wi; p.cin = cin; p.nsrc = (int)srcs.size();
        p.ho = ho; p.wo = wo; p.cout = cw.cout;
        p.kh = cw.kh; p.kw = cw.kw; p.sh = sh; p.sw = sw; p.pt = pt; p.pl = pl;
        p.act = act; p.res_scale = res_scale; p.out_cstride = out_cstride; p.out_coff = out_coff; p.dtype = m_.dtype;
        std::vector<int> reads;
        for (size_t i = 0; i < srcs.size(); ++i) {
            p.src[i].channels = srcs[i].channels; p.src[i].cstride = srcs[i].cstride; p.src[i].coff = srcs[i].coff;
            p.src[i].scale = srcs[i].scale; p.src[i].mode = srcs[i].mode;
            reads.push_back(srcs[i].tid);
        }
        reads.push_back(residual);
        // BF16 with tensor cores: one plain NHWC source -> tcgen05 implicit GEMM
        // (TMA boxes per tap); other BF16 convs with NHWC sources -> the
        // register-tiled SIMT implicit GEMM (gemm_simt.cu).
        // FP32: the halo-tiled kernel (conv_halo.cu) where its geometries apply:
        // blocked per-quad sums where any order is allowed (the detector head),
        // else its tap-major mode, which keeps the direct kernel's (ky, kx,
        // channel) order and needs the tile's whole input in one stage (the
        // image stem, stem2a/2b).  Elsewhere the direct kernel (conv.cu), 16
        // output channels per thread when cout >= 16 (8 otherwise).  The
        // detector's chaotic spec-weight parity check flipped a pixel when the
        // stem and neck convs were re-associated, so those keep the tap-major
        // order.
        const bool tcconv = tc_ && m_.dtype == DT_BF16 && residual < 0 && conv_tc_supported(p);
        p.halo_order = any_order ? 2 : 1;
        const bool halo = !tcconv && m_.dtype == DT_F32 && conv_halo_supported(p);
        const bool gemm = !tcconv && !halo && m_.dtype == DT_BF16 && conv_gemm_supported(p);
        // The NCHW image input has 3 channels: one thread covers up to 64 output
        // channels so each loaded input feeds 64 FMAs.
        const bool image_src = srcs.size() == 1 && srcs[0].mode == SRC_NCHW_F32;
        const int co_tile = image_src && cw.cout % 64 == 0 ? 64 : image_src && cw.cout % 32 == 0 ? 32 : cw.cout >= 16 ? 16 : 8;
        int n_pad = 0;
        size_t woff;
        if (tcconv) {
            p.tc_n_pad = (cw.cout + 15) / 16 * 16;
            p.tc_cin_pad = (cin + 63) / 64 * 64;
            woff = m_.blob.add_bf16(pack_conv_tc(cw, p.tc_n_pad, p.tc_cin_pad));
        } else if (halo) {
            woff = m_.blob.add_f32(pack_conv_halo(cw, conv_halo_bn(cw.cout)));
            p.halo = 1;
        } else {
            woff = gemm ? m_.blob.add_f32(pack_conv_kn(cw, n_pad)) : m_.blob.add_f32(pack_conv_tiles(cw, co_tile));
        }
        std::vector<float> bias = cw.b;
        bias.resize(std::max((cw.cout + co_tile - 1) / co_tile * co_tile, conv_halo_bn(cw.cout)), 0.f);
        const size_t boff = m_.blob.add_f32(bias);
        p.co_tile = co_tile;
        p.n_pad = n_pad;
        const int otid = out.tid;
        std::vector<Src> s2 = srcs;
        m_.plan.add_op(name, reads, {otid}, [p, s2, woff, boff, residual, otid, gemm, tcconv](const Ctx& c, cudaStream_t st) mutable {
            for (size_t i = 0; i < s2.size(); ++i) p.src[i].ptr = c.act(s2[i].tid);
            p.weight = (gemm || tcconv) ? nullptr : c.wf(woff);
            p.weight_kn = gemm ? c.wf(woff) : nullptr;
            p.w_tc = tcconv ? c.wb(woff) : nullptr;
            p.bias = c.wf(boff);
            p.residual = c.act(residual);
            p.out = c.act(otid);
            p.err = c.err;
            return launch_conv(p, st);
        }, "conv", (double)cw.w.size() * 4, 2.0 * n * ho * wo * cw.cout * cin * cw.kh * cw.kw);
        return out;
    }

    Act4 conv1(const std::string& name, const ConvWeight& cw, const Act4& in, int sh, int sw, int pt, int pl, int pb, int pr,
               int act, int residual = -1, int res_scale = 1, const Act4* into = nullptr, int into_coff = 0) {
        return conv(name, cw, {{in.tid, in.c, in.c, 0, 1, SRC_NHWC}}, in.n, in.h, in.w, sh, sw, pt, pl, pb, pr, act, residual,
                    res_scale, into, into_coff);
    }

    // 2x2 stride-1 "same-upper" max pool of `x` into channels [coff, coff + x.c) of `into`.
    void maxpool_into(const std::string& name, const Act4& x, const Act4& into, int coff) {
        MaxPoolParams p;
        p.n = x.n; p.h = x.h; p.w = x.w; p.c = x.c; p.out_cstride = into.c; p.out_coff = coff; p.dtype = m_.dtype;
        const int xt = x.tid, ot = into.tid;
        m_.plan.add_op(name, {xt}, {ot}, [p, xt, ot](const Ctx& c, cudaStream_t st) mutable {
            p.in = c.act(xt);
            p.out = c.act(ot);
            return launch_maxpool_same_upper(p, st);
        }, "pool", 0, 3.0 * x.n * x.h * x.w * x.c);
    }

    // Depthwise conv (dwconv.cu).  cw is [C, 1, kh, kw].
    Act4 dwconv(const std::string& name, const ConvWeight& cw, const Act4& in, int sh, int sw, int pt, int pl, int pb, int pr,
                int act, bool has_bias, int residual = -1) {
        if (cw.cout != in.c || cw.cin != 1) fail(PPOCR_ERR_INVALID_MODEL, name + ": depthwise weight does not match its input");
        const int ho = out_size(in.h, cw.kh, sh, pt, pb), wo = out_size(in.w, cw.kw, sw, pl, pr);
        Act4 out = tensor(name, in.n, ho, wo, in.c);
        const size_t woff = m_.blob.add_f32(pack_depthwise(cw));
        const size_t boff = m_.blob.add_f32(cw.b);
        DwParams p;
        p.n = in.n; p.hi = in.h; p.wi = in.w; p.c = in.c; p.in_cstride = in.c; p.in_coff = 0;
        p.ho = ho; p.wo = wo; p.kh = cw.kh; p.kw = cw.kw; p.sh = sh; p.sw = sw; p.pt = pt; p.pl = pl;
        p.act = act; p.dtype = m_.dtype;
        const int itid = in.tid, otid = out.tid;
        m_.plan.add_op(name, {itid, residual}, {otid}, [p, woff, boff, has_bias, itid, otid, residual](const Ctx& c, cudaStream_t st) mutable {
            p.in = c.act(itid);
            p.weight = c.wf(woff);
            p.bias = has_bias ? c.wf(boff) : nullptr;
            p.residual = c.act(residual);
            p.out = c.act(otid);
            return launch_dwconv(p, st);
        }, "dwconv", (double)cw.w.size() * 4, 2.0 * in.n * ho * wo * in.c * cw.kh * cw.kw);
        return out;
    }

    // FP32 operands on tcgen05 through the split GEMM (gemm_split.cu): A split
    // into three BF16 pieces in shared memory, the SE gate applied there.  The
    // tensor core rounds its FP32 accumulator once per 16-wide K step, toward
    // zero, so the kernel sums at most K = 320 into one accumulator and adds
    // longer sums' partial accumulators in the epilogue (K up to 1,792 on the
    // medium detector).
    bool split_gemm_ok(int k, int n) const {
        if (!split_gemms()) return false;
        SplitGemmParams p;
        p.m = 1; p.n = n; p.k = k; p.lda = k; p.ldc = n;
        const int bn = gemm_split_tile_n(n, k);
        if (bn <= 0) return false;
        p.n_pad = (n + bn - 1) / bn * bn;
        p.k_pad = (k + 63) / 64 * 64;
        return gemm_split_supported(p);
    }

    void split_gemm(const std::string& name, const ConvWeight& cw, int in_tid, int rows, const GemmOpts& o, int out_tid) {
        const int k = cw.cin * cw.kh * cw.kw;
        ConvWeight flat = cw;
        flat.cin = k; flat.kh = 1; flat.kw = 1;
        SplitGemmParams p;
        p.m = rows; p.n = cw.cout; p.k = k; p.lda = k;
        const int bn = gemm_split_tile_n(cw.cout, k);
        p.n_pad = (cw.cout + bn - 1) / bn * bn;
        p.k_pad = (k + 63) / 64 * 64;
        p.rows_per_image = o.rows_per_image;
        p.act = o.act;
        p.ldr = cw.cout;
        p.res_scale = o.res_scale; p.out_h = o.h; p.out_w = o.w;
        p.ldc = o.ldc ? o.ldc : cw.cout;
        const size_t woff = m_.blob.add_bf16(pack_engine_kn(flat, 3, p.n_pad, p.k_pad));
        const size_t boff = m_.blob.add_f32(cw.b);
        const bool has_bias = o.has_bias;
        const int gate = o.gate, res_gate = o.res_gate, residual = o.residual;
        // Many N tiles: A is split into its three BF16 pieces once, by its own
        // op, instead of once per N tile inside the GEMM (same pieces, same C).
        int planes = -1;
        if (gemm_split_presplit_pays(rows, cw.cout, k)) {
            planes = m_.plan.add_raw(name + ".planes", (size_t)6 * rows * p.k_pad);
            m_.plan.add_op(name + ".split", {in_tid, gate}, {planes}, [p, in_tid, gate, planes](const Ctx& c, cudaStream_t st) mutable {
                p.a = static_cast<const float*>(c.act(in_tid));
                p.gate = gate >= 0 ? static_cast<const float*>(c.act(gate)) : nullptr;
                return launch_split_planes(p, c.act(planes), st);
            }, "gemm", 0, 0.0);
        }
        const std::vector<int> reads = planes >= 0 ? std::vector<int>{planes, res_gate, residual}
                                                   : std::vector<int>{in_tid, gate, res_gate, residual};
        m_.plan.add_op(name, reads, {out_tid},
                       [p, woff, boff, has_bias, in_tid, gate, res_gate, residual, out_tid, planes](const Ctx& c, cudaStream_t st) mutable {
                           p.a = planes >= 0 ? nullptr : static_cast<const float*>(c.act(in_tid));
                           p.a_planes = planes >= 0 ? c.act(planes) : nullptr;
                           p.w = c.wb(woff);
                           p.bias = has_bias ? c.wf(boff) : nullptr;
                           p.gate = (gate >= 0 && planes < 0) ? static_cast<const float*>(c.act(gate)) : nullptr;
                           p.res_gate = res_gate >= 0 ? static_cast<const float*>(c.act(res_gate)) : nullptr;
                           p.residual = static_cast<const float*>(c.act(residual));
                           p.c = static_cast<float*>(c.act(out_tid));
                           p.err = c.err;
                           return launch_gemm_split(p, st);
                       },
                       "gemm", (double)3 * p.n_pad * p.k_pad * 2, 2.0 * rows * cw.cout * k);
    }

    // Pointwise conv / linear over `rows` rows of `in` (gemm_simt.cu / tcgen05 GEMM).
    void gemm_rows(const std::string& name, const ConvWeight& cw, int in_tid, int rows, const GemmOpts& o, int out_tid) {
        const int k = cw.cin * cw.kh * cw.kw;
        if (split_gemm_ok(k, cw.cout)) {
            split_gemm(name, cw, in_tid, rows, o, out_tid);
            return;
        }
        if (tensor_core_f32() && k % 4 == 0 && o.res_gate < 0) {
            TcEngineParams tp;
            tp.mode = 0;
            tp.m = rows;
            tp.lda = k;
            tp.rows_per_image = o.rows_per_image;
            tp.act = o.act;
            tp.ldr = cw.cout;
            tp.res_scale = o.res_scale;
            tp.out_h = o.h; tp.out_w = o.w;
            tp.ldc = o.ldc ? o.ldc : cw.cout;
            ConvWeight flat = cw;
            flat.cin = k; flat.kh = 1; flat.kw = 1;
            if (!o.has_bias) flat.b.assign(cw.cout, 0.f);
            engine_op(name, flat, tp, {}, in_tid, o.gate, o.residual, out_tid, 2.0 * rows * cw.cout * k);
            return;
        }
        int n_pad = 0;
        const size_t woff = m_.blob.add_f32(pack_gemm_kn(cw, n_pad));
        const size_t boff = m_.blob.add_f32(cw.b);
        GemmParams p;
        p.m = rows; p.n = cw.cout; p.k = k; p.lda = k; p.n_pad = n_pad;
        p.rows_per_image = o.rows_per_image; p.act = o.act; p.ldr = cw.cout;
        p.res_scale = o.res_scale; p.h = o.h; p.w_px = o.w; p.ldc = o.ldc ? o.ldc : cw.cout; p.coff = 0; p.dtype = m_.dtype;
        p.c_f32 = o.c_f32 ? 1 : 0;
        const bool tc = tc_ && m_.dtype == DT_BF16;
        size_t tcoff = 0;
        if (tc) {
            const int np = (cw.cout + 15) / 16 * 16, kp = (k + 63) / 64 * 64;
            tcoff = m_.blob.add_bf16(pack_gemm_nk(cw, np, kp));
            p.k_pad = kp;
        }
        const int gate = o.gate, res_gate = o.res_gate, residual = o.residual;
        const bool has_bias = o.has_bias;
        m_.plan.add_op(name, {in_tid, gate, res_gate, residual}, {out_tid},
                       [p, woff, boff, tcoff, tc, has_bias, in_tid, gate, res_gate, residual, out_tid](const Ctx& c, cudaStream_t st) mutable {
                           p.a = c.act(in_tid);
                           p.w = c.wf(woff);
                           p.w_tc = tc ? c.wb(tcoff) : nullptr;
                           p.bias = has_bias ? c.wf(boff) : nullptr;
                           p.gate = gate >= 0 ? static_cast<const float*>(c.act(gate)) : nullptr;
                           p.res_gate = res_gate >= 0 ? static_cast<const float*>(c.act(res_gate)) : nullptr;
                           p.residual = c.act(residual);
                           p.c = c.act(out_tid);
                           p.err = c.err;
                           return launch_gemm(p, st);
                       },
                       "gemm", (double)k * cw.cout * (tc ? 2 : 4), 2.0 * rows * cw.cout * k);
    }

    Act4 pointwise(const std::string& name, const ConvWeight& cw, const Act4& in, GemmOpts o) {
        if (cw.cin != in.c) fail(PPOCR_ERR_INVALID_MODEL, name + ": pointwise weight does not match its input");
        Act4 out = tensor(name, in.n, in.h, in.w, cw.cout);
        o.rows_per_image = in.h * in.w;
        o.h = in.h; o.w = in.w;
        gemm_rows(name, cw, in.tid, in.n * in.h * in.w, o, out.tid);
        return out;
    }

    // Fused LCNet channel pair (rowgemm.cu) where its register tile fits.
    // The fused SIMT pair serves the CUDA-core mode only: with tcgen05 GEMMs
    // (BF16, FP32_TC) the pair runs as two tensor-core GEMMs.
    bool pair_rows_ok(int c_in, int c_out) const { return !tc_ && pair_rows_supported(c_in, c_out); }

    Act4 pair(const std::string& name, const ConvWeight& pw1, const ConvWeight& pw2, const Act4& x, int gate, bool residual) {
        const int c = pw1.cin, h = pw1.cout, co = pw2.cout;
        if (pw2.cin != h || x.c != c || (residual && co != c)) fail(PPOCR_ERR_INVALID_MODEL, name + ": pair weights do not match");
        Act4 out = tensor(name, x.n, x.h, x.w, co);
        std::vector<float> w2t((size_t)h * co);
        for (int o = 0; o < co; ++o)
            for (int j = 0; j < h; ++j) w2t[(size_t)j * co + o] = pw2.w[(size_t)o * h + j];
        const size_t o1 = m_.blob.add_f32(pw1.w), o2 = m_.blob.add_f32(w2t);
        const size_t ob1 = m_.blob.add_f32(pw1.b), ob2 = m_.blob.add_f32(pw2.b);
        PairRowsParams p;
        p.m = (long long)x.n * x.h * x.w;
        p.c_in = c; p.c_out = co; p.rows_per_image = x.h * x.w; p.residual = residual ? 1 : 0; p.dtype = m_.dtype;
        const int xt = x.tid, ot = out.tid;
        m_.plan.add_op(name, {xt, gate}, {ot}, [p, o1, o2, ob1, ob2, xt, gate, ot](const Ctx& ctx, cudaStream_t st) mutable {
            p.a = ctx.act(xt);
            p.gate = gate >= 0 ? static_cast<const float*>(ctx.act(gate)) : nullptr;
            p.w1t = ctx.wf(o1); p.w2 = ctx.wf(o2); p.b1 = ctx.wf(ob1); p.b2 = ctx.wf(ob2);
            p.c = ctx.act(ot);
            return launch_pair_rows(p, st);
        }, "gemm", (double)(pw1.w.size() + w2t.size()) * 4, 2.0 * p.m * ((double)c * h + (double)h * co));
        return out;
    }

    // SE gate of `x` (channel_sum + se_mlp); returns an FP32 [n][c] tensor id.
    int se_gate(const std::string& name, const Act4& x, const ConvWeight& reduce, const ConvWeight& expand, float alpha) {
        const int n = x.n, c = x.c, hw = x.h * x.w, r = reduce.cout, xt = x.tid;
        const int chunks = channel_sum_chunks(hw, c);
        const int sum = m_.plan.add_raw(name + ".sum", (size_t)n * chunks * c * 4);
        const int gate = m_.plan.add_raw(name + ".gate", (size_t)n * c * 4);
        const size_t w1 = m_.blob.add_f32(reduce.w), b1 = m_.blob.add_f32(reduce.b);
        const size_t w2 = m_.blob.add_f32(expand.w), b2 = m_.blob.add_f32(expand.b);
        const DType dt = m_.dtype;
        const int f64 = dt == DT_F32 ? 1 : 0;
        const double mlp_bytes = (double)(reduce.w.size() + expand.w.size()) * 4;
        if ((double)n * mlp_bytes > 8e6) {
            // Large batches of wide SE blocks (the recognizers at batch 256): a
            // separate MLP launch in which each block serves several images and
            // streams the weights once for them.
            m_.plan.add_op(name + ".pool", {xt}, {sum}, [n, c, hw, chunks, xt, sum, dt](const Ctx& ctx, cudaStream_t st) {
                PoolParams p;
                p.n = n; p.hw = hw; p.c = c; p.in = ctx.act(xt); p.in_cstride = c; p.chunks = chunks;
                p.sum = static_cast<float*>(ctx.act(sum)); p.dtype = dt;
                return launch_channel_sum(p, st);
            }, "se.pool", 0, (double)n * hw * c);
            m_.plan.add_op(name + ".mlp", {sum}, {gate}, [n, c, r, hw, chunks, sum, gate, w1, b1, w2, b2, alpha, f64](const Ctx& ctx, cudaStream_t st) {
                SeMlpParams p;
                p.n = n; p.c = c; p.r = r; p.hw = hw; p.chunks = chunks;
                p.sum = static_cast<const float*>(ctx.act(sum));
                p.w1 = ctx.wf(w1); p.b1 = ctx.wf(b1); p.w2 = ctx.wf(w2); p.b2 = ctx.wf(b2);
                p.alpha = alpha;
                p.gate = static_cast<float*>(ctx.act(gate));
                p.f64 = f64;
                return launch_se_mlp(p, st);
            }, "se.mlp", mlp_bytes, 4.0 * n * c * r);
            return gate;
        }
        // One launch: chunk sums, then the MLP in each image's last block.
        const int slot = m_.counter_slots;
        m_.counter_slots += n;
        m_.plan.add_op(name + ".pool", {xt}, {sum, gate},
                       [n, c, r, hw, chunks, xt, sum, gate, w1, b1, w2, b2, alpha, f64, dt, slot](const Ctx& ctx, cudaStream_t st) {
            SePoolParams sp;
            PoolParams& p = sp.pool;
            p.n = n; p.hw = hw; p.c = c; p.in = ctx.act(xt); p.in_cstride = c; p.chunks = chunks;
            p.sum = static_cast<float*>(ctx.act(sum)); p.dtype = dt;
            SeMlpParams& q = sp.mlp;
            q.n = n; q.c = c; q.r = r; q.hw = hw; q.chunks = chunks;
            q.sum = p.sum;
            q.w1 = ctx.wf(w1); q.b1 = ctx.wf(b1); q.w2 = ctx.wf(w2); q.b2 = ctx.wf(b2);
            q.alpha = alpha;
            q.gate = static_cast<float*>(ctx.act(gate));
            q.f64 = f64;
            sp.counters = ctx.counters + slot;
            return launch_se_pool_mlp(sp, st);
        }, "se.pool", (double)(reduce.w.size() + expand.w.size()) * 4, (double)n * hw * c + 4.0 * n * c * r);
        return gate;
    }

    // out = x*g (mode 0) or x + x*g (mode 1), + upsample(addend)
    Act4 gate_apply(const std::string& name, const Act4& x, int gate, int mode, const Act4* addend, int add_scale) {
        Act4 out = tensor(name, x.n, x.h, x.w, x.c);
        GateApplyParams p;
        p.n = x.n; p.h = x.h; p.w = x.w; p.c = x.c; p.mode = mode; p.add_scale = add_scale;
        p.out_cstride = x.c; p.out_coff = 0; p.dtype = m_.dtype;
        const int xt = x.tid, at = addend ? addend->tid : -1, ot = out.tid;
        m_.plan.add_op(name, {xt, gate, at}, {ot}, [p, xt, gate, at, ot](const Ctx& c, cudaStream_t st) mutable {
            p.x = c.act(xt);
            p.gate = gate >= 0 ? static_cast<const float*>(c.act(gate)) : nullptr;
            p.addend = c.act(at);
            p.out = c.act(ot);
            return launch_gate_apply(p, st);
        }, "gate", 0, 2.0 * x.n * x.h * x.w * x.c);
        return out;
    }

    WeightBlob& blob() { return m_.blob; }
    BuiltModel& model() { return m_; }

private:
    BuiltModel& m_;
    const WeightReader& r_;
    bool tc_, all_;
};

// ---------------------------------------------------------------------------
// Backbone
// ---------------------------------------------------------------------------

Act4 large_stem(Builder& b, int in_tid, int n, int h, int w, int mid, int out) {
    // LargeStem (src/cpu/model.rs:626-693), every conv BN + ReLU
    const WeightReader& r = b.reader();
    const std::string p = "model.backbone.encoder.convolution.";
    Act4 e = b.conv("stem1", r.conv_bn(p + "stem1", mid, 3, 3, 3, false), {{in_tid, 3, 3, 0, 1, SRC_NCHW_F32}}, n, h, w, 2, 2,
                    1, 1, 1, 1, ACT_RELU);
    // cat(max_pool_same_upper(stem1), stem2b) is materialised once: the pool
    // writes channels [0, mid) and stem2b channels [mid, 2 mid) of one tensor,
    // so stem3's 3x3 window reads plain pixels instead of re-pooling per tap.
    // The bandwidth-bound pool runs on the side stream beside stem2a/2b.
    Act4 cat = b.tensor("stem.cat", n, e.h, e.w, 2 * mid);
    b.begin_region();
    b.lane(1);
    b.maxpool_into("stem.pool", e, cat, 0);
    b.lane(0);
    Act4 br = b.conv1("stem2a", r.conv_bn(p + "stem2a", mid / 2, mid, 2, 2, false), e, 1, 1, 0, 0, 1, 1, ACT_RELU);
    b.conv1("stem2b", r.conv_bn(p + "stem2b", mid, mid / 2, 2, 2, false), br, 1, 1, 0, 0, 1, 1, ACT_RELU, -1, 1, &cat, mid);
    b.end_region();
    Act4 x = b.conv1("stem3", r.conv_bn(p + "stem3", mid, mid * 2, 3, 3, false), cat, 2, 2, 1, 1, 1, 1, ACT_RELU);
    GemmOpts o;
    o.act = ACT_RELU;
    return b.pointwise("stem4", r.conv_bn(p + "stem4", out, mid, 1, 1, false), x, o);
}

Act4 small_stem(Builder& b, int in_tid, int n, int h, int w, int mid, int out) {
    // SmallStem (src/cpu/model.rs:695-733): conv1 + BN + GELU, conv2 + BN
    const WeightReader& r = b.reader();
    const std::string p = "model.backbone.encoder.convolution.";
    Act4 e = b.conv("conv1", r.conv_bn(p + "conv1", mid, 3, 3, 3, false), {{in_tid, 3, 3, 0, 1, SRC_NCHW_F32}}, n, h, w, 2, 2,
                    1, 1, 1, 1, ACT_GELU);
    return b.conv1("conv2", r.conv_bn(p + "conv2", out, mid, 3, 3, false), e, 2, 2, 1, 1, 1, 1, ACT_NONE);
}

Act4 lcnet_block(Builder& b, const std::string& prefix, const Blk& blk, const Act4& x) {
    // LcNetBlock (src/cpu/model.rs:526-602): token dw3x3 -> [SE] -> 1x1 C->2C GELU -> 1x1 2C->C' (+ token output)
    const WeightReader& r = b.reader();
    ConvWeight tok = blk.residual() ? r.conv(prefix + ".token_conv", blk.cout, 1, 3, 3, true)
                                    : r.conv_bn(prefix + ".token_conv", blk.cin, 1, 3, 3, false);
    Act4 y = b.dwconv(prefix + ".token", tok, x, blk.sh, blk.sw, 1, 1, 1, 1, ACT_NONE, true);
    int gate = -1;
    if (blk.se) {
        const int c = blk.cin;
        gate = b.se_gate(prefix + ".se", y, r.conv(prefix + ".token_squeeze_excitation.convolutions.0", c / 4, c, 1, 1, true),
                         r.conv(prefix + ".token_squeeze_excitation.convolutions.2", c, c / 4, 1, 1, true), 1.f / 6.f);
    }
    // The fused pair saves the hidden tensor's round trip, which pays on large
    // maps; on small ones (fewer than ~100k pixel rows) its one-row-per-thread
    // grid is too small and the two tiled GEMMs (same sums, same order) win.
    if (b.pair_rows_ok(blk.cin, blk.cout) && (long long)y.n * y.h * y.w >= 98304) {
        return b.pair(prefix + ".pair", r.conv_bn(prefix + ".channel_conv1", blk.cin * 2, blk.cin, 1, 1, false),
                      r.conv_bn(prefix + ".channel_conv2", blk.cout, blk.cin * 2, 1, 1, false), y, gate, blk.residual());
    }
    if (gate >= 0) {
        // The BF16 and engine tensor-core GEMMs take no residual gate: apply the
        // SE gate once.  (The FP32 split GEMM gates A and the residual itself.)
        const bool split = b.split_gemm_ok(blk.cin, blk.cin * 2) && b.split_gemm_ok(blk.cin * 2, blk.cout);
        if (b.tensor_core_gemms() || (b.split_gemms() && !split)) {
            y = b.gate_apply(prefix + ".se.apply", y, gate, 0, nullptr, 1);
            gate = -1;
        }
    }
    GemmOpts o1;
    o1.act = ACT_GELU;
    o1.gate = gate;
    Act4 hdn = b.pointwise(prefix + ".pw1", r.conv_bn(prefix + ".channel_conv1", blk.cin * 2, blk.cin, 1, 1, false), y, o1);
    GemmOpts o2;
    if (blk.residual()) {
        // The residual is the token / SE output (src/cpu/backend.rs:504-521), so it is
        // read through the same gate.
        o2.residual = y.tid;
        o2.res_gate = gate;
    }
    return b.pointwise(prefix + ".pw2", r.conv_bn(prefix + ".channel_conv2", blk.cout, blk.cin * 2, 1, 1, false), hdn, o2);
}

std::vector<Act4> backbone(Builder& b, const std::vector<std::vector<Blk>>& stages, Act4 x) {
    std::vector<Act4> outs;
    for (size_t si = 0; si < stages.size(); ++si) {
        for (size_t bi = 0; bi < stages[si].size(); ++bi) {
            std::ostringstream p;
            p << "model.backbone.encoder.blocks." << si << ".blocks." << bi;
            x = lcnet_block(b, p.str(), stages[si][bi], x);
        }
        outs.push_back(x);
    }
    return outs;
}

// ---------------------------------------------------------------------------
// Detector necks and head
// ---------------------------------------------------------------------------

std::vector<Act4> rep_lk_fpn(Builder& b, const std::vector<Act4>& stages, int neck, int kernel) {
    // RepLkFpn (src/cpu/model.rs:1197-1254)
    const WeightReader& r = b.reader();
    std::vector<Act4> hid(4);
    std::vector<int> gates(4);
    // The pyramid levels are independent until the top-down adds: level 0
    // (the largest map) on the launch stream, levels 1-3 on the side stream.
    b.begin_region();
    for (int i = 0; i < 4; ++i) {
        b.lane(i == 0 ? 0 : 1);
        const std::string p = "model.neck.insert_conv." + std::to_string(i);
        GemmOpts o;
        o.has_bias = false;
        hid[i] = b.pointwise(p + ".in_conv", r.conv(p + ".in_conv", neck, stages[i].c, 1, 1, false), stages[i], o);
        gates[i] = b.se_gate(p + ".se", hid[i], r.conv(p + ".squeeze_excitation_block.conv1", neck / 4, neck, 1, 1, true),
                             r.conv(p + ".squeeze_excitation_block.conv2", neck, neck / 4, 1, 1, true), 0.2f);
    }
    b.end_region();
    // Residual SE (x + x g) then the top-down nearest x2 upsample-add, deepest first.
    std::vector<Act4> fused(4);
    fused[3] = b.gate_apply("model.neck.fused.3", hid[3], gates[3], 1, nullptr, 1);
    for (int i = 2; i >= 0; --i)
        fused[i] = b.gate_apply("model.neck.fused." + std::to_string(i), hid[i], gates[i], 1, &fused[i + 1], 2);
    std::vector<Act4> feats(4);
    const int pad = kernel / 2;
    b.begin_region();
    for (int i = 0; i < 4; ++i) {
        b.lane(i == 0 ? 0 : 1);
        const std::string p = "model.neck.input_conv." + std::to_string(i);
        Act4 d = b.dwconv(p + ".dw", r.conv(p + ".depthwise_convolution", neck, 1, kernel, kernel, true), fused[i], 1, 1, pad, pad,
                          pad, pad, ACT_NONE, true);
        GemmOpts o;
        o.has_bias = false;
        Act4 pw = b.pointwise(p + ".pw", r.conv(p + ".pointwise_convolution", neck / 4, neck, 1, 1, false), d, o);
        int g = b.se_gate(p + ".se", pw, r.conv(p + ".squeeze_excitation_module.conv1", neck / 16, neck / 4, 1, 1, true),
                          r.conv(p + ".squeeze_excitation_module.conv2", neck / 4, neck / 16, 1, 1, true), 0.2f);
        feats[i] = b.gate_apply(p + ".out", pw, g, 1, nullptr, 1);
    }
    b.end_region();
    return feats;
}

Act4 rank_one(Builder& b, const std::string& prefix, const Act4& x, int cin, int cout, int k, int residual = -1) {
    // RankOneConv2d (src/cpu/model.rs:165-219): depthwise k x k then 1x1 + bias
    const WeightReader& r = b.reader();
    const std::vector<float> w = r.get(prefix + ".weight", {(size_t)cout, (size_t)cin, (size_t)k, (size_t)k});
    const std::vector<float> bias = r.get(prefix + ".bias", {(size_t)cout});
    ConvWeight dw, pw;
    factor_rank_one(w, cin, cout, k, dw.w, pw.w);
    dw.cout = cin; dw.cin = 1; dw.kh = k; dw.kw = k; dw.b.assign(cin, 0.f);
    pw.cout = cout; pw.cin = cin; pw.kh = 1; pw.kw = 1; pw.b = bias;
    const int pad = k / 2;
    Act4 d = b.dwconv(prefix + ".dw", dw, x, 1, 1, pad, pad, pad, pad, ACT_NONE, false);
    GemmOpts o;
    o.residual = residual;
    return b.pointwise(prefix + ".pw", pw, d, o);
}

std::vector<Act4> medium_neck(Builder& b, const std::vector<Act4>& stages) {
    // DetectorNeck (src/cpu/model.rs:948-1067)
    const WeightReader& r = b.reader();
    const int chans[4] = {128, 256, 512, 896};
    std::vector<Act4> td(4);
    for (int i = 3; i >= 0; --i) {
        const std::string p = "model.neck.input_channel_adjustment_convolution." + std::to_string(i);
        GemmOpts o;
        o.has_bias = false;
        if (i < 3) { o.residual = td[i + 1].tid; o.res_scale = 2; }   // + upsample_x2(top_down[i+1])
        td[i] = b.pointwise(p, r.conv(p, 256, chans[i], 1, 1, false), stages[i], o);
    }
    std::vector<Act4> bu(4);
    for (int i = 0; i < 4; ++i) {
        Act4 proj = rank_one(b, "model.neck.input_feature_projection_convolution." + std::to_string(i), td[i], 256, 64, 9);
        if (i == 0) {
            bu[i] = proj;
        } else {
            const std::string p = "model.neck.path_aggregation_head_convolution." + std::to_string(i - 1);
            bu[i] = b.conv1(p, r.conv(p, 64, 64, 3, 3, false), bu[i - 1], 2, 2, 1, 1, 1, 1, ACT_NONE, proj.tid, 1);
        }
    }
    std::vector<Act4> refined(4);
    for (int i = 0; i < 4; ++i) {
        Act4 lat = rank_one(b, "model.neck.path_aggregation_lateral_convolution." + std::to_string(i), bu[i], 64, 64, 9);
        // IntraclassBlock (src/cpu/model.rs:890-946)
        const std::string p = "model.neck.intraclass_blocks." + std::to_string(i);
        GemmOpts o;
        Act4 h = b.pointwise(p + ".reduce", r.conv(p + ".conv_reduce_channel", 32, 64, 1, 1, true), lat, o);
        const char* ratios[3] = {"longratio", "midratio", "shortratio"};
        const int ks[3] = {7, 5, 3};
        for (int j = 0; j < 3; ++j) {
            const std::string rs = ratios[j];
            const int k = ks[j];
            ConvWeight fw = fuse_intraclass(r.conv(p + ".symmetric_conv_long_" + rs, 32, 32, k, k, true),
                                            r.conv(p + ".vertical_long_to_small_conv_" + rs, 32, 32, k, 1, true),
                                            r.conv(p + ".horizontal_small_to_long_conv_" + rs, 32, 32, 1, k, true));
            h = b.conv1(p + "." + rs, fw, h, 1, 1, k / 2, k / 2, k / 2, k / 2, ACT_NONE);
        }
        GemmOpts of;
        of.act = ACT_RELU;
        of.residual = lat.tid;   // input + relu(bn(conv_final(h)))
        refined[i] = b.pointwise(p + ".final", r.conv_bn(p + ".conv_final", 64, 32, 1, 1, true, "norm"), h, of);
    }
    return refined;
}

void detector_head(Builder& b, const std::vector<Act4>& feats, int channels) {
    // DetectorHead (src/cpu/model.rs:1479-1521) over upsample_and_cat_nchw(reversed feats, [8, 4, 2, 1]).
    const WeightReader& r = b.reader();
    BuiltModel& m = b.model();
    const int hidden = channels / 4;
    std::vector<Src> srcs;
    const int scales[4] = {8, 4, 2, 1};
    int total = 0;
    for (int i = 0; i < 4; ++i) {
        const Act4& f = feats[3 - i];
        srcs.push_back({f.tid, f.c, f.c, 0, scales[i], SRC_NHWC});
        total += f.c;
    }
    if (total != channels) fail(PPOCR_ERR_INVALID_MODEL, "detector neck produced the wrong channel count");
    const Act4& base = feats[0];
    Act4 down = b.conv("head.conv_down", r.conv_bn("head.conv_down", hidden, channels, 3, 3, false, "norm"), srcs, base.n, base.h,
                       base.w, 1, 1, 1, 1, 1, 1, ACT_RELU, -1, 1, nullptr, 0, true);
    std::vector<float> up_w = r.get("head.conv_up.convolution.weight", {(size_t)hidden, (size_t)hidden, 2, 2});
    std::vector<float> up_b = r.get("head.conv_up.convolution.bias", {(size_t)hidden});
    fold_transpose_bn(up_w, up_b, hidden, hidden, r, "head.conv_up.norm");
    const std::vector<float> fin_w = r.get("head.conv_final.weight", {(size_t)hidden, 1, 2, 2});
    const std::vector<float> fin_b = r.get("head.conv_final.bias", {1});
    // [ci][co][ky][kx] -> [tap][ci][co];  [ci][0][ky][kx] -> [tap][ci]
    std::vector<float> wup((size_t)4 * hidden * hidden), wfin((size_t)4 * hidden);
    for (int ci = 0; ci < hidden; ++ci)
        for (int co = 0; co < hidden; ++co)
            for (int t = 0; t < 4; ++t) wup[((size_t)t * hidden + ci) * hidden + co] = up_w[((size_t)ci * hidden + co) * 4 + t];
    for (int ci = 0; ci < hidden; ++ci)
        for (int t = 0; t < 4; ++t) wfin[(size_t)t * hidden + ci] = fin_w[(size_t)ci * 4 + t];
    const size_t wu = m.blob.add_f32(wup), bu = m.blob.add_f32(up_b), wf = m.blob.add_f32(wfin);
    const int H = down.h * 4, W = down.w * 4;
    m.prob = m.plan.add_raw("prob", (size_t)down.n * H * W * 4, true);
    m.mask = m.plan.add_raw("mask", (size_t)down.n * H * W, true);
    HeadParams p;
    p.n = down.n; p.h = down.h; p.w = down.w; p.ch = hidden; p.b_fin = fin_b[0]; p.dtype = m.dtype;
    const int dt = down.tid, pt = m.prob, mt = m.mask;
    std::shared_ptr<float> thr = m.mask_threshold;
    m.plan.add_op("head.tail", {dt}, {pt, mt}, [p, wu, bu, wf, dt, pt, mt, thr](const Ctx& c, cudaStream_t st) mutable {
        p.in = c.act(dt);
        p.w_up = c.wf(wu); p.b_up = c.wf(bu); p.w_fin = c.wf(wf);
        p.prob = static_cast<float*>(c.act(pt));
        p.mask = static_cast<uint8_t*>(c.act(mt));
        p.threshold = *thr;
        return launch_det_head(p, st);
    }, "head", (double)(wup.size() + wfin.size() + hidden) * 4,
                   2.0 * down.n * down.h * down.w * (4.0 * hidden * hidden + 16.0 * hidden));
}

// ---------------------------------------------------------------------------
// Recognizer heads
// ---------------------------------------------------------------------------

// Classifier logits with rows padded to a 16-byte pitch (whole-line TMA stores
// from the GEMM epilogue, 16-byte loads in the softmax).
int logits_tensor(BuiltModel& m, int rows) {
    m.logits_ld = (m.classes + 3) / 4 * 4;
    m.logits = m.plan.add_raw("logits", (size_t)rows * m.logits_ld * 4, true);
    return m.logits;
}

void ctc_outputs(Builder& b, int logits_tid, int rows, int classes) {
    BuiltModel& m = b.model();
    const int ld = m.logits_ld;
    m.probs = m.plan.add_raw("probs", (size_t)rows * classes * 4, true);
    m.index = m.plan.add_raw("index", (size_t)rows * 4, true);
    m.max_prob = m.plan.add_raw("max_prob", (size_t)rows * 4, true);
    m.margin = m.plan.add_raw("margin", (size_t)rows * 4, true);
    const int lt = logits_tid, pt = m.probs, it = m.index, mt = m.max_prob, gt = m.margin;
    m.plan.add_op("ctc.softmax", {lt}, {pt, it, mt, gt}, [rows, classes, ld, lt, pt, it, mt, gt](const Ctx& c, cudaStream_t st) {
        SoftmaxParams p;
        p.rows = rows; p.classes = classes; p.ld = ld;
        p.logits = static_cast<const float*>(c.act(lt));
        p.prob = static_cast<float*>(c.act(pt));
        p.index = static_cast<int32_t*>(c.act(it));
        p.max_prob = static_cast<float*>(c.act(mt));
        p.margin = static_cast<float*>(c.act(gt));
        return launch_softmax_ctc(p, st);
    }, "softmax", 0, 4.0 * rows * classes);
}

void tiny_rec_head(Builder& b, const Act4& x) {
    // TinyRecognizerHead (src/cpu/model.rs:1913-1936)
    const WeightReader& r = b.reader();
    BuiltModel& m = b.model();
    ConvWeight c1;
    c1.cout = 160; c1.cin = 1; c1.kh = 1; c1.kw = 5;
    c1.w = r.get("head.conv1.weight", {160, 1, 5});
    c1.b.assign(160, 0.f);
    r.fold_bn(c1, "head.norm1");
    Act4 h = b.dwconv("head.conv1", c1, x, 1, 1, 0, 2, 0, 2, ACT_HSWISH, true);
    ConvWeight c2;
    c2.cout = 160; c2.cin = 160; c2.kh = 1; c2.kw = 1;
    c2.w = r.get("head.conv2.weight", {160, 160, 1});
    c2.b.assign(160, 0.f);
    r.fold_bn(c2, "head.norm2");
    GemmOpts o;
    o.act = ACT_HSWISH;
    h = b.pointwise("head.conv2", c2, h, o);
    h = b.pointwise("head.fc1", r.linear("head.fc1", 160, 80), h, GemmOpts{});
    const int rows = h.n * h.h * h.w;
    logits_tensor(m, rows);
    GemmOpts of;
    of.c_f32 = true;
    of.ldc = m.logits_ld;
    of.rows_per_image = h.h * h.w;
    b.gemm_rows("head.fc2", r.linear("head.fc2", 80, m.classes), h.tid, rows, of, m.logits);
    ctc_outputs(b, m.logits, rows, m.classes);
}

void svtr_head(Builder& b, const Act4& x, int cin, int hidden, int mlp) {
    // RecEncoder + LightSvtrRecognizerHead (src/cpu/model.rs:1775-1875)
    const WeightReader& r = b.reader();
    BuiltModel& m = b.model();
    const std::string e = "head.encoder";
    GemmOpts silu;
    silu.act = ACT_SILU;
    Act4 skip = b.pointwise(e + ".skip", r.conv_bn(e + ".conv_block.0", hidden, cin, 1, 1, false), x, silu);
    Act4 red = b.pointwise(e + ".reduce", r.conv_bn(e + ".conv_block.1", hidden, cin, 1, 1, false), x, silu);
    // hidden + SiLU(BN(dw 1x7(hidden)))
    Act4 seq = b.dwconv(e + ".local", r.conv_bn(e + ".conv_block.2", hidden, 1, 1, 7, false), red, 1, 1, 0, 3, 0, 3, ACT_SILU, true,
                        red.tid);
    const int rows = seq.n * seq.h * seq.w;
    const int heads = 8, d = hidden / heads;
    auto layer_norm = [&](const std::string& name, const std::string& prefix, const Act4& in, int residual) {
        Act4 out = b.tensor(name, in.n, in.h, in.w, in.c);
        const size_t wo = m.blob.add_f32(r.get(prefix + ".weight", {(size_t)hidden}));
        const size_t bo = m.blob.add_f32(r.get(prefix + ".bias", {(size_t)hidden}));
        LayerNormParams p;
        p.rows = rows; p.c = hidden; p.eps = 1e-6f; p.dtype = m.dtype;
        const int it = in.tid, ot = out.tid;
        m.plan.add_op(name, {it, residual}, {ot}, [p, wo, bo, it, ot, residual](const Ctx& c, cudaStream_t st) mutable {
            p.in = c.act(it); p.weight = c.wf(wo); p.bias = c.wf(bo); p.residual = c.act(residual); p.out = c.act(ot);
            return launch_layernorm(p, st);
        }, "layernorm", 8.0 * hidden, 8.0 * rows * hidden);
        return out;
    };
    for (int i = 0; i < 2; ++i) {
        const std::string p = e + ".svtr_block." + std::to_string(i);
        Act4 a = layer_norm(p + ".ln1", p + ".layer_norm1", seq, -1);
        Act4 qkv = b.pointwise(p + ".qkv", r.linear(p + ".self_attn.qkv", hidden, hidden * 3), a, GemmOpts{});
        Act4 att = b.tensor(p + ".attn", seq.n, seq.h, seq.w, hidden);
        AttentionParams ap;
        ap.n = seq.n; ap.t = seq.h * seq.w; ap.heads = heads; ap.d = d; ap.scale = std::pow((float)d, -0.5f); ap.dtype = m.dtype;
        const int qt = qkv.tid, at = att.tid;
        m.plan.add_op(p + ".attention", {qt}, {at}, [ap, qt, at](const Ctx& c, cudaStream_t st) mutable {
            ap.qkv = c.act(qt); ap.out = c.act(at);
            return launch_attention(ap, st);
        }, "attention", 0, 4.0 * seq.n * heads * (double)ap.t * ap.t * d);
        GemmOpts op;
        op.residual = seq.tid;
        Act4 x2 = b.pointwise(p + ".proj", r.linear(p + ".self_attn.projection", hidden, hidden), att, op);
        Act4 a2 = layer_norm(p + ".ln2", p + ".layer_norm2", x2, -1);
        GemmOpts of1;
        of1.act = ACT_SILU;
        Act4 h1 = b.pointwise(p + ".fc1", r.linear(p + ".mlp.fc1", hidden, mlp), a2, of1);
        GemmOpts of2;
        of2.residual = x2.tid;
        seq = b.pointwise(p + ".fc2", r.linear(p + ".mlp.fc2", mlp, hidden), h1, of2);
    }
    Act4 fin = layer_norm(e + ".norm", e + ".norm", seq, skip.tid);
    logits_tensor(m, rows);
    GemmOpts oc;
    oc.c_f32 = true;
    oc.ldc = m.logits_ld;
    oc.rows_per_image = seq.h * seq.w;
    b.gemm_rows("head.head", r.linear("head.head", hidden, m.classes), fin.tid, rows, oc, m.logits);
    ctc_outputs(b, m.logits, rows, m.classes);
}

void check_count(const SafeTensors& st, const char* what, int size, size_t expected) {
    if (!st.recording() && st.size() != expected) {
        std::ostringstream o;
        o << size_name(size) << " " << what << " has " << st.size() << " tensors; expected " << expected;
        fail(PPOCR_ERR_INVALID_MODEL, o.str());
    }
}

}  // namespace

BuiltModel build_detector(const SafeTensors& st, int size, const size_t shape[4], DType dt, int tc_mode) {
    // validate_detector_shape (src/gpu/model.rs:268-276)
    const size_t n = shape[0], c = shape[1], h = shape[2], w = shape[3];
    if (n == 0 || c != 3 || h < 32 || w < 32 || h % 32 || w % 32) {
        std::ostringstream o;
        o << "detector expects [N, 3, H, W] with N > 0, H/W >= 32 and divisible by 32; got [" << n << ", " << c << ", " << h << ", "
          << w << "]";
        fail(PPOCR_ERR_INVALID_INPUT, o.str());
    }
    if (size != PPOCR_MEDIUM && size != PPOCR_SMALL && size != PPOCR_TINY) fail(PPOCR_ERR_INVALID_INPUT, "unknown model size");
    // Tensor counts per tier (src/gpu/model.rs:11-16, 58-65)
    check_count(st, "detector", size, size == PPOCR_MEDIUM ? 350 : 271);
    BuiltModel m;
    m.kind = Kind::Detector;
    m.size = size;
    m.dtype = dt;
    m.n = (int)n; m.h = (int)h; m.w = (int)w;
    m.tensor_count = (int)st.size();
    WeightReader r(st);
    Builder b(m, r, tc_mode);
    m.input = m.plan.add_raw("input", n * 3 * h * w * 4, true);
    int s1, s2, s3, s4, mid, out;
    if (size == PPOCR_MEDIUM) { s1 = 128; s2 = 256; s3 = 512; s4 = 896; mid = 64; out = 128; }
    else if (size == PPOCR_SMALL) { s1 = 48; s2 = 96; s3 = 192; s4 = 384; mid = 24; out = 48; }
    else { s1 = 32; s2 = 48; s3 = 64; s4 = 160; mid = 16; out = 32; }
    Act4 x = large_stem(b, m.input, (int)n, (int)h, (int)w, mid, out);
    std::vector<Act4> stages = backbone(b, detector_stages(s1, s2, s3, s4), x);
    std::vector<Act4> feats;
    int neck_channels;
    if (size == PPOCR_MEDIUM) {
        feats = medium_neck(b, stages);
        neck_channels = 256;
    } else {
        const int neck = size == PPOCR_SMALL ? 96 : 64, kernel = size == PPOCR_SMALL ? 7 : 5;
        feats = rep_lk_fpn(b, stages, neck, kernel);
        neck_channels = neck;
    }
    detector_head(b, feats, neck_channels);
    m.output_shape = {n, 1, h, w};
    m.output_elements = n * h * w;
    m.plan.finalize();
    return m;
}

BuiltModel build_recognizer(const SafeTensors& st, int size, const size_t shape[4], DType dt, int tc_mode) {
    // validate_recognizer_shape (src/gpu/model.rs:278-286)
    const size_t n = shape[0], c = shape[1], h = shape[2], w = shape[3];
    if (n == 0 || c != 3 || h != 48 || w < 32 || w % 4) {
        std::ostringstream o;
        o << "recognizer expects [N, 3, 48, W] with N > 0, W >= 32 and divisible by 4; got [" << n << ", " << c << ", " << h << ", "
          << w << "]";
        fail(PPOCR_ERR_INVALID_INPUT, o.str());
    }
    if (size != PPOCR_MEDIUM && size != PPOCR_SMALL && size != PPOCR_TINY) fail(PPOCR_ERR_INVALID_INPUT, "unknown model size");
    check_count(st, "recognizer", size, size == PPOCR_MEDIUM ? 269 : size == PPOCR_SMALL ? 250 : 150);
    BuiltModel m;
    m.kind = Kind::Recognizer;
    m.size = size;
    m.dtype = dt;
    m.n = (int)n; m.h = (int)h; m.w = (int)w;
    m.tensor_count = (int)st.size();
    m.classes = size == PPOCR_TINY ? 6906 : 18710;
    WeightReader r(st);
    Builder b(m, r, tc_mode);
    m.input = m.plan.add_raw("input", n * 3 * h * w * 4, true);
    Act4 x;
    if (size == PPOCR_TINY) x = small_stem(b, m.input, (int)n, (int)h, (int)w, 24, 48);
    else if (size == PPOCR_SMALL) x = large_stem(b, m.input, (int)n, (int)h, (int)w, 48, 96);
    else x = large_stem(b, m.input, (int)n, (int)h, (int)w, 64, 128);
    std::vector<Act4> stages = backbone(b, recognizer_stages(size), x);
    const Act4& last = stages.back();
    // AvgPool [3, 2] / [3, 2] (src/cpu/model.rs:2034-2039)
    Act4 pooled = b.tensor("avg_pool", last.n, last.h / 3, last.w / 2, last.c);
    const int backbone_channels = size == PPOCR_TINY ? 160 : size == PPOCR_SMALL ? 384 : 768;
    if (pooled.h != 1 || pooled.c != backbone_channels || pooled.w < 1)
        fail(PPOCR_ERR_INVALID_MODEL, std::string(size_name(size)) + " recognizer pooling produced an unexpected shape");
    {
        AvgPoolParams p;
        p.n = last.n; p.h = last.h; p.w = last.w; p.c = last.c; p.dtype = m.dtype;
        const int it = last.tid, ot = pooled.tid;
        m.plan.add_op("avg_pool", {it}, {ot}, [p, it, ot](const Ctx& c, cudaStream_t st) mutable {
            p.in = c.act(it); p.out = c.act(ot);
            return launch_avgpool_3x2(p, st);
        }, "pool", 0, 6.0 * pooled.n * pooled.w * pooled.c);
    }
    m.t = pooled.w;
    if (size == PPOCR_TINY) tiny_rec_head(b, pooled);
    else if (size == PPOCR_SMALL) svtr_head(b, pooled, 384, 120, 240);
    else svtr_head(b, pooled, 768, 192, 768);
    m.output_shape = {n, (size_t)m.t, (size_t)m.classes};
    m.output_elements = n * (size_t)m.t * m.classes;
    m.plan.finalize();
    return m;
}

}  // namespace ppocr
