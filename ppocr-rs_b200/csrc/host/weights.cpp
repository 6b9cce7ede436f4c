// Load-time weight rewrites.  All arithmetic is done in the precision the
// reference CPU path uses (F32 folds, F64 power iteration); this file is
// compiled with -ffp-contract=off so products and sums round separately, as
// Rust evaluates `a * b + c`.
#include "weights.hpp"

#include <cmath>
#include <cstring>
#include <sstream>

#include "common.hpp"

namespace ppocr {

ConvWeight WeightReader::conv(const std::string& prefix, int cout, int cin_per_group, int kh, int kw, bool bias) const {
    ConvWeight cw;
    cw.cout = cout; cw.cin = cin_per_group; cw.kh = kh; cw.kw = kw;
    cw.w = get(prefix + ".weight", {(size_t)cout, (size_t)cin_per_group, (size_t)kh, (size_t)kw});
    cw.b = bias ? get(prefix + ".bias", {(size_t)cout}) : std::vector<float>(cout, 0.f);
    return cw;
}

void WeightReader::fold_bn(ConvWeight& cw, const std::string& norm) const {
    const size_t c = (size_t)cw.cout;
    const std::vector<float> gamma = get(norm + ".weight", {c});
    const std::vector<float> beta = get(norm + ".bias", {c});
    const std::vector<float> mean = get(norm + ".running_mean", {c});
    const std::vector<float> var = get(norm + ".running_var", {c});
    const size_t row = cw.w.size() / c;
    for (size_t ch = 0; ch < c; ++ch) {
        const float scale = gamma[ch] / std::sqrt(var[ch] + 1e-5f);
        for (size_t i = 0; i < row; ++i) cw.w[ch * row + i] *= scale;
        cw.b[ch] = (cw.b[ch] - mean[ch]) * scale + beta[ch];
    }
}

ConvWeight WeightReader::conv_bn(const std::string& prefix, int cout, int cin_per_group, int kh, int kw, bool bias,
                                 const std::string& norm) const {
    ConvWeight cw = conv(prefix + ".convolution", cout, cin_per_group, kh, kw, bias);
    fold_bn(cw, prefix + "." + norm);
    return cw;
}

ConvWeight WeightReader::linear(const std::string& prefix, int in, int out) const {
    ConvWeight cw;
    cw.cout = out; cw.cin = in; cw.kh = 1; cw.kw = 1;
    cw.w = get(prefix + ".weight", {(size_t)out, (size_t)in});
    cw.b = get(prefix + ".bias", {(size_t)out});
    return cw;
}

void factor_rank_one(const std::vector<float>& src, int cin, int cout, int k, std::vector<float>& depthwise,
                     std::vector<float>& pointwise) {
    const int sp = k * k;
    if (k <= 0 || k % 2 == 0) fail(PPOCR_ERR_INVALID_MODEL, "rank-one convolution kernel must be positive and odd");
    if ((int)src.size() != cout * cin * sp) fail(PPOCR_ERR_INVALID_MODEL, "rank-one convolution weight has invalid shape");
    for (float v : src)
        if (!std::isfinite(v)) fail(PPOCR_ERR_INVALID_MODEL, "rank-one convolution weight contains non-finite values");
    depthwise.assign((size_t)cin * sp, 0.f);
    pointwise.assign((size_t)cout * cin, 0.f);
    std::vector<double> dir(sp), scales(cout);
    for (int i = 0; i < cin; ++i) {
        int o0 = 0;
        double e0 = 0.0;
        for (int o = 0; o < cout; ++o) {
            const float* blk = &src[((size_t)o * cin + i) * sp];
            double e = 0.0;
            for (int s = 0; s < sp; ++s) e += (double)blk[s] * (double)blk[s];
            if (e > e0) { o0 = o; e0 = e; }
        }
        if (e0 == 0.0) continue;
        const double n0 = std::sqrt(e0);
        for (int s = 0; s < sp; ++s) dir[s] = (double)src[((size_t)o0 * cin + i) * sp + s] / n0;
        for (int it = 0; it < 4; ++it) {
            double se = 0.0;
            for (int o = 0; o < cout; ++o) {
                const float* blk = &src[((size_t)o * cin + i) * sp];
                double a = 0.0;
                for (int s = 0; s < sp; ++s) a += (double)blk[s] * dir[s];
                scales[o] = a;
                se += a * a;
            }
            if (!std::isfinite(se) || se <= 0.0) fail(PPOCR_ERR_INVALID_MODEL, "rank-one convolution factorization became degenerate");
            double nn = 0.0;
            for (int s = 0; s < sp; ++s) {
                double a = 0.0;
                for (int o = 0; o < cout; ++o) a += (double)src[((size_t)o * cin + i) * sp + s] * scales[o];
                dir[s] = a / se;
            }
            for (int s = 0; s < sp; ++s) nn += dir[s] * dir[s];
            nn = std::sqrt(nn);
            if (!std::isfinite(nn) || nn <= 0.0) fail(PPOCR_ERR_INVALID_MODEL, "rank-one convolution spatial factor became degenerate");
            for (int s = 0; s < sp; ++s) dir[s] /= nn;
        }
        for (int o = 0; o < cout; ++o) {
            const float* blk = &src[((size_t)o * cin + i) * sp];
            double a = 0.0;
            for (int s = 0; s < sp; ++s) a += (double)blk[s] * dir[s];
            pointwise[(size_t)o * cin + i] = (float)a;
        }
        for (int s = 0; s < sp; ++s) depthwise[(size_t)i * sp + s] = (float)dir[s];
    }
    double max_src = 0.0, max_err = 0.0, src_e = 0.0, err_e = 0.0;
    for (int o = 0; o < cout; ++o)
        for (int i = 0; i < cin; ++i) {
            const float scale = pointwise[(size_t)o * cin + i];
            for (int s = 0; s < sp; ++s) {
                const float expected = src[((size_t)o * cin + i) * sp + s];
                const float actual = scale * depthwise[(size_t)i * sp + s];
                const double err = std::fabs(expected - actual);
                max_src = std::max(max_src, (double)std::fabs(expected));
                max_err = std::max(max_err, err);
                src_e += (double)expected * (double)expected;
                err_e += err * err;
            }
        }
    const double rel = src_e == 0.0 ? 0.0 : std::sqrt(err_e / src_e);
    const double limit = max_src * 1e-5 + 1e-12;
    if (!(max_err <= limit && rel <= 1e-6)) {
        std::ostringstream o;
        o << "fused convolution is not rank-one separable: max error " << max_err << " (limit " << limit
          << "), relative Frobenius error " << rel << " (limit 1e-6)";
        fail(PPOCR_ERR_INVALID_MODEL, o.str());
    }
}

ConvWeight fuse_intraclass(const ConvWeight& sym, const ConvWeight& ver, const ConvWeight& hor) {
    if (sym.kh != sym.kw || sym.kh % 2 == 0) fail(PPOCR_ERR_INVALID_MODEL, "intraclass symmetric kernel must be odd and square");
    if (ver.kh != sym.kh || ver.kw != 1 || hor.kh != 1 || hor.kw != sym.kw || ver.cout != sym.cout || hor.cout != sym.cout ||
        ver.cin != sym.cin || hor.cin != sym.cin)
        fail(PPOCR_ERR_INVALID_MODEL, "intraclass branch weight has invalid shape");
    ConvWeight out = sym;
    const int k = sym.kh, c = k / 2;
    for (int o = 0; o < sym.cout; ++o)
        for (int i = 0; i < sym.cin; ++i) {
            const size_t branch = ((size_t)o * sym.cin + i) * k;
            const size_t base = branch * k;
            for (int r = 0; r < k; ++r) out.w[base + r * k + c] += ver.w[branch + r];
            for (int col = 0; col < k; ++col) out.w[base + c * k + col] += hor.w[branch + col];
        }
    for (int o = 0; o < sym.cout; ++o) {
        out.b[o] += ver.b[o];
        out.b[o] += hor.b[o];
    }
    return out;
}

void fold_transpose_bn(std::vector<float>& w, std::vector<float>& b, int cin, int cout, const WeightReader& r,
                       const std::string& norm) {
    const std::vector<float> gamma = r.get(norm + ".weight", {(size_t)cout});
    const std::vector<float> beta = r.get(norm + ".bias", {(size_t)cout});
    const std::vector<float> mean = r.get(norm + ".running_mean", {(size_t)cout});
    const std::vector<float> var = r.get(norm + ".running_var", {(size_t)cout});
    const size_t kernel = w.size() / ((size_t)cin * cout);
    for (int o = 0; o < cout; ++o) {
        const float scale = gamma[o] / std::sqrt(var[o] + 1e-5f);
        for (int i = 0; i < cin; ++i) {
            const size_t st = ((size_t)i * cout + o) * kernel;
            for (size_t q = 0; q < kernel; ++q) w[st + q] *= scale;
        }
        b[o] = (b[o] - mean[o]) * scale + beta[o];
    }
}

size_t WeightBlob::reserve(size_t bytes) {
    size_t off = (data_.size() + 255) & ~(size_t)255;
    data_.resize(off + bytes);
    return off;
}

size_t WeightBlob::add_f32(const std::vector<float>& v) {
    const size_t off = reserve(v.size() * 4 + 16);
    if (!v.empty()) std::memcpy(data_.data() + off, v.data(), v.size() * 4);
    return off;
}

static inline uint16_t to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);   // NaN stays NaN
    u += 0x7fffu + ((u >> 16) & 1u);                                            // round to nearest even
    return (uint16_t)(u >> 16);
}

size_t WeightBlob::add_bf16(const std::vector<float>& v) {
    const size_t off = reserve(v.size() * 2 + 16);
    uint16_t* d = reinterpret_cast<uint16_t*>(data_.data() + off);
    for (size_t i = 0; i < v.size(); ++i) d[i] = to_bf16(v[i]);
    return off;
}

std::vector<float> pack_conv_tiles(const ConvWeight& cw, int tile) {
    const int tiles = (cw.cout + tile - 1) / tile;
    const int taps = cw.kh * cw.kw;
    std::vector<float> out((size_t)tiles * taps * cw.cin * tile, 0.f);
    for (int o = 0; o < cw.cout; ++o)
        for (int i = 0; i < cw.cin; ++i)
            for (int t = 0; t < taps; ++t)
                out[(((size_t)(o / tile) * taps + t) * cw.cin + i) * tile + (o % tile)] =
                    cw.w[((size_t)o * cw.cin + i) * taps + t];
    return out;
}

std::vector<float> pack_conv_kn(const ConvWeight& cw, int& n_pad) {
    n_pad = (cw.cout + 3) / 4 * 4;
    const int taps = cw.kh * cw.kw;
    std::vector<float> out((size_t)taps * cw.cin * n_pad, 0.f);
    for (int o = 0; o < cw.cout; ++o)
        for (int i = 0; i < cw.cin; ++i)
            for (int t = 0; t < taps; ++t)
                out[((size_t)t * cw.cin + i) * n_pad + o] = cw.w[((size_t)o * cw.cin + i) * taps + t];
    return out;
}

std::vector<float> pack_conv_halo(const ConvWeight& cw, int bn) {
    const int taps = cw.kh * cw.kw, quads = (cw.cin + 3) / 4;
    std::vector<float> out((size_t)quads * taps * 4 * bn, 0.f);
    for (int o = 0; o < cw.cout; ++o)
        for (int i = 0; i < cw.cin; ++i)
            for (int t = 0; t < taps; ++t)
                out[(((size_t)(i / 4) * taps + t) * 4 + i % 4) * bn + o] = cw.w[((size_t)o * cw.cin + i) * taps + t];
    return out;
}

float bf16_round(float f) {
    const uint16_t h = to_bf16(f);
    const uint32_t u = (uint32_t)h << 16;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}

std::vector<float> pack_engine_kn(const ConvWeight& cw, int planes, int n_pad, int k_pad, int cin_pad) {
    const int taps = cw.kh * cw.kw;
    const int cpt = cin_pad > 0 ? cin_pad : cw.cin;   // K columns per tap (the padding stays zero)
    std::vector<float> out((size_t)planes * n_pad * k_pad, 0.f);
    for (int o = 0; o < cw.cout; ++o)
        for (int t = 0; t < taps; ++t)
            for (int i = 0; i < cw.cin; ++i) {
                float v = cw.w[((size_t)o * cw.cin + i) * taps + t];
                const size_t col = (size_t)t * cpt + i;
                for (int pl = 0; pl < planes; ++pl) {
                    const float piece = bf16_round(v);   // x0 = bf16(x), x1 = bf16(x - x0), x2 = bf16(x - x0 - x1)
                    out[((size_t)pl * n_pad + o) * k_pad + col] = piece;
                    v = v - piece;
                }
            }
    return out;
}

std::vector<float> pack_conv_tc(const ConvWeight& cw, int n_pad, int cin_pad) {
    const int taps = cw.kh * cw.kw;
    const size_t k = (size_t)taps * cin_pad;
    std::vector<float> out((size_t)n_pad * k, 0.f);
    for (int o = 0; o < cw.cout; ++o)
        for (int t = 0; t < taps; ++t)
            for (int i = 0; i < cw.cin; ++i) out[(size_t)o * k + (size_t)t * cin_pad + i] = cw.w[((size_t)o * cw.cin + i) * taps + t];
    return out;
}

std::vector<float> pack_depthwise(const ConvWeight& cw) {
    const int taps = cw.kh * cw.kw;
    std::vector<float> out((size_t)taps * cw.cout);
    for (int c = 0; c < cw.cout; ++c)
        for (int t = 0; t < taps; ++t) out[(size_t)t * cw.cout + c] = cw.w[(size_t)c * taps + t];
    return out;
}

std::vector<float> pack_gemm_kn(const ConvWeight& cw, int& n_pad) {
    n_pad = (cw.cout + 3) / 4 * 4;
    const int k = cw.cin * cw.kh * cw.kw;
    std::vector<float> out((size_t)k * n_pad, 0.f);
    for (int n = 0; n < cw.cout; ++n)
        for (int kk = 0; kk < k; ++kk) out[(size_t)kk * n_pad + n] = cw.w[(size_t)n * k + kk];
    return out;
}


std::vector<float> pack_gemm_nk(const ConvWeight& cw, int n_pad, int k_pad) {
    const int k = cw.cin * cw.kh * cw.kw;
    std::vector<float> out((size_t)n_pad * k_pad, 0.f);
    for (int n = 0; n < cw.cout; ++n)
        for (int kk = 0; kk < k; ++kk) out[(size_t)n * k_pad + kk] = cw.w[(size_t)n * k + kk];
    return out;
}

}  // namespace ppocr
