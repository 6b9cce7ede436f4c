// CPU restatement of the PP-OCRv6 tiny / small detector forward in C++
// (FP32, NCHW) -- TEST INFRASTRUCTURE ONLY: the timed CPU baseline of
// bench.py, checked against oracle/model.py by tests/test_cpu_detector.py.
// The product (ppocr-rs_b200/) never links or calls it.
//
// It follows the reference's CPU model (ppocr-rs src/cpu/model.rs):
//   LargeStem (626-693), LcNetBlock (526-602) with SqueezeExcitation (456-493),
//   RepLkFpn (1197-1254) with VariantSqueezeExcitation in residual form
//   (1069-1143, kernels/mod.rs:777-796), DetectorHead (1479-1521), BN folding
//   with eps 1e-5 (371-407), the A&S erf GELU (kernels/mod.rs:2383-2403),
//   max-pool same-upper (ops.rs:1520-1535), nearest upsampling and
//   concatenation deepest first (1265-1417), ConvTranspose 2x2 IOHW
//   (backend.rs:1088-1181).
// Images of a batch run on separate threads (OpenMP), each image
// single-threaded, so the baseline scales with the host's cores.
//
// Build: oracle/Makefile (g++ -O3 -march=native -fopenmp).
#include <omp.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// safetensors (F32 only): u64 header length, JSON header, data.
// ---------------------------------------------------------------------------
struct Entry {
    std::vector<size_t> shape;
    size_t begin = 0, end = 0;
};

class Weights {
public:
    explicit Weights(const std::string& path) {
        std::ifstream f(path, std::ios::binary);
        if (!f) throw std::runtime_error("read " + path);
        bytes_.assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
        if (bytes_.size() < 8) throw std::runtime_error("short safetensors file");
        uint64_t n = 0;
        for (int k = 7; k >= 0; --k) n = (n << 8) | (unsigned char)bytes_[k];
        const std::string h(bytes_.data() + 8, bytes_.data() + 8 + n);
        base_ = 8 + n;
        // Entries look like "name":{"dtype":"F32","shape":[..],"data_offsets":[a,b]}.
        size_t i = 0;
        while ((i = h.find("\"dtype\"", i)) != std::string::npos) {
            const size_t obj = h.rfind('{', i);
            const size_t q1 = h.rfind('"', h.rfind(':', obj) - 1);
            const size_t q0 = h.rfind('"', q1 - 1);
            const std::string name = h.substr(q0 + 1, q1 - q0 - 1);
            Entry e;
            const size_t s0 = h.find('[', h.find("\"shape\"", i)), s1 = h.find(']', s0);
            std::string dims = h.substr(s0 + 1, s1 - s0 - 1);
            for (size_t p = 0; p < dims.size();) {
                size_t c = dims.find(',', p);
                if (c == std::string::npos) c = dims.size();
                if (c > p) e.shape.push_back(std::stoull(dims.substr(p, c - p)));
                p = c + 1;
            }
            const size_t o0 = h.find('[', h.find("\"data_offsets\"", i)), o1 = h.find(']', o0);
            const std::string offs = h.substr(o0 + 1, o1 - o0 - 1);
            e.begin = std::stoull(offs.substr(0, offs.find(',')));
            e.end = std::stoull(offs.substr(offs.find(',') + 1));
            map_[name] = e;
            i = o1;
        }
    }
    std::vector<float> get(const std::string& name, size_t count) const {
        auto it = map_.find(name);
        if (it == map_.end()) throw std::runtime_error("missing tensor " + name);
        if (it->second.end - it->second.begin != count * 4) throw std::runtime_error("bad size of " + name);
        std::vector<float> v(count);
        std::memcpy(v.data(), bytes_.data() + base_ + it->second.begin, count * 4);
        return v;
    }

private:
    std::vector<char> bytes_;
    size_t base_ = 0;
    std::map<std::string, Entry> map_;
};

// ---------------------------------------------------------------------------
// Tensors and operators (one image, NCHW)
// ---------------------------------------------------------------------------
struct T {
    int c = 0, h = 0, w = 0;
    std::vector<float> d;
    T() = default;
    T(int c_, int h_, int w_) : c(c_), h(h_), w(w_), d((size_t)c_ * h_ * w_, 0.f) {}
    float* ch(int i) { return d.data() + (size_t)i * h * w; }
    const float* ch(int i) const { return d.data() + (size_t)i * h * w; }
};

enum Act { NONE, RELU, GELU };

inline float erf_as(float x) {
    const float s = x < 0.f ? -1.f : 1.f;
    const float a = std::fabs(x);
    const float t = 1.f / std::fma(a, 0.3275911f, 1.f);
    const float p = t * (0.2548296f + t * (-0.28449672f + t * (1.4214138f + t * (-1.4531521f + t * 1.0614054f))));
    return s * (1.f - p * std::exp(-a * a));
}
inline float act(float v, Act a) {
    if (a == RELU) return v > 0.f ? v : 0.f;
    if (a == GELU) return 0.5f * v * (1.f + erf_as(v * 0.70710678118654752f));
    return v;
}

struct Conv {
    int cout = 0, cin = 0, kh = 1, kw = 1, sh = 1, sw = 1, pt = 0, pl = 0, pb = 0, pr = 0, groups = 1;
    Act a = NONE;
    std::vector<float> w, b;   // OIHW (I per group), bias [cout]
};

Conv load(const Weights& W, const std::string& prefix, int cin, int cout, int k, int s, int pad, bool bias, int groups,
          Act a = NONE, const char* bn = nullptr) {
    Conv c;
    c.cout = cout; c.cin = cin; c.kh = c.kw = k; c.sh = c.sw = s; c.pt = c.pl = c.pb = c.pr = pad; c.groups = groups; c.a = a;
    const size_t wn = (size_t)cout * (cin / groups) * k * k;
    const std::string wname = bn ? prefix + ".convolution.weight" : prefix + ".weight";
    c.w = W.get(wname, wn);
    c.b = bias ? W.get((bn ? prefix + ".convolution.bias" : prefix + ".bias"), cout) : std::vector<float>(cout, 0.f);
    if (bn) {
        // BN fold (src/cpu/model.rs:371-407): scale = g / sqrt(v + 1e-5)
        const std::string n = prefix + "." + bn;
        const auto g = W.get(n + ".weight", cout), be = W.get(n + ".bias", cout), m = W.get(n + ".running_mean", cout),
                   v = W.get(n + ".running_var", cout);
        const size_t per = wn / cout;
        for (int o = 0; o < cout; ++o) {
            const float scale = g[o] / std::sqrt(v[o] + 1e-5f);
            for (size_t i = 0; i < per; ++i) c.w[o * per + i] *= scale;
            c.b[o] = (c.b[o] - m[o]) * scale + be[o];
        }
    }
    return c;
}

T conv(const Conv& cv, const T& x) {
    const int ho = (x.h + cv.pt + cv.pb - cv.kh) / cv.sh + 1, wo = (x.w + cv.pl + cv.pr - cv.kw) / cv.sw + 1;
    T y(cv.cout, ho, wo);
    const int cig = cv.cin / cv.groups, cog = cv.cout / cv.groups;
    const size_t hw = (size_t)ho * wo;
    if (cv.kh == 1 && cv.kw == 1 && cv.sh == 1 && cv.sw == 1 && cv.groups == 1) {
        // Pointwise: four output channels per pass over the input rows.
        for (int o = 0; o < cv.cout; o += 4) {
            const int n = cv.cout - o < 4 ? cv.cout - o : 4;
            float* out[4];
            for (int j = 0; j < 4; ++j) out[j] = y.ch(o + (j < n ? j : 0));
            for (int j = 0; j < n; ++j)
                for (size_t p = 0; p < hw; ++p) out[j][p] = cv.b[o + j];
            for (int i = 0; i < cv.cin; ++i) {
                const float* xi = x.ch(i);
                if (n == 4) {
                    const float w0 = cv.w[(size_t)(o + 0) * cv.cin + i], w1 = cv.w[(size_t)(o + 1) * cv.cin + i],
                                w2 = cv.w[(size_t)(o + 2) * cv.cin + i], w3 = cv.w[(size_t)(o + 3) * cv.cin + i];
                    float *o0 = out[0], *o1 = out[1], *o2 = out[2], *o3 = out[3];
#pragma omp simd
                    for (size_t p = 0; p < hw; ++p) {
                        const float v = xi[p];
                        o0[p] += w0 * v; o1[p] += w1 * v; o2[p] += w2 * v; o3[p] += w3 * v;
                    }
                } else {
                    for (int j = 0; j < n; ++j) {
                        const float wj = cv.w[(size_t)(o + j) * cv.cin + i];
                        float* oj = out[j];
#pragma omp simd
                        for (size_t p = 0; p < hw; ++p) oj[p] += wj * xi[p];
                    }
                }
            }
        }
    } else {
        for (int o = 0; o < cv.cout; ++o) {
            float* yo = y.ch(o);
            for (size_t p = 0; p < hw; ++p) yo[p] = cv.b[o];
            const int g = o / cog;
            for (int i = 0; i < cig; ++i) {
                const float* xi = x.ch(g * cig + i);
                for (int ky = 0; ky < cv.kh; ++ky)
                    for (int kx = 0; kx < cv.kw; ++kx) {
                        const float wv = cv.w[(((size_t)o * cig + i) * cv.kh + ky) * cv.kw + kx];
                        // output columns whose input column lies inside the image
                        int ox0 = 0;
                        while (ox0 < wo && ox0 * cv.sw + kx - cv.pl < 0) ++ox0;
                        int ox1 = wo;
                        while (ox1 > ox0 && (ox1 - 1) * cv.sw + kx - cv.pl >= x.w) --ox1;
                        for (int oy = 0; oy < ho; ++oy) {
                            const int iy = oy * cv.sh + ky - cv.pt;
                            if (iy < 0 || iy >= x.h) continue;
                            const float* xr = xi + (size_t)iy * x.w + kx - cv.pl;
                            float* yr = yo + (size_t)oy * wo;
                            if (cv.sw == 1) {
#pragma omp simd
                                for (int ox = ox0; ox < ox1; ++ox) yr[ox] += wv * xr[ox];
                            } else {
                                for (int ox = ox0; ox < ox1; ++ox) yr[ox] += wv * xr[ox * cv.sw];
                            }
                        }
                    }
            }
        }
    }
    if (cv.a != NONE)
        for (auto& v : y.d) v = act(v, cv.a);
    return y;
}

T max_pool_same_upper(const T& x) {
    T y(x.c, x.h, x.w);
    for (int c = 0; c < x.c; ++c)
        for (int i = 0; i < x.h; ++i)
            for (int j = 0; j < x.w; ++j) {
                float m = x.ch(c)[(size_t)i * x.w + j];
                if (j + 1 < x.w) m = std::max(m, x.ch(c)[(size_t)i * x.w + j + 1]);
                if (i + 1 < x.h) {
                    m = std::max(m, x.ch(c)[(size_t)(i + 1) * x.w + j]);
                    if (j + 1 < x.w) m = std::max(m, x.ch(c)[(size_t)(i + 1) * x.w + j + 1]);
                }
                y.ch(c)[(size_t)i * x.w + j] = m;
            }
    return y;
}

T cat(const std::vector<const T*>& xs) {
    int c = 0;
    for (auto* x : xs) c += x->c;
    T y(c, xs[0]->h, xs[0]->w);
    size_t off = 0;
    for (auto* x : xs) {
        std::memcpy(y.d.data() + off, x->d.data(), x->d.size() * 4);
        off += x->d.size();
    }
    return y;
}

T upsample(const T& x, int s) {
    if (s == 1) return x;
    T y(x.c, x.h * s, x.w * s);
    for (int c = 0; c < x.c; ++c)
        for (int i = 0; i < y.h; ++i)
            for (int j = 0; j < y.w; ++j) y.ch(c)[(size_t)i * y.w + j] = x.ch(c)[(size_t)(i / s) * x.w + j / s];
    return y;
}

// Squeeze-excitation: mean -> 1x1 ReLU -> 1x1 -> hard-sigmoid(alpha, 0.5);
// out = x g (plain) or x + x g (residual form).
struct SE {
    Conv reduce, expand;
    float alpha = 1.f / 6.f;
    bool residual = false;
    T operator()(const T& x) const {
        const size_t hw = (size_t)x.h * x.w;
        std::vector<float> mean(x.c), hid(reduce.cout), g(x.c);
        for (int c = 0; c < x.c; ++c) {
            float s = 0.f;
            for (size_t p = 0; p < hw; ++p) s += x.ch(c)[p];
            mean[c] = s / (float)hw;
        }
        for (int o = 0; o < reduce.cout; ++o) {
            float s = reduce.b[o];
            for (int i = 0; i < x.c; ++i) s += reduce.w[(size_t)o * x.c + i] * mean[i];
            hid[o] = s > 0.f ? s : 0.f;
        }
        for (int o = 0; o < x.c; ++o) {
            float s = expand.b[o];
            for (int i = 0; i < reduce.cout; ++i) s += expand.w[(size_t)o * reduce.cout + i] * hid[i];
            g[o] = std::min(std::max(s * alpha + 0.5f, 0.f), 1.f);
        }
        T y = x;
        for (int c = 0; c < x.c; ++c) {
            float* yc = y.ch(c);
            for (size_t p = 0; p < hw; ++p) yc[p] = residual ? yc[p] + yc[p] * g[c] : yc[p] * g[c];
        }
        return y;
    }
};

struct Block {
    bool residual = false, se_on = false;
    Conv token, pw1, pw2;
    SE se;
    T operator()(const T& x) const {
        T y = conv(token, x);
        if (se_on) y = se(y);
        T out = conv(pw2, conv(pw1, y));
        if (residual)
            for (size_t i = 0; i < out.d.size(); ++i) out.d[i] = y.d[i] + out.d[i];
        return out;
    }
};

struct Detector {
    Conv stem1, stem2a, stem2b, stem3, stem4;
    std::vector<std::vector<Block>> stages;
    std::vector<Conv> in_conv, dw, pw;
    std::vector<SE> insert_se, input_se;
    Conv down;
    std::vector<float> up_w, up_b, fin_w;
    float fin_b = 0.f;
    int hidden = 0;

    Detector(const Weights& W, int size) {
        // Stage widths, stems and necks (src/cpu/model.rs:1578-1680).
        const bool small = size == 1;
        const int s1 = small ? 48 : 32, s2 = small ? 96 : 48, s3 = small ? 192 : 64, s4 = small ? 384 : 160;
        const int mid = small ? 24 : 16, out = small ? 48 : 32, neck = small ? 96 : 64, k = small ? 7 : 5;
        const std::string p = "model.backbone.encoder.convolution.";
        stem1 = load(W, p + "stem1", 3, mid, 3, 2, 1, false, 1, RELU, "normalization");
        stem2a = load(W, p + "stem2a", mid, mid / 2, 2, 1, 0, false, 1, RELU, "normalization");
        stem2a.pb = stem2a.pr = 1;
        stem2b = load(W, p + "stem2b", mid / 2, mid, 2, 1, 0, false, 1, RELU, "normalization");
        stem2b.pb = stem2b.pr = 1;
        stem3 = load(W, p + "stem3", mid * 2, mid, 3, 2, 1, false, 1, RELU, "normalization");
        stem4 = load(W, p + "stem4", mid, out, 1, 1, 0, false, 1, RELU, "normalization");
        struct B { int cin, cout, s; bool se; };
        const std::vector<std::vector<B>> st = {
            {{s1, s1, 1, true}, {s1, s1, 1, false}},
            {{s1, s2, 2, false}, {s2, s2, 1, true}, {s2, s2, 1, false}},
            {{s2, s3, 2, false}, {s3, s3, 1, true}, {s3, s3, 1, false}, {s3, s3, 1, true}, {s3, s3, 1, false}},
            {{s3, s4, 2, false}, {s4, s4, 1, true}, {s4, s4, 1, false}},
        };
        for (size_t si = 0; si < st.size(); ++si) {
            stages.emplace_back();
            for (size_t bi = 0; bi < st[si].size(); ++bi) {
                const B& b = st[si][bi];
                const std::string q = "model.backbone.encoder.blocks." + std::to_string(si) + ".blocks." + std::to_string(bi);
                Block blk;
                blk.residual = b.cin == b.cout && b.s == 1;
                blk.token = blk.residual ? load(W, q + ".token_conv", b.cin, b.cin, 3, b.s, 1, true, b.cin)
                                         : load(W, q + ".token_conv", b.cin, b.cin, 3, b.s, 1, false, b.cin, NONE, "normalization");
                blk.se_on = b.se;
                if (b.se) {
                    blk.se.reduce = load(W, q + ".token_squeeze_excitation.convolutions.0", b.cin, b.cin / 4, 1, 1, 0, true, 1);
                    blk.se.expand = load(W, q + ".token_squeeze_excitation.convolutions.2", b.cin / 4, b.cin, 1, 1, 0, true, 1);
                }
                blk.pw1 = load(W, q + ".channel_conv1", b.cin, b.cin * 2, 1, 1, 0, false, 1, GELU, "normalization");
                blk.pw2 = load(W, q + ".channel_conv2", b.cin * 2, b.cout, 1, 1, 0, false, 1, NONE, "normalization");
                stages.back().push_back(std::move(blk));
            }
        }
        const int chans[4] = {s1, s2, s3, s4};
        for (int i = 0; i < 4; ++i) {
            const std::string q = "model.neck.insert_conv." + std::to_string(i);
            in_conv.push_back(load(W, q + ".in_conv", chans[i], neck, 1, 1, 0, false, 1));
            SE se;
            se.reduce = load(W, q + ".squeeze_excitation_block.conv1", neck, neck / 4, 1, 1, 0, true, 1);
            se.expand = load(W, q + ".squeeze_excitation_block.conv2", neck / 4, neck, 1, 1, 0, true, 1);
            se.alpha = 0.2f;
            se.residual = true;
            insert_se.push_back(se);
            const std::string r = "model.neck.input_conv." + std::to_string(i);
            dw.push_back(load(W, r + ".depthwise_convolution", neck, neck, k, 1, k / 2, true, neck));
            pw.push_back(load(W, r + ".pointwise_convolution", neck, neck / 4, 1, 1, 0, false, 1));
            SE se2;
            se2.reduce = load(W, r + ".squeeze_excitation_module.conv1", neck / 4, neck / 16, 1, 1, 0, true, 1);
            se2.expand = load(W, r + ".squeeze_excitation_module.conv2", neck / 16, neck / 4, 1, 1, 0, true, 1);
            se2.alpha = 0.2f;
            se2.residual = true;
            input_se.push_back(se2);
        }
        hidden = neck / 4;
        down = load(W, "head.conv_down", neck, hidden, 3, 1, 1, false, 1, RELU, "norm");
        // ConvT 2x2 with its BN folded over the output axis (src/cpu/model.rs:1440-1477).
        up_w = W.get("head.conv_up.convolution.weight", (size_t)hidden * hidden * 4);
        up_b = W.get("head.conv_up.convolution.bias", hidden);
        const auto g = W.get("head.conv_up.norm.weight", hidden), be = W.get("head.conv_up.norm.bias", hidden),
                   m = W.get("head.conv_up.norm.running_mean", hidden), v = W.get("head.conv_up.norm.running_var", hidden);
        for (int o = 0; o < hidden; ++o) {
            const float scale = g[o] / std::sqrt(v[o] + 1e-5f);
            for (int i = 0; i < hidden; ++i)
                for (int t = 0; t < 4; ++t) up_w[((size_t)i * hidden + o) * 4 + t] *= scale;
            up_b[o] = (up_b[o] - m[o]) * scale + be[o];
        }
        fin_w = W.get("head.conv_final.weight", (size_t)hidden * 4);
        fin_b = W.get("head.conv_final.bias", 1)[0];
    }

    // ConvTranspose 2x2 stride 2, IOHW weight [ci][co][2][2]
    static T conv_t(const T& x, const std::vector<float>& w, const std::vector<float>& b, int co, bool relu) {
        T y(co, x.h * 2, x.w * 2);
        for (int o = 0; o < co; ++o) {
            float* yo = y.ch(o);
            for (size_t p = 0; p < y.d.size() / co; ++p) yo[p] = b[o];
            for (int i = 0; i < x.c; ++i) {
                const float* xi = x.ch(i);
                for (int ky = 0; ky < 2; ++ky)
                    for (int kx = 0; kx < 2; ++kx) {
                        const float wv = w[(((size_t)i * co + o) * 2 + ky) * 2 + kx];
                        for (int yy = 0; yy < x.h; ++yy) {
                            float* yr = yo + (size_t)(2 * yy + ky) * y.w + kx;
                            const float* xr = xi + (size_t)yy * x.w;
                            for (int xx = 0; xx < x.w; ++xx) yr[2 * xx] += wv * xr[xx];
                        }
                    }
            }
        }
        if (relu)
            for (auto& v : y.d) v = v > 0.f ? v : 0.f;
        return y;
    }

    void forward(const float* img, int h, int w, float* prob) const {
        T x(3, h, w);
        std::memcpy(x.d.data(), img, x.d.size() * 4);
        T e = conv(stem1, x);
        T br = conv(stem2b, conv(stem2a, e));
        T pooled = max_pool_same_upper(e);
        T s = conv(stem4, conv(stem3, cat({&pooled, &br})));
        std::vector<T> feats;
        for (auto& stage : stages) {
            for (auto& blk : stage) s = blk(s);
            feats.push_back(s);
        }
        std::vector<T> fused(4);
        for (int i = 0; i < 4; ++i) fused[i] = insert_se[i](conv(in_conv[i], feats[i]));
        for (int i = 2; i >= 0; --i) {
            T u = upsample(fused[i + 1], 2);
            for (size_t k = 0; k < fused[i].d.size(); ++k) fused[i].d[k] += u.d[k];
        }
        std::vector<T> f(4);
        for (int i = 0; i < 4; ++i) f[i] = input_se[i](conv(pw[i], conv(dw[i], fused[i])));
        T u3 = upsample(f[3], 8), u2 = upsample(f[2], 4), u1 = upsample(f[1], 2);
        T neck = cat({&u3, &u2, &u1, &f[0]});
        T hd = conv(down, neck);
        T up = conv_t(hd, up_w, up_b, hidden, true);
        T fin = conv_t(up, fin_w, std::vector<float>(1, fin_b), 1, false);
        for (size_t p = 0; p < fin.d.size(); ++p) prob[p] = 1.f / (1.f + std::exp(-fin.d[p]));
    }
};

thread_local std::string g_error;

}  // namespace

extern "C" {

const char* cpu_det_error() { return g_error.c_str(); }

// size: 0 tiny, 1 small.  Returns 0 on success.
int cpu_det_load(const char* path, int size, void** out) {
    try {
        Weights w(path);
        *out = new Detector(w, size);
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

void cpu_det_free(void* det) { delete static_cast<Detector*>(det); }

// x: [n][3][h][w] F32, prob: [n][h][w].  Images run on up to `threads` threads.
int cpu_det_forward(void* det, const float* x, int n, int h, int w, float* prob, int threads) {
    try {
        const Detector* d = static_cast<const Detector*>(det);
        const size_t in = (size_t)3 * h * w, out = (size_t)h * w;
        int failed = 0;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : omp_get_max_threads())
        for (int i = 0; i < n; ++i) {
            try {
                d->forward(x + i * in, h, w, prob + i * out);
            } catch (...) {
#pragma omp atomic write
                failed = 1;
            }
        }
        if (failed) throw std::runtime_error("forward failed");
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return 1;
    }
}

}  // extern "C"
