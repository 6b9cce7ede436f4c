// Host steps of the end-to-end pipeline (ppocr-rs src/ocr.rs); see pipeline.hpp.
#include "pipeline.hpp"

#include <algorithm>
#include <charconv>
#include <cmath>
#include <cstring>
#include <deque>
#include <limits>

#include "common.hpp"
#include "ppocr_b200.h"

namespace ppocr {
namespace {

constexpr float kMaxRectifiedEdge = 4096.f;
constexpr float kMaxRectifiedPixels = 8000000.f;
constexpr size_t kRecognizerBatch = 6;
constexpr size_t kRecognizerWidth = 320;
constexpr size_t kRecognizerHeight = 48;
constexpr float kProbabilityEpsilon = 1e-8f;

// f32::total_cmp as an integer key.
int32_t total_key(float v) {
    int32_t b;
    std::memcpy(&b, &v, 4);
    return b < 0 ? (b ^ 0x7fffffff) : b;
}
bool total_less(float a, float b) { return total_key(a) < total_key(b); }

float sum4(const float (&v)[4]) {
    float s = -0.f;
    for (float x : v) s = s + x;
    return s;
}

Pt polygon_center(const Pt (&p)[4]) {
    const float xs[4] = {p[0].x, p[1].x, p[2].x, p[3].x}, ys[4] = {p[0].y, p[1].y, p[2].y, p[3].y};
    return Pt{sum4(xs) / 4.f, sum4(ys) / 4.f};
}

float distance(Pt a, Pt b) {
    const float dx = a.x - b.x, dy = a.y - b.y;
    return std::sqrt(dx * dx + dy * dy);
}

struct Component {
    std::vector<Pt> points;
    double score_sum = 0.0;
};

// collect_component (src/ocr.rs:993-1043): breadth-first, 8 neighbours in a fixed order.
void collect_component(const float* values, size_t out_w, size_t cw, size_t ch, size_t sx, size_t sy, float thr,
                       std::vector<uint8_t>& visited, Component& comp, std::deque<std::pair<size_t, size_t>>& queue) {
    static const int kNeighbors[8][2] = {{-1, -1}, {0, -1}, {1, -1}, {-1, 0}, {1, 0}, {-1, 1}, {0, 1}, {1, 1}};
    comp.points.clear();
    comp.score_sum = 0.0;
    queue.clear();
    queue.emplace_back(sx, sy);
    visited[sy * cw + sx] = 1;
    while (!queue.empty()) {
        const auto [x, y] = queue.front();
        queue.pop_front();
        comp.points.push_back(Pt{(float)x + 0.5f, (float)y + 0.5f});
        comp.score_sum += (double)values[y * out_w + x];
        for (const auto& d : kNeighbors) {
            const long long nx = (long long)x + d[0], ny = (long long)y + d[1];
            if (nx < 0 || ny < 0 || nx >= (long long)cw || ny >= (long long)ch) continue;
            const size_t ni = (size_t)ny * cw + (size_t)nx;
            if (!visited[ni] && values[(size_t)ny * out_w + (size_t)nx] >= thr) {
                visited[ni] = 1;
                queue.emplace_back((size_t)nx, (size_t)ny);
            }
        }
    }
}

// fit_rotated_box (src/ocr.rs:1045-1113), f32 in the reference's order.
void fit_rotated_box(const std::vector<Pt>& pts, float unclip, Pt (&out)[4]) {
    const float count = (float)pts.size();
    float sx = -0.f, sy = -0.f;
    for (const Pt& p : pts) sx = sx + p.x;
    for (const Pt& p : pts) sy = sy + p.y;
    Pt c{sx / count, sy / count};
    float cxx = 0.f, cxy = 0.f, cyy = 0.f;
    for (const Pt& p : pts) {
        const float dx = p.x - c.x, dy = p.y - c.y;
        cxx = cxx + dx * dx;
        cxy = cxy + dx * dy;
        cyy = cyy + dy * dy;
    }
    const float angle = 0.5f * std::atan2(2.f * cxy, cxx - cyy);
    Pt axis{std::cos(angle), std::sin(angle)};
    if (axis.x < 0.f || (std::fabs(axis.x) < std::numeric_limits<float>::epsilon() && axis.y < 0.f))
        axis = Pt{-axis.x, -axis.y};
    const Pt normal{-axis.y, axis.x};
    float min_a = INFINITY, max_a = -INFINITY, min_n = INFINITY, max_n = -INFINITY;
    for (const Pt& p : pts) {
        const Pt d{p.x - c.x, p.y - c.y};
        const float along_a = d.x * axis.x + d.y * axis.y;
        const float along_n = d.x * normal.x + d.y * normal.y;
        min_a = std::fmin(min_a, along_a);
        max_a = std::fmax(max_a, along_a);
        min_n = std::fmin(min_n, along_n);
        max_n = std::fmax(max_n, along_n);
    }
    const float axis_center = (min_a + max_a) * 0.5f;
    const float normal_center = (min_n + max_n) * 0.5f;
    const float half_a = ((max_a - min_a + 1.f) * unclip) * 0.5f;
    const float half_n = ((max_n - min_n + 1.f) * unclip) * 0.5f;
    const Pt off{axis.x * axis_center + normal.x * normal_center, axis.y * axis_center + normal.y * normal_center};
    c = Pt{c.x + off.x, c.y + off.y};
    const float sa[4] = {-1.f, 1.f, 1.f, -1.f}, sn[4] = {-1.f, -1.f, 1.f, 1.f};
    for (int i = 0; i < 4; ++i) {
        const float a = sa[i] * half_a, n = sn[i] * half_n;
        const Pt d{axis.x * a + normal.x * n, axis.y * a + normal.y * n};
        out[i] = Pt{c.x + d.x, c.y + d.y};
    }
}

float map_to_source(float v, uint32_t source, uint32_t content) {
    const float m = v * (float)source / (float)content;
    return std::min(std::max(m, 0.f), (float)source);
}

void sort_detections(std::vector<Detection>& d) {
    std::stable_sort(d.begin(), d.end(), [](const Detection& l, const Detection& r) {
        const Pt lc = polygon_center(l.poly), rc = polygon_center(r.poly);
        if (total_key(lc.y) != total_key(rc.y)) return total_less(lc.y, rc.y);
        if (total_key(lc.x) != total_key(rc.x)) return total_less(lc.x, rc.x);
        return total_less(l.score, r.score);
    });
}

void crop_size(const Pt (&p)[4], float* w, float* h) {
    *w = std::max(distance(p[0], p[1]), distance(p[3], p[2]));
    *h = std::max(distance(p[0], p[3]), distance(p[1], p[2]));
}

float round_half_away(float v) { return std::round(v); }

void bounded_crop_dimensions(float width, float height, uint32_t* w, uint32_t* h) {
    if (!std::isfinite(width) || !std::isfinite(height) || width <= 0.f || height <= 0.f)
        fail(PPOCR_ERR_INVALID_INPUT, "text polygon has an invalid crop size " + std::to_string(width) + " by " +
                                          std::to_string(height));
    const float edge = std::min(kMaxRectifiedEdge / std::max(width, height), 1.f);
    const float pixel = std::min(std::sqrt(kMaxRectifiedPixels / (width * height)), 1.f);
    const float s = std::min(edge, pixel);
    *w = (uint32_t)std::min(std::max(round_half_away(width * s), 1.f), kMaxRectifiedEdge);
    *h = (uint32_t)std::min(std::max(round_half_away(height * s), 1.f), kMaxRectifiedEdge);
}

bool is_ascii_space(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\v' || c == '\f'; }

std::string trim_start(const std::string& s) {
    size_t i = 0;
    while (i < s.size() && is_ascii_space(s[i])) ++i;
    return s.substr(i);
}

std::string trim(const std::string& s) {
    std::string t = trim_start(s);
    size_t e = t.size();
    while (e > 0 && is_ascii_space(t[e - 1])) --e;
    return t.substr(0, e);
}

// str::lines: split at "\n" (a preceding "\r" belongs to the ending), no final empty line.
std::vector<std::string> rust_lines(const std::string& s) {
    std::vector<std::string> out;
    size_t start = 0;
    while (start < s.size()) {
        size_t nl = s.find('\n', start);
        std::string line = s.substr(start, nl == std::string::npos ? std::string::npos : nl - start);
        if (nl != std::string::npos && !line.empty() && line.back() == '\r') line.pop_back();
        out.push_back(line);
        if (nl == std::string::npos) break;
        start = nl + 1;
    }
    return out;
}

std::string strip_cr(const std::string& s) { return (!s.empty() && s.back() == '\r') ? s.substr(0, s.size() - 1) : s; }

std::string parse_yaml_scalar(const std::string& v, size_t line) {
    if (!v.empty() && v[0] == '\'') {
        if (v.size() < 2 || v.back() != '\'')
            fail(PPOCR_ERR_INVALID_INPUT, "unterminated single-quoted character on line " + std::to_string(line));
        std::string inner = v.substr(1, v.size() - 2), out;
        for (size_t i = 0; i < inner.size(); ++i) {
            out += inner[i];
            if (inner[i] == '\'' && i + 1 < inner.size() && inner[i + 1] == '\'') ++i;
        }
        return out;
    }
    if (!v.empty() && v[0] == '"') {
        if (v.size() < 2 || v.back() != '"')
            fail(PPOCR_ERR_INVALID_INPUT, "unterminated double-quoted character on line " + std::to_string(line));
        return v.substr(1, v.size() - 2);
    }
    return v;
}

bool parse_paddlex(const std::string& contents, std::vector<std::string>& entries) {
    const std::vector<std::string> lines = rust_lines(contents);
    for (size_t index = 0; index < lines.size(); ++index) {
        const std::string& line = lines[index];
        if (trim(line) != "character_dict:") continue;
        const size_t indentation = line.size() - trim_start(line).size();
        for (size_t j = index + 1; j < lines.size(); ++j) {
            const std::string entry = strip_cr(lines[j]);
            if (trim(entry).empty()) continue;
            const std::string trimmed = trim_start(entry);
            if (trimmed.compare(0, 2, "- ") != 0) {
                if (entry.size() - trimmed.size() <= indentation) break;
                fail(PPOCR_ERR_INVALID_INPUT, "expected a character list entry on line " + std::to_string(j + 1));
            }
            entries.push_back(parse_yaml_scalar(trimmed.substr(2), j + 1));
        }
        return true;
    }
    return false;
}

// Unicode scalar values of a UTF-8 string (invalid bytes pass through one by one).
std::vector<uint32_t> code_points(const std::string& s) {
    std::vector<uint32_t> out;
    for (size_t i = 0; i < s.size();) {
        const unsigned char c = (unsigned char)s[i];
        int n = c < 0x80 ? 1 : (c >> 5) == 6 ? 2 : (c >> 4) == 14 ? 3 : (c >> 3) == 30 ? 4 : 1;
        if (i + n > s.size()) n = 1;
        uint32_t cp = n == 1 ? c : n == 2 ? (c & 0x1f) : n == 3 ? (c & 0x0f) : (c & 0x07);
        for (int k = 1; k < n; ++k) cp = (cp << 6) | ((unsigned char)s[i + k] & 0x3f);
        out.push_back(cp);
        i += n;
    }
    return out;
}

void append_utf8(std::string& s, uint32_t cp) {
    if (cp < 0x80) {
        s += (char)cp;
    } else if (cp < 0x800) {
        s += (char)(0xc0 | (cp >> 6));
        s += (char)(0x80 | (cp & 0x3f));
    } else if (cp < 0x10000) {
        s += (char)(0xe0 | (cp >> 12));
        s += (char)(0x80 | ((cp >> 6) & 0x3f));
        s += (char)(0x80 | (cp & 0x3f));
    } else {
        s += (char)(0xf0 | (cp >> 18));
        s += (char)(0x80 | ((cp >> 12) & 0x3f));
        s += (char)(0x80 | ((cp >> 6) & 0x3f));
        s += (char)(0x80 | (cp & 0x3f));
    }
}

size_t append_with_overlap(std::string& target, const std::string& next) {
    if (next.empty()) return 0;
    const std::vector<uint32_t> n = code_points(next);
    if (target.empty()) {
        target = next;
        return n.size();
    }
    const std::vector<uint32_t> t = code_points(target);
    const size_t maximum = std::min(std::min(t.size(), n.size()), (size_t)32);
    size_t overlap = 0;
    for (size_t size = maximum; size >= 1; --size) {
        if (std::equal(t.end() - size, t.end(), n.begin())) {
            overlap = size;
            break;
        }
    }
    for (size_t i = overlap; i < n.size(); ++i) append_utf8(target, n[i]);
    return n.size() - overlap;
}

void validate_decode(size_t classes, const std::vector<std::string>& dict, size_t content_width, size_t input_width,
                     bool* implicit_space) {
    *implicit_space = classes == dict.size() + 2;
    if (classes != dict.size() + 1 && !*implicit_space)
        fail(PPOCR_ERR_INVALID_INPUT, "recognizer output has " + std::to_string(classes) + " classes, but the dictionary has " +
                                          std::to_string(dict.size()) +
                                          " entries; expected dictionary entries plus the CTC blank class");
    if (content_width == 0 || content_width > input_width)
        fail(PPOCR_ERR_INVALID_INPUT, "recognizer content width " + std::to_string(content_width) + " is outside 1..=" +
                                          std::to_string(input_width));
}

size_t valid_steps(size_t content_width, size_t steps, size_t input_width) {
    size_t v = (content_width * steps + input_width - 1) / input_width;
    return std::min(std::max(v, (size_t)1), steps);
}

float row_probability(const float* row, size_t n, float value) {
    float sum = -0.f;
    bool nonneg = true;
    for (size_t i = 0; i < n; ++i) {
        sum = sum + row[i];
        nonneg = nonneg && row[i] >= 0.f;
    }
    if (nonneg && std::fabs(sum - 1.f) <= 0.01f) return std::min(std::max(value, 0.f), 1.f);
    float maximum = -INFINITY;
    for (size_t i = 0; i < n; ++i) maximum = std::fmax(maximum, row[i]);
    float denom = -0.f;
    for (size_t i = 0; i < n; ++i) denom = denom + std::exp(row[i] - maximum);
    return std::min(std::max(std::exp(value - maximum) / denom, 0.f), 1.f);
}

Decoded finish_decode(std::string text, double log_score, size_t emitted) {
    Decoded d;
    d.text = std::move(text);
    d.score = emitted == 0 ? 0.f : (float)std::exp(log_score / (double)emitted);
    return d;
}

// Shortest round-trip decimal of an f32, in the layout of the reference's JSON
// writer: integral values keep a ".0"; very large or small magnitudes use an
// exponent.
std::string json_float(float v) {
    if (!std::isfinite(v)) return "null";
    char buf[64];
    auto res = std::to_chars(buf, buf + sizeof(buf), v, std::chars_format::scientific);
    std::string sci(buf, res.ptr);   // d[.ddd]e[+-]XX
    const size_t e = sci.find('e');
    std::string mant = sci.substr(0, e);
    const int exp10 = std::stoi(sci.substr(e + 1));
    bool neg = false;
    if (!mant.empty() && mant[0] == '-') {
        neg = true;
        mant = mant.substr(1);
    }
    std::string digits;
    for (char ch : mant)
        if (ch != '.') digits += ch;
    const int length = (int)digits.size();
    const int kk = exp10 + 1;   // 10^(kk-1) <= |v| < 10^kk
    std::string out = neg ? "-" : "";
    if (kk >= length && kk <= 13) {
        out += digits + std::string(kk - length, '0') + ".0";
    } else if (kk > 0 && kk <= 13) {
        out += digits.substr(0, kk) + "." + digits.substr(kk);
    } else if (kk > -6 && kk <= 0) {
        out += "0." + std::string(-kk, '0') + digits;
    } else if (length == 1) {
        out += digits + "e" + std::to_string(kk - 1);
    } else {
        out += digits.substr(0, 1) + "." + digits.substr(1) + "e" + std::to_string(kk - 1);
    }
    return out;
}

std::string json_string(const std::string& s) {
    std::string out = "\"";
    for (unsigned char c : s) {
        switch (c) {
            case '"': out += "\\\""; break;
            case '\\': out += "\\\\"; break;
            case '\n': out += "\\n"; break;
            case '\r': out += "\\r"; break;
            case '\t': out += "\\t"; break;
            case 0x08: out += "\\b"; break;
            case 0x0c: out += "\\f"; break;
            default:
                if (c < 0x20) {
                    char b[8];
                    std::snprintf(b, sizeof(b), "\\u%04x", c);
                    out += b;
                } else {
                    out += (char)c;
                }
        }
    }
    return out + "\"";
}

}  // namespace

void PostOptions::validate() const {
    auto prob = [](float v, const char* name) {
        if (!std::isfinite(v) || v < 0.f || v > 1.f)
            fail(PPOCR_ERR_INVALID_INPUT, std::string(name) + " must be a finite value between zero and one");
    };
    prob(binary_threshold, "detector binary threshold");
    prob(box_threshold, "detector box threshold");
    if (min_area == 0) fail(PPOCR_ERR_INVALID_INPUT, "detector minimum area must be at least one pixel");
    if (max_boxes == 0) fail(PPOCR_ERR_INVALID_INPUT, "detector maximum box count must be at least one");
    if (!std::isfinite(unclip_ratio) || unclip_ratio <= 0.f)
        fail(PPOCR_ERR_INVALID_INPUT, "detector unclip ratio must be a finite value greater than zero");
}

std::vector<Detection> extract_detections(const float* values, size_t height, size_t width, uint32_t source_w,
                                          uint32_t source_h, uint32_t content_w, uint32_t content_h,
                                          const PostOptions& opts) {
    opts.validate();
    if (!values || height == 0 || width == 0) fail(PPOCR_ERR_INVALID_INPUT, "detector output is empty");
    if (source_w == 0 || source_h == 0 || content_w == 0 || content_h == 0)
        fail(PPOCR_ERR_INVALID_INPUT, "detector transform dimensions must be non-zero");
    for (size_t i = 0; i < height * width; ++i)
        if (!std::isfinite(values[i])) fail(PPOCR_ERR_INVALID_INPUT, "detector output contains non-finite values");
    const size_t cw = std::min((size_t)content_w, width), ch = std::min((size_t)content_h, height);
    std::vector<uint8_t> visited(cw * ch, 0);
    std::vector<Detection> dets;
    Component comp;
    std::deque<std::pair<size_t, size_t>> queue;
    const float thr = opts.binary_threshold;
    for (size_t y = 0; y < ch; ++y) {
        for (size_t x = 0; x < cw; ++x) {
            if (visited[y * cw + x] || values[y * width + x] < thr) continue;
            collect_component(values, width, cw, ch, x, y, thr, visited, comp, queue);
            if (comp.points.size() < opts.min_area) continue;
            const float score = (float)(comp.score_sum / (double)comp.points.size());
            if (score < opts.box_threshold) continue;
            Detection d;
            fit_rotated_box(comp.points, opts.unclip_ratio, d.poly);
            for (Pt& p : d.poly) p = Pt{map_to_source(p.x, source_w, content_w), map_to_source(p.y, source_h, content_h)};
            d.score = score;
            dets.push_back(d);
        }
    }
    sort_detections(dets);
    if (dets.size() > opts.max_boxes) {
        std::stable_sort(dets.begin(), dets.end(), [](const Detection& l, const Detection& r) {
            if (total_key(l.score) != total_key(r.score)) return total_less(r.score, l.score);
            const Pt lc = polygon_center(l.poly), rc = polygon_center(r.poly);
            if (total_key(lc.y) != total_key(rc.y)) return total_less(lc.y, rc.y);
            return total_less(lc.x, rc.x);
        });
        dets.resize(opts.max_boxes);
        sort_detections(dets);
    }
    return dets;
}

void detector_input_size(uint32_t width, uint32_t height, uint32_t max_side, uint32_t* in_w, uint32_t* in_h) {
    if (width == 0 || height == 0) fail(PPOCR_ERR_INVALID_INPUT, "image dimensions must be non-zero");
    double ratio;
    const double longest = (double)std::max(width, height);
    if (max_side > 0) {
        ratio = std::min((double)max_side / longest, 1.0);
    } else {
        const double min_side = (double)std::min(width, height);
        ratio = min_side < 736.0 ? 736.0 / min_side : 1.0;
        if (longest * ratio > 4000.0) ratio = 4000.0 / longest;
    }
    auto aligned = [](double v) {
        if (!std::isfinite(v) || v <= 0.0) fail(PPOCR_ERR_INVALID_INPUT, "invalid resized image dimension");
        const double units = std::max(std::round(v / 32.0), 1.0);
        if (units > (double)(UINT32_MAX / 32)) fail(PPOCR_ERR_INVALID_INPUT, "resized image dimension is too large");
        return (uint32_t)units * 32u;
    };
    *in_w = aligned((double)width * ratio);
    *in_h = aligned((double)height * ratio);
}

float polygon_aspect_ratio(const Pt (&poly)[4]) {
    float w, h;
    crop_size(poly, &w, &h);
    return w / std::max(h, std::numeric_limits<float>::epsilon());
}

size_t crop_content_width(const Pt (&poly)[4]) {
    float w, h;
    crop_size(poly, &w, &h);
    uint32_t bw, bh;
    bounded_crop_dimensions(w, h, &bw, &bh);
    const uint64_t scaled = ((uint64_t)kRecognizerHeight * bw + bh - 1) / bh;
    return (size_t)std::max<uint64_t>(scaled, 1);
}

size_t recognizer_batch_width(const std::vector<const Pt*>& polys) {
    size_t maximum = kRecognizerWidth;
    for (const Pt* p : polys) {
        const Pt(&q)[4] = *reinterpret_cast<const Pt(*)[4]>(p);
        maximum = std::max(maximum, crop_content_width(q));
    }
    return (maximum + 3) / 4 * 4;
}

std::vector<RecBatch> recognition_batches(const std::vector<Detection>& dets) {
    std::vector<size_t> order(dets.size());
    for (size_t i = 0; i < order.size(); ++i) order[i] = i;
    std::vector<float> aspect(dets.size());
    for (size_t i = 0; i < dets.size(); ++i) aspect[i] = polygon_aspect_ratio(dets[i].poly);
    std::stable_sort(order.begin(), order.end(), [&](size_t l, size_t r) { return total_less(aspect[l], aspect[r]); });
    std::vector<RecBatch> out;
    for (size_t s = 0; s < order.size(); s += kRecognizerBatch) {
        RecBatch b;
        std::vector<const Pt*> polys;
        for (size_t i = s; i < std::min(order.size(), s + kRecognizerBatch); ++i) {
            b.index.push_back(order[i]);
            polys.push_back(dets[order[i]].poly);
        }
        b.width = recognizer_batch_width(polys);
        for (size_t i : b.index) {
            const size_t c = crop_content_width(dets[i].poly);
            if (c > b.width) fail(PPOCR_ERR_INVALID_INPUT, "recognizer crop exceeds its batch canvas");
            b.content.push_back(c);
        }
        out.push_back(std::move(b));
    }
    return out;
}

std::vector<std::string> parse_dictionary(const std::string& contents) {
    std::vector<std::string> entries;
    if (!parse_paddlex(contents, entries)) {
        for (const std::string& l : rust_lines(contents)) entries.push_back(strip_cr(l));
    }
    if (!entries.empty()) {
        std::string& first = entries[0];
        while (first.compare(0, 3, "\xEF\xBB\xBF") == 0) first = first.substr(3);
    }
    if (entries.empty()) fail(PPOCR_ERR_INVALID_INPUT, "recognition dictionary is empty");
    for (size_t i = 0; i < entries.size(); ++i)
        if (entries[i].empty())
            fail(PPOCR_ERR_INVALID_INPUT, "recognition dictionary contains an empty entry on line " + std::to_string(i + 1));
    return entries;
}

Decoded decode_ctc_rows(const float* probs, size_t steps, size_t classes, const std::vector<std::string>& dict,
                        size_t content_width, size_t input_width) {
    if (steps == 0 || classes < 2) fail(PPOCR_ERR_INVALID_INPUT, "recognizer output shape, expected [1, time, classes>=2]");
    bool implicit_space;
    validate_decode(classes, dict, content_width, input_width, &implicit_space);
    for (size_t i = 0; i < steps * classes; ++i)
        if (!std::isfinite(probs[i])) fail(PPOCR_ERR_INVALID_INPUT, "recognizer output contains non-finite values");
    const size_t valid = valid_steps(content_width, steps, input_width);
    std::string text;
    double log_score = 0.0;
    size_t emitted = 0, previous = 0;
    for (size_t t = 0; t < valid; ++t) {
        const float* row = probs + t * classes;
        size_t cls = 0;
        for (size_t i = 1; i < classes; ++i)
            if (!total_less(row[i], row[cls])) cls = i;   // max_by keeps the last of equal maxima
        if (cls != 0 && cls != previous) {
            text += (implicit_space && cls == classes - 1) ? std::string(" ") : dict[cls - 1];
            log_score += std::log((double)std::max(row_probability(row, classes, row[cls]), kProbabilityEpsilon));
            ++emitted;
        }
        previous = cls;
    }
    return finish_decode(std::move(text), log_score, emitted);
}

Decoded decode_ctc_steps(const int32_t* index, const float* prob, size_t steps, size_t classes,
                         const std::vector<std::string>& dict, size_t content_width, size_t input_width) {
    if (steps == 0 || classes < 2) fail(PPOCR_ERR_INVALID_INPUT, "recognizer output shape, expected [1, time, classes>=2]");
    bool implicit_space;
    validate_decode(classes, dict, content_width, input_width, &implicit_space);
    const size_t valid = valid_steps(content_width, steps, input_width);
    std::string text;
    double log_score = 0.0;
    size_t emitted = 0, previous = 0;
    for (size_t t = 0; t < valid; ++t) {
        if (index[t] < 0 || (size_t)index[t] >= classes || !std::isfinite(prob[t]))
            fail(PPOCR_ERR_INVALID_INPUT, "recognizer output contains non-finite values");
        const size_t cls = (size_t)index[t];
        if (cls != 0 && cls != previous) {
            text += (implicit_space && cls == classes - 1) ? std::string(" ") : dict[cls - 1];
            const float p = std::min(std::max(prob[t], 0.f), 1.f);
            log_score += std::log((double)std::max(p, kProbabilityEpsilon));
            ++emitted;
        }
        previous = cls;
    }
    return finish_decode(std::move(text), log_score, emitted);
}

Decoded join_decoded_texts(const std::vector<Decoded>& parts) {
    Decoded out;
    double score_sum = 0.0;
    size_t weight = 0;
    for (const Decoded& p : parts) {
        const size_t added = append_with_overlap(out.text, p.text);
        if (added != 0) {
            score_sum += (double)p.score * (double)added;
            weight += added;
        }
    }
    out.score = weight == 0 ? 0.f : (float)(score_sum / (double)weight);
    return out;
}

std::string result_json(const OcrResult& r) {
    std::string s = "{\n";
    s += "  \"source_size\": [\n    " + std::to_string(r.source_w) + ",\n    " + std::to_string(r.source_h) + "\n  ],\n";
    s += "  \"detector_input_size\": [\n    " + std::to_string(r.input_w) + ",\n    " + std::to_string(r.input_h) +
         "\n  ],\n";
    if (r.lines.empty()) {
        s += "  \"lines\": []\n}";
        return s;
    }
    s += "  \"lines\": [\n";
    for (size_t i = 0; i < r.lines.size(); ++i) {
        const OcrLine& l = r.lines[i];
        s += "    {\n      \"polygon\": [\n";
        for (int k = 0; k < 4; ++k) {
            s += "        [\n          " + json_float(l.poly[k].x) + ",\n          " + json_float(l.poly[k].y) + "\n        ]";
            s += k < 3 ? ",\n" : "\n";
        }
        s += "      ],\n";
        s += "      \"detection_score\": " + json_float(l.detection_score) + ",\n";
        s += "      \"text\": " + json_string(l.text) + ",\n";
        s += "      \"recognition_score\": " + json_float(l.recognition_score) + "\n    }";
        s += i + 1 < r.lines.size() ? ",\n" : "\n";
    }
    s += "  ]\n}";
    return s;
}

std::string result_text(const OcrResult& r) {
    std::string s;
    bool first = true;
    for (const OcrLine& l : r.lines) {
        if (l.text.empty()) continue;
        if (!first) s += "\n";
        s += l.text;
        first = false;
    }
    return s;
}

}  // namespace ppocr
