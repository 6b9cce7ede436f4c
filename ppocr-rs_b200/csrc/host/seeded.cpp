// Seeded random-init checkpoints in the reference's tensor layout, for the
// bench CLI's --seed-weights (the real PP-OCRv6 weights are downloaded by the
// reference, src/models.rs:200-222, which this build cannot do offline).
// The tensor list comes from running the model builder against a recording
// SafeTensors; the values follow the benchmark configs' distributions.
#include <cmath>
#include <cstring>
#include <fstream>
#include <sstream>

#include "common.hpp"
#include "models.hpp"
#include "safetensors.hpp"

namespace ppocr {
namespace {

uint32_t crc32(const std::string& s) {
    uint32_t c = 0xFFFFFFFFu;
    for (unsigned char ch : s) {
        c ^= ch;
        for (int k = 0; k < 8; ++k) c = (c >> 1) ^ (0xEDB88320u & (0u - (c & 1u)));
    }
    return ~c;
}

// splitmix64 stream with Box-Muller normals.
class Rng {
public:
    Rng(uint64_t seed, uint32_t salt) : s_(seed * 0x9E3779B97F4A7C15ull ^ ((uint64_t)salt << 1 | 1)) {}
    uint64_t next() {
        uint64_t z = (s_ += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double uniform() { return ((next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }   // (0, 1)
    double normal() {
        if (have_) { have_ = false; return spare_; }
        const double r = std::sqrt(-2.0 * std::log(uniform())), t = 6.283185307179586 * uniform();
        spare_ = r * std::sin(t);
        have_ = true;
        return r * std::cos(t);
    }

private:
    uint64_t s_;
    double spare_ = 0;
    bool have_ = false;
};

bool ends_with(const std::string& s, const char* suffix) {
    const size_t n = std::strlen(suffix);
    return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

std::vector<float> draw(const std::string& name, const std::vector<size_t>& shape, bool detector, uint64_t seed) {
    size_t count = 1;
    for (size_t d : shape) count *= d;
    std::vector<float> v(count, 0.f);
    if (ends_with(name, ".running_var")) {
        std::fill(v.begin(), v.end(), 1.f);
        return v;
    }
    if (ends_with(name, ".running_mean")) return v;
    if (shape.size() == 1) {
        // Batch-norm gamma and layer-norm weight are the only 1-D weights; every
        // 1-D bias (conv, linear, batch-norm beta, layer-norm bias) is 0.
        if (ends_with(name, ".weight")) std::fill(v.begin(), v.end(), 1.f);
        return v;
    }
    Rng rng(seed, crc32(name));
    const bool rank_one = detector && shape.size() == 4 && shape[2] == 9 && shape[3] == 9 &&
                          (name.find("input_feature_projection_convolution") != std::string::npos ||
                           name.find("path_aggregation_lateral_convolution") != std::string::npos);
    if (rank_one) {
        const size_t o_n = shape[0], i_n = shape[1], taps = 81;
        std::vector<double> d(i_n * taps);
        for (size_t i = 0; i < i_n; ++i) {
            double norm = 0;
            for (size_t t = 0; t < taps; ++t) { d[i * taps + t] = rng.normal(); norm += d[i * taps + t] * d[i * taps + t]; }
            norm = std::sqrt(norm);
            for (size_t t = 0; t < taps; ++t) d[i * taps + t] /= norm;
        }
        const double sd = std::sqrt(2.0 / (double)(i_n * taps)) * 9.0;
        for (size_t o = 0; o < o_n; ++o)
            for (size_t i = 0; i < i_n; ++i) {
                const double p = rng.normal() * sd;
                for (size_t t = 0; t < taps; ++t) v[(o * i_n + i) * taps + t] = (float)(p * d[i * taps + t]);
            }
        return v;
    }
    double sd = 0.02;
    if (detector) {
        // Transposed convs (IOHW) take fan_in = input channels x taps.
        const bool transposed = name == "head.conv_up.convolution.weight" || name == "head.conv_final.weight";
        size_t fan_in = 1;
        for (size_t k = 1; k < shape.size(); ++k) fan_in *= shape[k];
        if (transposed) fan_in = shape[0] * shape[2] * shape[3];
        sd = std::sqrt(2.0 / (double)std::max<size_t>(fan_in, 1));
    }
    for (auto& x : v) x = (float)(rng.normal() * sd);
    return v;
}

}  // namespace

void write_seeded_weights(const std::string& path, bool detector, int size, uint64_t seed) {
    SafeTensors rec = SafeTensors::recorder();
    const size_t shape[4] = {1, 3, detector ? (size_t)64 : (size_t)48, 64};
    if (detector) build_detector(rec, size, shape, DT_F32, TC_NONE);
    else build_recognizer(rec, size, shape, DT_F32, TC_NONE);
    std::ostringstream head;
    head << "{\"__metadata__\":{\"format\":\"pt\"}";
    size_t off = 0;
    std::vector<std::vector<float>> values;
    for (const auto& kv : rec.requested()) {
        values.push_back(draw(kv.first, kv.second, detector, seed));
        const size_t bytes = values.back().size() * 4;
        head << ",\"" << kv.first << "\":{\"dtype\":\"F32\",\"shape\":[";
        for (size_t k = 0; k < kv.second.size(); ++k) head << (k ? "," : "") << kv.second[k];
        head << "],\"data_offsets\":[" << off << "," << off + bytes << "]}";
        off += bytes;
    }
    head << "}";
    std::string h = head.str();
    while (h.size() % 8) h.push_back(' ');
    std::ofstream f(path, std::ios::binary);
    if (!f) fail(PPOCR_ERR_READ_FILE, "write " + path);
    const uint64_t n = h.size();
    unsigned char len[8];
    for (int k = 0; k < 8; ++k) len[k] = (unsigned char)(n >> (8 * k));
    f.write(reinterpret_cast<const char*>(len), 8);
    f.write(h.data(), (std::streamsize)h.size());
    for (const auto& v : values) f.write(reinterpret_cast<const char*>(v.data()), (std::streamsize)(v.size() * 4));
    if (!f) fail(PPOCR_ERR_READ_FILE, "write " + path);
}

}  // namespace ppocr
