// ppocr-gpu-bench: the reference's benchmark CLI contract
// (ppocr-rs src/bin/ppocr-gpu-bench.rs:45-88, src/bin/benchmark.rs:13-320)
// over the C ABI.  Same flags, deterministic input, F32 reference / dump files
// and report keys; adds --batch, --precision and --no-graph.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "ppocr_b200.h"

namespace {

[[noreturn]] void die(const std::string& m) {
    std::fprintf(stderr, "Error: %s\n", m.c_str());
    std::exit(1);
}

void check(int status, const char* what) {
    if (status != PPOCR_OK) die(std::string(what) + ": " + ppocr_last_error());
}

struct Args {
    std::string kind, model_size = "tiny", model, input, reference, dump, precision = "fp32";
    long height = -1, width = -1, warmup = 5, runs = 30, batch = 1;
    bool graph = true;
};

Args parse(int argc, char** argv) {
    Args a;
    for (int i = 1; i < argc; ++i) {
        std::string k = argv[i];
        auto val = [&]() -> std::string {
            if (i + 1 >= argc) die("missing value for " + k);
            return argv[++i];
        };
        if (k == "--kind") a.kind = val();
        else if (k == "--model-size") a.model_size = val();
        else if (k == "--model") a.model = val();
        else if (k == "--model-dir") val();
        else if (k == "--offline" || k == "--verify-models") {}
        else if (k == "--height") a.height = std::stol(val());
        else if (k == "--width") a.width = std::stol(val());
        else if (k == "--input") a.input = val();
        else if (k == "--reference") a.reference = val();
        else if (k == "--dump") a.dump = val();
        else if (k == "--warmup") a.warmup = std::stol(val());
        else if (k == "--runs") a.runs = std::stol(val());
        else if (k == "--batch") a.batch = std::stol(val());
        else if (k == "--precision") a.precision = val();
        else if (k == "--no-graph") a.graph = false;
        else if (k == "-h" || k == "--help") {
            std::printf("usage: ppocr-gpu-bench --kind det|rec --model FILE [--model-size tiny|small|medium] [--height H] "
                        "[--width W] [--input F32] [--reference F32] [--dump F32] [--warmup 5] [--runs 30] [--batch 1] "
                        "[--precision fp32|bf16] [--no-graph]\n");
            std::exit(0);
        } else die("unknown argument " + k);
    }
    if (a.kind != "det" && a.kind != "rec") die("--kind must be det or rec");
    if (a.model.empty()) die("the pinned model store is not part of this build; pass --model FILE");
    if (a.runs <= 0) die("--runs must be positive");
    return a;
}

// benchmark.rs:126-134
std::vector<float> deterministic_input(size_t n) {
    std::vector<float> v(n);
    uint32_t state = 0x243f6a88u;
    for (size_t i = 0; i < n; ++i) {
        state = state * 1664525u + 1013904223u;
        v[i] = ((float)(state >> 8) / (float)0x00ffffff) * 2.0f - 1.0f;
    }
    return v;
}

std::vector<float> read_f32(const std::string& path, size_t expected) {
    std::ifstream f(path, std::ios::binary);
    if (!f) die("read " + path);
    std::vector<char> b((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    if (b.size() != expected * 4)
        die(path + " must contain " + std::to_string(expected) + " F32 values, found " + std::to_string(b.size()) + " bytes");
    std::vector<float> v(expected);
    std::memcpy(v.data(), b.data(), b.size());
    return v;
}

size_t argmax(const float* v, size_t n) {
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (v[i] >= v[best]) best = i;   // last maximum wins, as Iterator::max_by
    return best;
}

double percentile(const std::vector<double>& sorted, double p) {
    return sorted[(size_t)std::llround((sorted.size() - 1) * p)];
}

}  // namespace

int main(int argc, char** argv) {
    Args a = parse(argc, argv);
    const bool det = a.kind == "det";
    const size_t h = a.height > 0 ? (size_t)a.height : det ? 416 : 48;
    const size_t w = a.width > 0 ? (size_t)a.width : det ? 736 : 320;
    const size_t shape[4] = {(size_t)a.batch, 3, h, w};
    const size_t count = shape[0] * 3 * h * w;
    std::vector<float> input = a.input.empty() ? deterministic_input(count) : read_f32(a.input, count);
    int size = a.model_size == "medium" ? PPOCR_MEDIUM : a.model_size == "small" ? PPOCR_SMALL : a.model_size == "tiny" ? PPOCR_TINY : -1;
    if (size < 0) die("unknown --model-size " + a.model_size);

    ppocr_gpu* gpu = nullptr;
    check(ppocr_gpu_create(0, &gpu), "create GPU");
    ppocr_load_options o;
    ppocr_load_options_default(&o);
    o.precision = a.precision == "bf16" ? PPOCR_PRECISION_BF16 : a.precision == "fp32tc" ? PPOCR_PRECISION_FP32_TC : PPOCR_PRECISION_FP32;
    o.use_graph = a.graph ? 1 : 0;
    ppocr_model* model = nullptr;
    if (det) check(ppocr_detector_load_ex(gpu, a.model.c_str(), size, shape, &o, &model), "load detector");
    else check(ppocr_recognizer_load_ex(gpu, a.model.c_str(), size, shape, &o, nullptr, &model), "load recognizer");
    size_t out_shape[4], rank = 0, elements = 0;
    check(ppocr_model_output_shape(model, out_shape, &rank, &elements), "output shape");
    std::vector<float> out(elements);
    check(ppocr_model_forward(model, input.data(), input.size(), out.data(), out.size()), "forward");
    float mn = INFINITY, mx = -INFINITY;
    double sum = 0.0;
    for (float v : out) { mn = std::min(mn, v); mx = std::max(mx, v); sum += v; }
    std::vector<double> samples((size_t)a.runs);
    check(ppocr_model_benchmark(model, input.data(), input.size(), (size_t)a.warmup, (size_t)a.runs, samples.data()), "benchmark");
    double avg = 0.0;
    for (double s : samples) avg += s;
    avg /= samples.size();
    std::vector<double> sorted = samples;
    std::sort(sorted.begin(), sorted.end());

    std::printf("backend: b200\n");
    std::printf("kind: %s\n", a.kind.c_str());
    std::printf("model: %s\n", a.model.c_str());
    std::printf("input_shape: [%zu, %zu, %zu, %zu]\n", shape[0], shape[1], shape[2], shape[3]);
    std::printf("output_shape: [");
    for (size_t i = 0; i < rank; ++i) std::printf("%s%zu", i ? ", " : "", out_shape[i]);
    std::printf("]\n");
    std::printf("output_min: %.9e\noutput_max: %.9e\noutput_sum: %.9e\n", mn, mx, sum);
    std::printf("warmup: %ld\nruns: %ld\n", a.warmup, a.runs);
    std::printf("average_ms: %.3f\np50_ms: %.3f\np90_ms: %.3f\np95_ms: %.3f\n", avg, percentile(sorted, 0.5),
                percentile(sorted, 0.9), percentile(sorted, 0.95));
    std::printf("throughput: %.2f\n", 1000.0 / avg);
    std::printf("batch: %ld\n%s: %.2f\n", a.batch, det ? "images_per_s" : "crops_per_s", 1000.0 * a.batch / avg);

    if (!a.reference.empty()) {
        // report_reference (benchmark.rs:229-285)
        std::vector<float> ref = read_f32(a.reference, out.size());
        float maxd = 0.f;
        double tot = 0.0;
        for (size_t i = 0; i < out.size(); ++i) {
            const float d = std::fabs(out[i] - ref[i]);
            maxd = std::max(maxd, d);
            tot += d;
        }
        std::printf("reference_max_abs: %.9e\nreference_mean_abs: %.9e\n", maxd, tot / out.size());
        if (det) {
            size_t mism = 0;
            for (size_t i = 0; i < out.size(); ++i) mism += (out[i] >= 0.5f) != (ref[i] >= 0.5f);
            std::printf("reference_threshold_0.5_mismatches: %zu\n", mism);
        } else {
            const size_t classes = out_shape[rank - 1];
            size_t mism = 0;
            for (size_t r = 0; r < out.size() / classes; ++r)
                mism += argmax(&out[r * classes], classes) != argmax(&ref[r * classes], classes);
            std::printf("reference_argmax_mismatches: %zu\n", mism);
        }
    }
    if (!a.dump.empty()) {
        std::ofstream f(a.dump, std::ios::binary);
        f.write(reinterpret_cast<const char*>(out.data()), out.size() * 4);
        std::printf("dump: %s\n", a.dump.c_str());
    }
    ppocr_model_destroy(model);
    ppocr_gpu_destroy(gpu);
    return 0;
}
