// ppocr-gpu-bench: the reference's benchmark CLI contract
// (ppocr-rs src/bin/ppocr-gpu-bench.rs:45-88, src/bin/benchmark.rs:13-320)
// over the C ABI.  Same flags, deterministic input, F32 reference / dump files
// and report keys; adds --batch, --precision, --no-graph, --gpus (the same
// benchmark on N devices at once, one host thread and model per device) and
// --seed-weights (a seeded random-init checkpoint instead of --model).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <thread>
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
    long height = -1, width = -1, warmup = 5, runs = 30, batch = 1, gpus = 1;
    long long seed = -1;
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
        else if (k == "--gpus") a.gpus = std::stol(val());
        else if (k == "--seed-weights") a.seed = std::stoll(val());
        else if (k == "-h" || k == "--help") {
            std::printf("usage: ppocr-gpu-bench --kind det|rec --model FILE [--model-size tiny|small|medium] [--height H] "
                        "[--width W] [--input F32] [--reference F32] [--dump F32] [--warmup 5] [--runs 30] [--batch 1] "
                        "[--precision fp32|bf16|fp32tc] [--no-graph] [--gpus N] [--seed-weights SEED]\n");
            std::exit(0);
        } else die("unknown argument " + k);
    }
    if (a.kind != "det" && a.kind != "rec") die("--kind must be det or rec");
    if (a.seed >= 0 && !a.model.empty()) die("--model and --seed-weights are mutually exclusive");
    if (a.model.empty() && a.seed < 0)
        die("the pinned model store is not part of this build; pass --model FILE or --seed-weights SEED");
    if (a.runs <= 0) die("--runs must be positive");
    if (a.gpus <= 0) die("--gpus must be positive");
    if (a.batch <= 0) die("--batch must be positive");
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

    if (a.seed >= 0) {
        // A seeded checkpoint in the reference layout, written next to the
        // system's temporary files.
        const char* tmp = std::getenv("TMPDIR");
        a.model = std::string(tmp && *tmp ? tmp : "/tmp") + "/ppocr-seeded-" + a.kind + "-" + a.model_size + "-" +
                  std::to_string(a.seed) + ".safetensors";
        check(ppocr_write_seeded_weights(a.model.c_str(), det ? 0 : 1, size, (uint64_t)a.seed), "write seeded weights");
    }
    int devices = 0;
    check(ppocr_gpu_count(&devices), "count GPUs");
    if (a.gpus > devices) die("--gpus " + std::to_string(a.gpus) + " exceeds the " + std::to_string(devices) + " visible devices");

    // One worker per device: its own handle, model, output and samples.
    struct Worker {
        ppocr_gpu* gpu = nullptr;
        ppocr_model* model = nullptr;
        std::vector<float> out;
        std::vector<double> samples;
        size_t out_shape[4] = {0, 0, 0, 0}, rank = 0;
        int status = PPOCR_OK;
        std::string error;
    };
    std::vector<Worker> workers((size_t)a.gpus);
    auto run = [&](int dev) {
        Worker& wk = workers[(size_t)dev];
        auto ok = [&](int st, const char* what) {
            if (st != PPOCR_OK && wk.status == PPOCR_OK) {
                wk.status = st;
                wk.error = std::string(what) + ": " + ppocr_last_error();
            }
            return st == PPOCR_OK;
        };
        if (!ok(ppocr_gpu_create(dev, &wk.gpu), "create GPU")) return;
        ppocr_load_options o;
        ppocr_load_options_default(&o);
        o.precision = a.precision == "bf16" ? PPOCR_PRECISION_BF16 : a.precision == "fp32tc" ? PPOCR_PRECISION_FP32_TC : PPOCR_PRECISION_FP32;
        o.use_graph = a.graph ? 1 : 0;
        if (!ok(det ? ppocr_detector_load_ex(wk.gpu, a.model.c_str(), size, shape, &o, &wk.model)
                    : ppocr_recognizer_load_ex(wk.gpu, a.model.c_str(), size, shape, &o, nullptr, &wk.model),
                det ? "load detector" : "load recognizer"))
            return;
        size_t elements = 0;
        if (!ok(ppocr_model_output_shape(wk.model, wk.out_shape, &wk.rank, &elements), "output shape")) return;
        wk.out.resize(elements);
        if (!ok(ppocr_model_forward(wk.model, input.data(), input.size(), wk.out.data(), wk.out.size()), "forward")) return;
        wk.samples.resize((size_t)a.runs);
        ok(ppocr_model_benchmark(wk.model, input.data(), input.size(), (size_t)a.warmup, (size_t)a.runs, wk.samples.data()),
           "benchmark");
    };
    if (a.gpus == 1) {
        run(0);
    } else {
        std::vector<std::thread> threads;
        for (int d = 0; d < (int)a.gpus; ++d) threads.emplace_back(run, d);
        for (auto& t : threads) t.join();
    }
    for (size_t d = 0; d < workers.size(); ++d)
        if (workers[d].status != PPOCR_OK) die("GPU " + std::to_string(d) + ": " + workers[d].error);
    const Worker& w0 = workers[0];
    const std::vector<float>& out = w0.out;
    const size_t* out_shape = w0.out_shape;
    const size_t rank = w0.rank;
    float mn = INFINITY, mx = -INFINITY;
    double sum = 0.0;
    for (float v : out) { mn = std::min(mn, v); mx = std::max(mx, v); sum += v; }
    const std::vector<double>& samples = w0.samples;
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
    if (a.gpus > 1) {
        // Every device ran the same batch concurrently (weak scaling): the
        // aggregate is the sum of the per-device rates.
        double agg = 0.0;
        std::printf("gpus: %ld\n", a.gpus);
        for (size_t d = 0; d < workers.size(); ++d) {
            double m = 0.0;
            for (double s : workers[d].samples) m += s;
            m /= workers[d].samples.size();
            std::printf("gpu%zu_average_ms: %.3f\n", d, m);
            agg += 1000.0 * a.batch / m;
        }
        std::printf("aggregate_%s: %.2f\n", det ? "images_per_s" : "crops_per_s", agg);
    }
    if (a.seed >= 0) std::printf("seed_weights: %lld\n", a.seed);

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
    for (auto& wk : workers) {
        ppocr_model_destroy(wk.model);
        ppocr_gpu_destroy(wk.gpu);
    }
    return 0;
}
