// extern "C" boundary: the ppocr_rs::gpu API (src/gpu/mod.rs) as a C ABI.
//
// One ppocr_gpu per device owns a non-blocking stream and the activation
// arena shared by every model loaded on it (grown to the largest plan, as
// ppocr-rs's shared workspace is, src/gpu/runtime.rs:1718-1730).  A model
// owns its packed weights (shareable between recognizers of one file), its
// plan and, when enabled, the CUDA graph of its forward, re-captured when the
// arena moves.  Every wait is bounded: a stuck stream surfaces as Error::Gpu.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.hpp"
#include "handles.hpp"
#include "models.hpp"
#include "ppocr_b200.h"
#include "safetensors.hpp"

using namespace ppocr;

namespace ppocr {
std::string& last_error() {
    thread_local std::string message;
    return message;
}

void wait_stream(cudaStream_t s, int timeout_ms, ppocr_gpu* owner) {
    if (timeout_ms <= 0) timeout_ms = 60000;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    int spins = 0;
    while (true) {
        cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return;
        if (e != cudaErrorNotReady) cuda_check(e, "device execution");
        if (std::chrono::steady_clock::now() > deadline) {
            // Work still queued on the device may write the caller's buffers
            // later: the handle refuses every further call.
            if (owner) owner->poisoned = true;
            fail(PPOCR_ERR_GPU, "device did not finish within the wait limit");
        }
        if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}
}  // namespace ppocr

namespace {

// Per-model device flags, reset before and read back after every forward:
// [0] non-finite input, [1] non-finite output, [2] the code of a tensor-core
// pipeline wait that ran out (0: none), [3] unused.
constexpr size_t kFlags = 4;

// Process-wide pool of pinned host flag sets (kFlags ints): a model load takes one set
// instead of pinning a fresh page (cudaMallocHost costs milliseconds), and the
// pool outlives every device handle.
class PinnedFlags {
public:
    static int* acquire() {
        std::lock_guard<std::mutex> lock(mu());
        auto& f = free_list();
        if (f.empty()) {
            constexpr size_t kSets = 1024;
            int* slab = nullptr;
            cuda_check(cudaHostAlloc(reinterpret_cast<void**>(&slab), kSets * kFlags * sizeof(int), cudaHostAllocPortable),
                       "allocate host flags");
            for (size_t i = 0; i < kSets; ++i) f.push_back(slab + kFlags * i);
        }
        int* p = f.back();
        f.pop_back();
        return p;
    }
    static void release(int* p) {
        if (!p) return;
        std::lock_guard<std::mutex> lock(mu());
        free_list().push_back(p);
    }

private:
    // Never destroyed: models may be released by finalizers after static
    // destruction has begun at process exit.
    static std::mutex& mu() {
        static std::mutex* m = new std::mutex;
        return *m;
    }
    static std::vector<int*>& free_list() {
        static std::vector<int*>* f = new std::vector<int*>;
        return *f;
    }
};

struct DeviceWeights {
    void* ptr = nullptr;
    size_t bytes = 0;
    std::vector<uint8_t> host;   // kept for sharing checks
    ~DeviceWeights() {
        if (ptr) cudaFree(ptr);
    }
};
}  // namespace

// Staging buffers, copy streams and events of ppocr_model_forward_pipelined:
// two slots, so chunk s + 1 uploads while chunk s computes and chunk s - 1
// downloads.
struct ForwardPipe {
    cudaStream_t h2d = nullptr, d2h = nullptr;
    void* in_stage[2] = {nullptr, nullptr};
    void* out_stage[2] = {nullptr, nullptr};
    cudaEvent_t arrived[2] = {}, consumed[2] = {}, computed[2] = {}, downloaded[2] = {};
    ~ForwardPipe() {
        if (h2d) cudaStreamSynchronize(h2d);
        if (d2h) cudaStreamSynchronize(d2h);
        for (int i = 0; i < 2; ++i) {
            if (in_stage[i]) cudaFree(in_stage[i]);
            if (out_stage[i]) cudaFree(out_stage[i]);
            for (cudaEvent_t e : {arrived[i], consumed[i], computed[i], downloaded[i]})
                if (e) cudaEventDestroy(e);
        }
        if (h2d) cudaStreamDestroy(h2d);
        if (d2h) cudaStreamDestroy(d2h);
    }
};

struct ppocr_model {
    ppocr_gpu* gpu = nullptr;
    std::unique_ptr<ForwardPipe> pipe;
    BuiltModel m;
    std::shared_ptr<DeviceWeights> weights;
    ppocr_load_options opts{};
    cudaGraphExec_t exec = nullptr;
    uint64_t exec_gen = 0;
    float exec_threshold = 0.f;
    bool warmed = false;
    int* dflags = nullptr;   // device flags (kFlags ints, see above)
    int* hflags = nullptr;   // pinned host copy
    int* dcounters = nullptr;   // the plan's fused-SE arrival counters (zero between launches)

    ~ppocr_model() {
        if (exec) cudaGraphExecDestroy(exec);
        if (dflags) cudaFree(dflags);
        if (dcounters) cudaFree(dcounters);
        PinnedFlags::release(hflags);
    }

    Ctx ctx() const {
        Ctx c;
        c.arena = static_cast<char*>(gpu->arena);
        c.weights = static_cast<const char*>(weights->ptr);
        c.tensors = &m.plan.tensors;
        c.side = gpu->side;
        c.fork = gpu->fork;
        c.join = gpu->join;
        c.err = dflags + 2;
        c.counters = dcounters;
        return c;
    }
    void* tensor(int tid) const { return tid < 0 ? nullptr : static_cast<char*>(gpu->arena) + m.plan.tensors[tid].offset; }

    // Enqueue one forward over the arena input slot.
    void run(cudaStream_t s) {
        gpu->ensure_arena(m.plan.arena_bytes);
        if (!warmed || !opts.use_graph) {
            m.plan.run(ctx(), s);
            warmed = true;
            return;
        }
        if (!exec || exec_gen != gpu->arena_gen || exec_threshold != *m.mask_threshold) {
            if (exec) { cudaGraphExecDestroy(exec); exec = nullptr; }
            cudaStream_t cap;
            cuda_check(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking), "create capture stream");
            cudaGraph_t g = nullptr;
            cudaError_t e = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
            if (e == cudaSuccess) {
                try {
                    m.plan.run(ctx(), cap);
                } catch (...) {
                    cudaStreamEndCapture(cap, &g);
                    if (g) cudaGraphDestroy(g);
                    cudaStreamDestroy(cap);
                    throw;
                }
                e = cudaStreamEndCapture(cap, &g);
            }
            cudaStreamDestroy(cap);
            cuda_check(e, "capture forward graph");
            e = cudaGraphInstantiate(&exec, g, 0);
            cudaGraphDestroy(g);
            cuda_check(e, "instantiate forward graph");
            exec_gen = gpu->arena_gen;
            exec_threshold = *m.mask_threshold;
        }
        cuda_check(cudaGraphLaunch(exec, s), "launch forward graph");
    }

    int output_tid() const { return m.kind == Kind::Detector ? m.prob : m.probs; }
    size_t input_elements() const { return (size_t)m.n * 3 * m.h * m.w; }
};

namespace {

// Raises the reference's error for the flags read back after a forward:
// InvalidInput for a non-finite input (src/gpu/runtime.rs:1979-1983),
// Error::Gpu for a non-finite output (2217-2219) or a tensor-core pipeline
// wait that ran out (the forward's results are then incomplete).
void raise_flags(const ppocr_model* model) {
    if (model->hflags[2])
        fail(PPOCR_ERR_GPU, "GPU error: a tensor-core pipeline wait ran out (code " + std::to_string(model->hflags[2]) +
                                "); the forward's results are incomplete");
    if (model->hflags[0]) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: model input contains non-finite values");
    if (model->hflags[1]) fail(PPOCR_ERR_GPU, "GPU error: model output contains non-finite values");
}

void upload_and_run(ppocr_model* model, const float* input, size_t len) {
    if (!input) fail(PPOCR_ERR_INVALID_INPUT, "input pointer is null");
    if (len != model->input_elements()) {
        fail(PPOCR_ERR_INVALID_INPUT, "input has " + std::to_string(len) + " values; expected " +
                                          std::to_string(model->input_elements()));
    }
    ppocr_gpu* g = model->gpu;
    g->ensure_arena(model->m.plan.arena_bytes);
    cuda_check(cudaMemsetAsync(model->dflags, 0, kFlags * sizeof(int), g->stream), "reset flags");
    cuda_check(cudaMemcpyAsync(model->tensor(model->m.input), input, len * 4, cudaMemcpyHostToDevice, g->stream), "upload input");
    // Non-finite inputs are an InvalidInput (src/gpu/runtime.rs:1979-1983); the scan runs on the device.
    cuda_check(launch_check_finite(static_cast<const float*>(model->tensor(model->m.input)), len, model->dflags, g->stream),
               "check input");
    model->run(g->stream);
}

// Enqueues the output scan and the flag readback, waits, and raises the
// reference's errors: InvalidInput for a non-finite input, Error::Gpu for a
// non-finite output (src/gpu/runtime.rs:2217-2219).
// Reads the device flags after a forward; `checked_tid` (if any) is checked
// for non-finite values first, as `rows` rows of `cols` floats at stride `ld`.
void finish(ppocr_model* model, int checked_tid, size_t rows, size_t cols, size_t ld) {
    cudaStream_t s = model->gpu->stream;
    if (checked_tid >= 0)
        cuda_check(launch_check_finite_rows(static_cast<const float*>(model->tensor(checked_tid)), rows, cols, ld,
                                            model->dflags + 1, s),
                   "check output");
    cuda_check(cudaMemcpyAsync(model->hflags, model->dflags, kFlags * sizeof(int), cudaMemcpyDeviceToHost, s), "read flags");
    wait_stream(s, 0, model->gpu);
    raise_flags(model);
}

void finish(ppocr_model* model, int checked_tid, size_t checked_count) { finish(model, checked_tid, 1, checked_count, checked_count); }

}  // namespace

PreprocessParams ppocr::make_preprocess(const ppocr_image* image, const float corners[8], size_t content_width, size_t out_h,
                                        size_t out_w, bool detector) {
    PreprocessParams p;
    p.rgb = image->rgb;
    p.src_w = (int)image->width;
    p.src_h = (int)image->height;
    std::memcpy(p.corners, corners, sizeof(p.corners));
    p.out_w = (int)out_w;
    p.out_h = (int)out_h;
    p.content_w = (int)content_width;
    // Normalization::new (src/preprocess/kernels.rs:9-18): scale = 1/(255 std), bias = -mean/std, BGR order
    const float det_mean[3] = {0.485f, 0.456f, 0.406f}, det_std[3] = {0.229f, 0.224f, 0.225f};
    for (int c = 0; c < 3; ++c) {
        const float mean = detector ? det_mean[c] : 0.5f, sd = detector ? det_std[c] : 0.5f;
        p.scale[c] = 1.0f / (255.0f * sd);
        p.bias[c] = -mean / sd;
    }
    return p;
}

namespace {

void download(ppocr_model* model, int tid, void* dst, size_t bytes) {
    cuda_check(cudaMemcpyAsync(dst, model->tensor(tid), bytes, cudaMemcpyDeviceToHost, model->gpu->stream), "read output");
}

ppocr_model* load_model(ppocr_gpu* gpu, const char* path, int size, const size_t shape[4], const ppocr_load_options* options,
                        const ppocr_model* shared, bool detector) {
    if (!gpu) fail(PPOCR_ERR_INVALID_INPUT, "gpu handle is null");
    if (!path) fail(PPOCR_ERR_INVALID_INPUT, "model path is null");
    if (!shape) fail(PPOCR_ERR_INVALID_INPUT, "input shape is null");
    ppocr_load_options o;
    if (options) o = *options;
    else ppocr_load_options_default(&o);
    if (o.precision != PPOCR_PRECISION_FP32 && o.precision != PPOCR_PRECISION_BF16 && o.precision != PPOCR_PRECISION_FP32_TC)
        fail(PPOCR_ERR_INVALID_INPUT, "unknown precision");
    const DType dt = o.precision == PPOCR_PRECISION_BF16 ? DT_BF16 : DT_F32;
    SafeTensors st = SafeTensors::load(path);
    std::unique_ptr<ppocr_model> model(new ppocr_model());
    model->gpu = gpu;
    model->opts = o;
    // FP32 runs on the CUDA cores (exact FP32 FMA); BF16 and FP32_TC use tcgen05 unless simt_only.
    const int tc_mode = o.simt_only ? TC_NONE : o.precision == PPOCR_PRECISION_FP32_TC ? TC_ALL : TC_GEMMS;
    model->m = detector ? build_detector(st, size, shape, dt, tc_mode) : build_recognizer(st, size, shape, dt, tc_mode);
    std::lock_guard<std::mutex> lock(gpu->mu);
    gpu->bind();
    const std::vector<uint8_t>& blob = model->m.blob.bytes();
    if (shared && shared->weights && shared->weights->host == blob) {
        model->weights = shared->weights;
    } else {
        auto w = std::make_shared<DeviceWeights>();
        w->bytes = blob.size();
        cuda_check(cudaMalloc(&w->ptr, std::max<size_t>(w->bytes, 256)), "allocate weights");
        // Ordered on the model's (non-blocking) stream and completed before
        // returning: a plain cudaMemcpy from pageable memory may return before
        // its DMA lands, and the stream would not wait for it.
        cuda_check(cudaMemcpyAsync(w->ptr, blob.data(), w->bytes, cudaMemcpyHostToDevice, gpu->stream), "upload weights");
        cuda_check(cudaStreamSynchronize(gpu->stream), "upload weights");
        w->host = blob;
        model->weights = w;
    }
    // The packed host copy is no longer needed (the device weights hold one
    // host copy for sharing checks): an engine caching hundreds of recognizer
    // shapes would otherwise keep one per shape.
    model->m.blob = WeightBlob();
    if (o.keep_tensors) {
        // Diagnostics: no two tensors share memory, so every op's output
        // survives the forward for ppocr_model_read_tensor.
        for (auto& t : model->m.plan.tensors) t.pinned = true;
        model->m.plan.finalize();
    }
    gpu->ensure_arena(model->m.plan.arena_bytes);
    cuda_check(cudaMalloc(&model->dflags, kFlags * sizeof(int)), "allocate flags");
    if (model->m.counter_slots > 0) {
        cuda_check(cudaMalloc(&model->dcounters, (size_t)model->m.counter_slots * sizeof(int)), "allocate counters");
        cuda_check(cudaMemsetAsync(model->dcounters, 0, (size_t)model->m.counter_slots * sizeof(int), gpu->stream), "clear counters");
        cuda_check(cudaStreamSynchronize(gpu->stream), "clear counters");
    }
    model->hflags = PinnedFlags::acquire();
    gpu_retain(gpu);
    return model.release();
}

}  // namespace

void ppocr::gpu_retain(ppocr_gpu* gpu) { gpu->refs.fetch_add(1); }

void ppocr::gpu_release(ppocr_gpu* gpu) {
    if (gpu->refs.fetch_sub(1) != 1) return;
    cudaSetDevice(gpu->device);
    if (gpu->stream) cudaStreamSynchronize(gpu->stream);
    if (gpu->arena) cudaFree(gpu->arena);
    if (gpu->side) cudaStreamSynchronize(gpu->side);
    if (gpu->stream) cudaStreamDestroy(gpu->stream);
    if (gpu->side) cudaStreamDestroy(gpu->side);
    if (gpu->fork) cudaEventDestroy(gpu->fork);
    if (gpu->join) cudaEventDestroy(gpu->join);
    delete gpu;
}

extern "C" {

void ppocr_load_options_default(ppocr_load_options* options) {
    if (!options) return;
    std::memset(options, 0, sizeof(*options));
    options->precision = PPOCR_PRECISION_FP32;
    options->use_graph = 1;
}

const char* ppocr_last_error(void) { return last_error().c_str(); }

int ppocr_gpu_count(int* count) {
    return guard([&] {
        if (!count) fail(PPOCR_ERR_INVALID_INPUT, "count pointer is null");
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
            cudaGetLastError();
            n = 0;
        } else {
            cuda_check(e, "cudaGetDeviceCount");
        }
        *count = n;
    });
}

int ppocr_gpu_create(int device, ppocr_gpu** out) {
    return guard([&] {
        if (!out) fail(PPOCR_ERR_INVALID_INPUT, "output pointer is null");
        *out = nullptr;
        int n = 0;
        cudaError_t e = cudaGetDeviceCount(&n);
        if (e != cudaSuccess || n == 0) {
            cudaGetLastError();
            fail(PPOCR_ERR_GPU, "request CUDA device: no CUDA device is available");
        }
        if (device < 0 || device >= n) fail(PPOCR_ERR_GPU, "request CUDA device " + std::to_string(device) + ": out of range");
        std::unique_ptr<ppocr_gpu> g(new ppocr_gpu());
        g->device = device;
        g->bind();
        cudaDeviceProp prop;
        cuda_check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        if (prop.major < 10) fail(PPOCR_ERR_GPU, std::string("device ") + prop.name + " is not sm_100 class; this build targets sm_100a");
        g->name = prop.name;
        cuda_check(cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking), "create stream");
        cuda_check(cudaStreamCreateWithFlags(&g->side, cudaStreamNonBlocking), "create side stream");
        cuda_check(cudaEventCreateWithFlags(&g->fork, cudaEventDisableTiming), "create fork event");
        cuda_check(cudaEventCreateWithFlags(&g->join, cudaEventDisableTiming), "create join event");
        *out = g.release();
    });
}

void ppocr_gpu_destroy(ppocr_gpu* gpu) {
    if (gpu) gpu_release(gpu);
}

int ppocr_gpu_info(const ppocr_gpu* gpu, char* name, size_t capacity) {
    return guard([&] {
        if (!gpu || !name || capacity == 0) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        std::strncpy(name, gpu->name.c_str(), capacity - 1);
        name[capacity - 1] = 0;
    });
}

int ppocr_upload_rgb(ppocr_gpu* gpu, uint32_t width, uint32_t height, const uint8_t* pixels, size_t len, ppocr_image** out) {
    return guard([&] {
        if (!gpu || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        *out = nullptr;
        // Gpu::upload_rgb checks (src/gpu/runtime.rs:175-197)
        if (width == 0 || height == 0) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: source image dimensions must be non-zero");
        const size_t expected = (size_t)width * height * 3;
        if (len != expected || !pixels)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: source image has " + std::to_string(len) + " RGB bytes; expected " +
                                              std::to_string(expected) + " for " + std::to_string(width) + "x" + std::to_string(height));
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        std::unique_ptr<ppocr_image> img(new ppocr_image());
        img->gpu = gpu;
        img->width = width;
        img->height = height;
        img->capacity = expected;
        cuda_check(cudaMalloc(&img->rgb, expected), "allocate source image");
        cuda_check(cudaMemcpyAsync(img->rgb, pixels, expected, cudaMemcpyHostToDevice, gpu->stream), "upload source image");
        cuda_check(cudaStreamSynchronize(gpu->stream), "upload source image");
        gpu_retain(gpu);
        *out = img.release();
    });
}

void ppocr_image_destroy(ppocr_image* image) {
    if (!image) return;
    ppocr_gpu* gpu = image->gpu;
    if (image->rgb) {
        cudaSetDevice(gpu->device);
        cudaFree(image->rgb);
    }
    delete image;
    gpu_release(gpu);
}

int ppocr_detector_load(ppocr_gpu* gpu, const char* path, int size, const size_t input_shape[4], ppocr_model** out) {
    return ppocr_detector_load_ex(gpu, path, size, input_shape, nullptr, out);
}

int ppocr_detector_load_ex(ppocr_gpu* gpu, const char* path, int size, const size_t input_shape[4],
                           const ppocr_load_options* options, ppocr_model** out) {
    return guard([&] {
        if (!out) fail(PPOCR_ERR_INVALID_INPUT, "output pointer is null");
        *out = nullptr;
        *out = load_model(gpu, path, size, input_shape, options, nullptr, true);
    });
}

int ppocr_recognizer_load(ppocr_gpu* gpu, const char* path, int size, const size_t input_shape[4], ppocr_model** out) {
    return ppocr_recognizer_load_ex(gpu, path, size, input_shape, nullptr, nullptr, out);
}

int ppocr_recognizer_load_ex(ppocr_gpu* gpu, const char* path, int size, const size_t input_shape[4],
                             const ppocr_load_options* options, const ppocr_model* shared_weights_from, ppocr_model** out) {
    return guard([&] {
        if (!out) fail(PPOCR_ERR_INVALID_INPUT, "output pointer is null");
        *out = nullptr;
        if (shared_weights_from && shared_weights_from->m.kind != Kind::Recognizer)
            fail(PPOCR_ERR_INVALID_INPUT, "shared weights must come from a recognizer");
        *out = load_model(gpu, path, size, input_shape, options, shared_weights_from, false);
    });
}

void ppocr_model_destroy(ppocr_model* model) {
    if (!model) return;
    {
        // Never throws: this also runs from finalizers at process exit, when
        // the CUDA runtime may already be shutting down.
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        if (cudaSetDevice(model->gpu->device) == cudaSuccess) cudaStreamSynchronize(model->gpu->stream);
    }
    ppocr_gpu* gpu = model->gpu;
    delete model;
    gpu_release(gpu);
}

int ppocr_write_seeded_weights(const char* path, int kind, int size, uint64_t seed) {
    return guard([&] {
        if (!path) fail(PPOCR_ERR_INVALID_INPUT, "path is null");
        if (kind != 0 && kind != 1) fail(PPOCR_ERR_INVALID_INPUT, "kind must be 0 (detector) or 1 (recognizer)");
        if (size != PPOCR_MEDIUM && size != PPOCR_SMALL && size != PPOCR_TINY) fail(PPOCR_ERR_INVALID_INPUT, "unknown model size");
        write_seeded_weights(path, kind == 0, size, seed);
    });
}

int ppocr_inspect_model(const char* path, int kind, int size, const size_t input_shape[4], int precision, size_t* ops,
                        size_t* arena_bytes, size_t* weight_bytes, size_t output_shape[4]) {
    return guard([&] {
        if (!path || !input_shape) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (kind != 0 && kind != 1) fail(PPOCR_ERR_INVALID_INPUT, "kind must be 0 (detector) or 1 (recognizer)");
        if (precision != PPOCR_PRECISION_FP32 && precision != PPOCR_PRECISION_BF16 && precision != PPOCR_PRECISION_FP32_TC)
            fail(PPOCR_ERR_INVALID_INPUT, "unknown precision");
        const DType dt = precision == PPOCR_PRECISION_BF16 ? DT_BF16 : DT_F32;
        const int tc = precision == PPOCR_PRECISION_FP32_TC ? TC_ALL : TC_GEMMS;
        SafeTensors st = SafeTensors::load(path);
        BuiltModel m = kind == 0 ? build_detector(st, size, input_shape, dt, tc) : build_recognizer(st, size, input_shape, dt, tc);
        if (ops) *ops = m.plan.ops.size();
        if (arena_bytes) *arena_bytes = m.plan.arena_bytes;
        if (weight_bytes) *weight_bytes = m.blob.bytes().size();
        if (output_shape)
            for (size_t i = 0; i < 4; ++i) output_shape[i] = i < m.output_shape.size() ? m.output_shape[i] : 0;
    });
}

int ppocr_model_output_shape(const ppocr_model* model, size_t shape[4], size_t* rank, size_t* elements) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        const auto& s = model->m.output_shape;
        if (shape)
            for (size_t i = 0; i < 4; ++i) shape[i] = i < s.size() ? s[i] : 0;
        if (rank) *rank = s.size();
        if (elements) *elements = model->m.output_elements;
    });
}

int ppocr_model_input_shape(const ppocr_model* model, size_t shape[4]) {
    return guard([&] {
        if (!model || !shape) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        shape[0] = model->m.n; shape[1] = 3; shape[2] = model->m.h; shape[3] = model->m.w;
    });
}

int ppocr_model_forward(ppocr_model* model, const float* input, size_t input_len, float* output, size_t output_capacity) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (!output || output_capacity < model->m.output_elements)
            fail(PPOCR_ERR_INVALID_INPUT, "output buffer holds " + std::to_string(output_capacity) + " values; " +
                                              std::to_string(model->m.output_elements) + " required");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        upload_and_run(model, input, input_len);
        download(model, model->output_tid(), output, model->m.output_elements * 4);
        finish(model, model->output_tid(), model->m.output_elements);
    });
}

namespace {

// What a pipelined forward hands back per chunk: `stage` enqueues, on the
// compute stream, the copy of the chunk's results into a download slot
// (stage_bytes bytes); `download` enqueues that slot's copy to the host on the
// download stream.
struct PipeOutput {
    size_t stage_bytes = 0;
    std::function<void(cudaStream_t, void* slot)> stage;
    std::function<void(size_t chunk, const void* slot, cudaStream_t)> download;
};

// images / batch chunks: each chunk's upload, forward and download run on
// their own streams through two slots, so chunk c + 1 uploads while chunk c
// computes and chunk c - 1 downloads.
void forward_pipelined(ppocr_model* model, const float* input, size_t images, const PipeOutput& out) {
    if (!input) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
    const size_t batch = (size_t)model->m.n;
    if (images == 0 || images % batch)
        fail(PPOCR_ERR_INVALID_INPUT, "invalid input: image count " + std::to_string(images) + " is not a multiple of the model batch " +
                                          std::to_string(batch));
    const size_t chunks = images / batch;
    const size_t in_elems = model->input_elements(), out_elems = model->m.output_elements;
    if (out.stage_bytes > out_elems * 4) fail(PPOCR_ERR_INVALID_INPUT, "pipelined output larger than the model output");
    std::lock_guard<std::mutex> lock(model->gpu->mu);
    model->gpu->bind();
    model->gpu->ensure_arena(model->m.plan.arena_bytes);
    if (!model->pipe) {
        std::unique_ptr<ForwardPipe> p(new ForwardPipe());
        cuda_check(cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking), "create upload stream");
        cuda_check(cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking), "create download stream");
        for (int i = 0; i < 2; ++i) {
            cuda_check(cudaMalloc(&p->in_stage[i], in_elems * 4), "allocate input staging");
            cuda_check(cudaMalloc(&p->out_stage[i], out_elems * 4), "allocate output staging");
            for (cudaEvent_t* e : {&p->arrived[i], &p->consumed[i], &p->computed[i], &p->downloaded[i]})
                cuda_check(cudaEventCreateWithFlags(e, cudaEventDisableTiming), "create pipeline event");
        }
        model->pipe = std::move(p);
    }
    ForwardPipe& pp = *model->pipe;
    cudaStream_t cs = model->gpu->stream;
    float* dinput = static_cast<float*>(model->tensor(model->m.input));
    try {
        cuda_check(cudaMemsetAsync(model->dflags, 0, kFlags * sizeof(int), cs), "reset flags");
        for (size_t c = 0; c < chunks; ++c) {
            const int slot = (int)(c & 1);
            // Upload chunk c once the forward of chunk c - 2 has taken its copy of the slot.
            cuda_check(cudaStreamWaitEvent(pp.h2d, pp.consumed[slot], 0), "order upload");
            cuda_check(cudaMemcpyAsync(pp.in_stage[slot], input + c * in_elems, in_elems * 4, cudaMemcpyHostToDevice, pp.h2d),
                       "upload input");
            cuda_check(cudaEventRecord(pp.arrived[slot], pp.h2d), "record upload");
            // Forward chunk c on the model stream.
            cuda_check(cudaStreamWaitEvent(cs, pp.arrived[slot], 0), "order forward");
            // Staging copies run as kernels (with the finiteness checks folded
            // in): a copy-engine copy here would queue behind the next chunk's upload.
            cuda_check(launch_copy_check(static_cast<const float*>(pp.in_stage[slot]), dinput, in_elems, model->dflags, cs),
                       "stage input");
            cuda_check(cudaEventRecord(pp.consumed[slot], cs), "record staging");
            model->run(cs);
            // Hand the results to the download slot once chunk c - 2 has left it.
            cuda_check(cudaStreamWaitEvent(cs, pp.downloaded[slot], 0), "order output staging");
            out.stage(cs, pp.out_stage[slot]);
            cuda_check(cudaEventRecord(pp.computed[slot], cs), "record forward");
            cuda_check(cudaStreamWaitEvent(pp.d2h, pp.computed[slot], 0), "order download");
            out.download(c, pp.out_stage[slot], pp.d2h);
            cuda_check(cudaEventRecord(pp.downloaded[slot], pp.d2h), "record download");
        }
        cuda_check(cudaStreamWaitEvent(cs, pp.downloaded[(chunks - 1) & 1], 0), "join download");
        cuda_check(cudaMemcpyAsync(model->hflags, model->dflags, kFlags * sizeof(int), cudaMemcpyDeviceToHost, cs), "read flags");
        wait_stream(cs, 0, model->gpu);
    } catch (...) {
        // The caller's buffers must not be touched after return.
        cudaStreamSynchronize(pp.h2d);
        cudaStreamSynchronize(cs);
        cudaStreamSynchronize(pp.d2h);
        throw;
    }
    raise_flags(model);
}

}  // namespace

int ppocr_model_forward_pipelined(ppocr_model* model, const float* input, size_t images, float* output,
                                  size_t output_capacity) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (!input || !output) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        const size_t batch = (size_t)model->m.n, out_elems = model->m.output_elements;
        const size_t chunks = images / batch;
        if (images % batch == 0 && output_capacity < chunks * out_elems)
            fail(PPOCR_ERR_INVALID_INPUT, "output buffer holds " + std::to_string(output_capacity) + " values; " +
                                              std::to_string(chunks * out_elems) + " required");
        const int otid = model->output_tid();
        PipeOutput po;
        po.stage_bytes = out_elems * 4;
        po.stage = [&](cudaStream_t cs, void* slot) {
            cuda_check(launch_copy_check(static_cast<const float*>(model->tensor(otid)), static_cast<float*>(slot), out_elems,
                                         model->dflags + 1, cs),
                       "stage output");
        };
        po.download = [&](size_t c, const void* slot, cudaStream_t d2h) {
            cuda_check(cudaMemcpyAsync(output + c * out_elems, slot, out_elems * 4, cudaMemcpyDeviceToHost, d2h), "read output");
        };
        forward_pipelined(model, input, images, po);
    });
}

int ppocr_recognizer_forward_pipelined_ctc(ppocr_model* model, const float* input, size_t images, int32_t* indices,
                                           float* probabilities, size_t capacity) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (model->m.kind != Kind::Recognizer) fail(PPOCR_ERR_INVALID_INPUT, "CTC decode needs a recognizer");
        if (!input || !indices || !probabilities) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        const size_t batch = (size_t)model->m.n, rows = batch * (size_t)model->m.t;
        const size_t chunks = images / batch;
        if (images % batch == 0 && capacity < chunks * rows)
            fail(PPOCR_ERR_INVALID_INPUT, "output arrays hold " + std::to_string(capacity) + " rows; " +
                                              std::to_string(chunks * rows) + " required");
        PipeOutput po;
        po.stage_bytes = rows * 8;
        po.stage = [&](cudaStream_t cs, void* slot) {
            // The finiteness check of the full probability rows (as
            // ppocr_recognizer_forward_ctc does), then the two compact rows.
            cuda_check(launch_check_finite(static_cast<const float*>(model->tensor(model->m.probs)), model->m.output_elements,
                                           model->dflags + 1, cs),
                       "check output");
            cuda_check(launch_copy_words(model->tensor(model->m.index), slot, rows, cs), "stage indices");
            cuda_check(launch_copy_words(model->tensor(model->m.max_prob), static_cast<uint8_t*>(slot) + rows * 4, rows, cs),
                       "stage probabilities");
        };
        po.download = [&](size_t c, const void* slot, cudaStream_t d2h) {
            cuda_check(cudaMemcpyAsync(indices + c * rows, slot, rows * 4, cudaMemcpyDeviceToHost, d2h), "read indices");
            cuda_check(cudaMemcpyAsync(probabilities + c * rows, static_cast<const uint8_t*>(slot) + rows * 4, rows * 4,
                                       cudaMemcpyDeviceToHost, d2h),
                       "read probabilities");
        };
        forward_pipelined(model, input, images, po);
    });
}

int ppocr_model_forward_image(ppocr_model* model, const ppocr_image* image, const float corners[8], size_t content_width,
                              float* output, size_t output_capacity) {
    return guard([&] {
        if (!model || !image || !corners) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (image->gpu != model->gpu) fail(PPOCR_ERR_INVALID_INPUT, "image was uploaded to a different GPU");
        if (model->m.n != 1) fail(PPOCR_ERR_INVALID_INPUT, "image forward requires batch 1");
        if (!output || output_capacity < model->m.output_elements) fail(PPOCR_ERR_INVALID_INPUT, "output buffer is too small");
        for (int i = 0; i < 8; ++i)
            if (!std::isfinite(corners[i])) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: corners must be finite");
        const bool det = model->m.kind == Kind::Detector;
        const size_t cw = det ? (size_t)model->m.w : content_width;
        if (cw == 0 || cw > (size_t)model->m.w) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: content width outside 1..=input width");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        model->gpu->ensure_arena(model->m.plan.arena_bytes);
        PreprocessParams p = make_preprocess(image, corners, cw, (size_t)model->m.h, (size_t)model->m.w, det);
        p.out = static_cast<float*>(model->tensor(model->m.input));
        cuda_check(cudaMemsetAsync(model->dflags, 0, kFlags * sizeof(int), model->gpu->stream), "reset flags");
        cuda_check(launch_preprocess(p, model->gpu->stream), "launch preprocess");
        model->run(model->gpu->stream);
        download(model, model->output_tid(), output, model->m.output_elements * 4);
        finish(model, model->output_tid(), model->m.output_elements);
    });
}

int ppocr_model_benchmark(ppocr_model* model, const float* input, size_t input_len, size_t warmup, size_t runs,
                          double* samples_ms) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (runs > 0 && !samples_ms) fail(PPOCR_ERR_INVALID_INPUT, "samples pointer is null");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        upload_and_run(model, input, input_len);   // upload once (src/gpu/runtime.rs:1814)
        finish(model, -1, 0);
        cudaStream_t s = model->gpu->stream;
        for (size_t i = 0; i < warmup; ++i) model->run(s);
        wait_stream(s, 0, model->gpu);
        cudaEvent_t a, b;
        cuda_check(cudaEventCreate(&a), "event");
        cuda_check(cudaEventCreate(&b), "event");
        for (size_t i = 0; i < runs; ++i) {
            cuda_check(cudaEventRecord(a, s), "record");
            model->run(s);
            cuda_check(cudaEventRecord(b, s), "record");
            wait_stream(s, 0, model->gpu);
            float ms = 0.f;
            cuda_check(cudaEventElapsedTime(&ms, a, b), "elapsed");
            samples_ms[i] = ms;
        }
        cudaEventDestroy(a);
        cudaEventDestroy(b);
        finish(model, -1, 0);   // a pipeline wait that ran out in any run fails the call
    });
}

int ppocr_model_forward_device(ppocr_model* model, const float* device_input, float* device_output, void* stream) {
    return guard([&] {
        if (!model || !device_input || !device_output) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        model->gpu->ensure_arena(model->m.plan.arena_bytes);
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : model->gpu->stream;
        cuda_check(cudaMemsetAsync(model->dflags, 0, kFlags * sizeof(int), s), "reset flags");
        cuda_check(cudaMemcpyAsync(model->tensor(model->m.input), device_input, model->input_elements() * 4,
                                   cudaMemcpyDeviceToDevice, s), "copy input");
        model->run(s);
        cuda_check(cudaMemcpyAsync(device_output, model->tensor(model->output_tid()), model->m.output_elements * 4,
                                   cudaMemcpyDeviceToDevice, s), "copy output");
    });
}

int ppocr_model_device_buffers(ppocr_model* model, float** device_input, float** device_output) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        model->gpu->ensure_arena(model->m.plan.arena_bytes);
        if (device_input) *device_input = static_cast<float*>(model->tensor(model->m.input));
        if (device_output) *device_output = static_cast<float*>(model->tensor(model->output_tid()));
    });
}

int ppocr_model_run(ppocr_model* model, void* stream) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : model->gpu->stream;
        cuda_check(cudaMemsetAsync(model->dflags, 0, kFlags * sizeof(int), s), "reset flags");
        model->run(s);
    });
}

int ppocr_model_synchronize(ppocr_model* model, int timeout_ms) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        model->gpu->bind();
        wait_stream(model->gpu->stream, timeout_ms, model->gpu);
        // Device-resident runs on a caller stream report a tensor-core wait that
        // ran out here, once the caller's stream has completed.
        cuda_check(cudaMemcpyAsync(model->hflags, model->dflags, kFlags * sizeof(int), cudaMemcpyDeviceToHost,
                                   model->gpu->stream), "read flags");
        wait_stream(model->gpu->stream, timeout_ms, model->gpu);
        if (model->hflags[2])
            fail(PPOCR_ERR_GPU, "GPU error: a tensor-core pipeline wait ran out (code " + std::to_string(model->hflags[2]) +
                                    "); the forward's results are incomplete");
    });
}

int ppocr_recognizer_forward_ctc(ppocr_model* model, const float* input, size_t input_len, int32_t* indices, float* probabilities,
                                 float* margins) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (model->m.kind != Kind::Recognizer) fail(PPOCR_ERR_INVALID_INPUT, "CTC decode needs a recognizer");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        upload_and_run(model, input, input_len);
        const size_t rows = (size_t)model->m.n * model->m.t;
        if (indices) download(model, model->m.index, indices, rows * 4);
        if (probabilities) download(model, model->m.max_prob, probabilities, rows * 4);
        if (margins) download(model, model->m.margin, margins, rows * 4);
        finish(model, model->m.probs, model->m.output_elements);
    });
}

namespace {

// Checks of a crop forward's arguments.
void check_crops(const ppocr_model* model, const ppocr_image* const* images, size_t count, const float* corners,
                 const size_t* content_widths) {
    if (!model || !images || !corners || !content_widths) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
    if (model->m.kind != Kind::Recognizer) fail(PPOCR_ERR_INVALID_INPUT, "crop forward needs a recognizer");
    if (count == 0 || count > (size_t)model->m.n)
        fail(PPOCR_ERR_INVALID_INPUT, "crop count " + std::to_string(count) + " is outside 1..=" + std::to_string(model->m.n));
    for (size_t i = 0; i < count; ++i) {
        if (!images[i]) fail(PPOCR_ERR_INVALID_INPUT, "null image");
        if (images[i]->gpu != model->gpu) fail(PPOCR_ERR_INVALID_INPUT, "image was uploaded to a different GPU");
        if (content_widths[i] == 0 || content_widths[i] > (size_t)model->m.w)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: content width outside 1..=input width");
    }
    for (size_t i = 0; i < count * 8; ++i)
        if (!std::isfinite(corners[i])) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: corners must be finite");
}

// Enqueues on the model's stream (lock held): the rectification of the
// crops into input slots 0..count-1, zeros in the unused slots, the forward
// and the copies of the first `count` rows' greedy-CTC statistics to the
// host arrays (any may be null).
void enqueue_crops(ppocr_model* model, const ppocr_image* const* images, size_t count, const float* corners,
                   const size_t* content_widths, int32_t* indices, float* probabilities, float* margins, bool reset_flags) {
    model->gpu->bind();
    model->gpu->ensure_arena(model->m.plan.arena_bytes);
    cudaStream_t s = model->gpu->stream;
    float* in = static_cast<float*>(model->tensor(model->m.input));
    const size_t per = (size_t)3 * model->m.h * model->m.w;
    for (size_t i = 0; i < count; ++i) {
        PreprocessParams p = make_preprocess(images[i], corners + 8 * i, content_widths[i], (size_t)model->m.h,
                                             (size_t)model->m.w, false);
        p.out = in + i * per;
        cuda_check(launch_preprocess(p, s), "launch crop rectification");
    }
    if (count < (size_t)model->m.n)
        cuda_check(cudaMemsetAsync(in + count * per, 0, ((size_t)model->m.n - count) * per * sizeof(float), s),
                   "clear unused crop slots");
    if (reset_flags) cuda_check(cudaMemsetAsync(model->dflags, 0, kFlags * sizeof(int), s), "reset flags");
    model->run(s);
    const size_t rows = count * model->m.t;
    if (indices) download(model, model->m.index, indices, rows * 4);
    if (probabilities) download(model, model->m.max_prob, probabilities, rows * 4);
    if (margins) download(model, model->m.margin, margins, rows * 4);
}

// After the stream wait: a non-finite logit row leaves no arg-max (index -1)
// or a non-finite probability.
void check_ctc_rows(const ppocr_model* model, const int32_t* idx, const float* prob, size_t rows) {
    for (size_t r = 0; r < rows; ++r)
        if (idx[r] < 0 || idx[r] >= model->m.classes || !std::isfinite(prob[r]))
            fail(PPOCR_ERR_GPU, "GPU error: model output contains non-finite values");
}

// Rectifies crops of (possibly different) images into the recognizer's input
// slots 0..count-1, zero-fills the unused slots, runs the forward and returns
// the greedy-CTC statistics of the first `count` rows.
void forward_crops(ppocr_model* model, const ppocr_image* const* images, size_t count, const float* corners,
                   const size_t* content_widths, int32_t* indices, float* probabilities, float* margins) {
    check_crops(model, images, count, corners, content_widths);
    std::lock_guard<std::mutex> lock(model->gpu->mu);
    const size_t rows = count * model->m.t;
    std::vector<int32_t> idx(rows);
    std::vector<float> prob(rows);
    enqueue_crops(model, images, count, corners, content_widths, idx.data(), prob.data(), margins, true);
    cudaStream_t s = model->gpu->stream;
    cuda_check(cudaMemcpyAsync(model->hflags, model->dflags, kFlags * sizeof(int), cudaMemcpyDeviceToHost, s), "read flags");
    wait_stream(s, 0, model->gpu);
    raise_flags(model);
    check_ctc_rows(model, idx.data(), prob.data(), rows);
    if (indices) std::memcpy(indices, idx.data(), rows * 4);
    if (probabilities) std::memcpy(probabilities, prob.data(), rows * 4);
}

}  // namespace

void ppocr::CropBatch::add(ppocr_model* model, const ppocr_image* const* images, size_t count, const float* corners,
                           const size_t* content_widths, int32_t* indices, float* probabilities) {
    check_crops(model, images, count, corners, content_widths);
    if (gpu_ && model->gpu != gpu_) fail(PPOCR_ERR_INVALID_INPUT, "crop batch spans two GPUs");
    gpu_ = model->gpu;
    std::lock_guard<std::mutex> lock(model->gpu->mu);
    const bool first = std::find(models_.begin(), models_.end(), model) == models_.end();
    enqueue_crops(model, images, count, corners, content_widths, indices, probabilities, nullptr, first);
    if (first) models_.push_back(model);
    rows_.push_back({model, indices, probabilities, count * (size_t)model->m.t});
}

void ppocr::CropBatch::wait() {
    if (!gpu_) return;
    {
        std::lock_guard<std::mutex> lock(gpu_->mu);
        gpu_->bind();
        for (ppocr_model* m : models_)
            cuda_check(cudaMemcpyAsync(m->hflags, m->dflags, kFlags * sizeof(int), cudaMemcpyDeviceToHost, gpu_->stream),
                       "read flags");
        wait_stream(gpu_->stream, 0, gpu_);
    }
    for (ppocr_model* m : models_) raise_flags(m);
    for (const Rows& r : rows_) check_ctc_rows(r.model, r.idx, r.prob, r.rows);
    models_.clear();
    rows_.clear();
    gpu_ = nullptr;
}

int ppocr_recognizer_forward_crops(ppocr_model* model, const ppocr_image* image, size_t count, const float* corners,
                                   const size_t* content_widths, int32_t* indices, float* probabilities,
                                   float* margins) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (count != (size_t)model->m.n)
            fail(PPOCR_ERR_INVALID_INPUT, "crop count " + std::to_string(count) + " does not match the batch " +
                                              std::to_string(model->m.n));
        std::vector<const ppocr_image*> images(count, image);
        forward_crops(model, images.data(), count, corners, content_widths, indices, probabilities, margins);
    });
}

int ppocr_recognizer_forward_crops_ex(ppocr_model* model, const ppocr_image* const* images, size_t count,
                                      const float* corners, const size_t* content_widths, int32_t* indices,
                                      float* probabilities, float* margins) {
    return guard([&] { forward_crops(model, images, count, corners, content_widths, indices, probabilities, margins); });
}

int ppocr_detector_forward_images(ppocr_model* model, const ppocr_image* const* images, size_t count,
                                  float* probabilities) {
    return guard([&] {
        if (!model || !images || !probabilities) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (model->m.kind != Kind::Detector) fail(PPOCR_ERR_INVALID_INPUT, "image batch forward needs a detector");
        if (count != (size_t)model->m.n)
            fail(PPOCR_ERR_INVALID_INPUT, "image count " + std::to_string(count) + " does not match the batch " +
                                              std::to_string(model->m.n));
        for (size_t i = 0; i < count; ++i) {
            if (!images[i]) fail(PPOCR_ERR_INVALID_INPUT, "null image");
            if (images[i]->gpu != model->gpu) fail(PPOCR_ERR_INVALID_INPUT, "image was uploaded to a different GPU");
        }
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        model->gpu->ensure_arena(model->m.plan.arena_bytes);
        cudaStream_t s = model->gpu->stream;
        float* in = static_cast<float*>(model->tensor(model->m.input));
        const size_t per = (size_t)3 * model->m.h * model->m.w;
        for (size_t i = 0; i < count; ++i) {
            const float w = (float)images[i]->width, h = (float)images[i]->height;
            const float corners[8] = {0.f, 0.f, w, 0.f, w, h, 0.f, h};
            PreprocessParams p = make_preprocess(images[i], corners, (size_t)model->m.w, (size_t)model->m.h,
                                                 (size_t)model->m.w, true);
            p.out = in + i * per;
            cuda_check(launch_preprocess(p, s), "launch preprocess");
        }
        cuda_check(cudaMemsetAsync(model->dflags, 0, kFlags * sizeof(int), s), "reset flags");
        model->run(s);
        download(model, model->output_tid(), probabilities, model->m.output_elements * 4);
        finish(model, model->output_tid(), model->m.output_elements);
    });
}

int ppocr_model_op_count(const ppocr_model* model, size_t* count) {
    return guard([&] {
        if (!model || !count) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        *count = model->m.plan.ops.size();
    });
}

int ppocr_model_op_info(const ppocr_model* model, size_t index, char* name, size_t name_capacity, char* kind,
                        size_t kind_capacity, double* bytes, double* flops) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (index >= model->m.plan.ops.size()) fail(PPOCR_ERR_INVALID_INPUT, "op index out of range");
        const OpRec& op = model->m.plan.ops[index];
        if (name && name_capacity) {
            std::strncpy(name, op.name.c_str(), name_capacity - 1);
            name[name_capacity - 1] = 0;
        }
        if (kind && kind_capacity) {
            std::strncpy(kind, op.kind.c_str(), kind_capacity - 1);
            kind[kind_capacity - 1] = 0;
        }
        if (bytes) *bytes = model->m.plan.op_bytes(index);
        if (flops) *flops = op.flops;
    });
}

int ppocr_model_tensor_count(const ppocr_model* model, size_t* count) {
    return guard([&] {
        if (!model || !count) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        *count = model->m.plan.tensors.size();
    });
}

int ppocr_model_tensor_info(const ppocr_model* model, size_t index, char* name, size_t name_capacity, size_t shape[4],
                            int* dtype) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (index >= model->m.plan.tensors.size()) fail(PPOCR_ERR_INVALID_INPUT, "tensor index out of range");
        const TensorDesc& t = model->m.plan.tensors[index];
        if (name && name_capacity) {
            std::strncpy(name, t.name.c_str(), name_capacity - 1);
            name[name_capacity - 1] = 0;
        }
        const bool raw = t.n == 0;
        if (shape) {
            shape[0] = raw ? 1 : (size_t)t.n;
            shape[1] = raw ? 1 : (size_t)t.h;
            shape[2] = raw ? 1 : (size_t)t.w;
            shape[3] = raw ? t.bytes / dtype_size(t.dt) : (size_t)t.c;
        }
        if (dtype) *dtype = (int)t.dt;
    });
}

int ppocr_model_read_tensor(ppocr_model* model, size_t index, float* out, size_t capacity) {
    return guard([&] {
        if (!model || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (index >= model->m.plan.tensors.size()) fail(PPOCR_ERR_INVALID_INPUT, "tensor index out of range");
        const TensorDesc& t = model->m.plan.tensors[index];
        const size_t count = t.bytes / dtype_size(t.dt);
        if (capacity < count)
            fail(PPOCR_ERR_INVALID_INPUT, "output buffer holds " + std::to_string(capacity) + " values; " +
                                              std::to_string(count) + " required");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        model->gpu->ensure_arena(model->m.plan.arena_bytes);
        cudaStream_t s = model->gpu->stream;
        if (t.dt == DT_F32) {
            download(model, (int)index, out, count * 4);
        } else {
            std::vector<uint16_t> h(count);
            download(model, (int)index, h.data(), count * 2);
            wait_stream(s, 0, model->gpu);
            for (size_t i = 0; i < count; ++i) {
                const uint32_t u = (uint32_t)h[i] << 16;
                std::memcpy(out + i, &u, 4);
            }
        }
        wait_stream(s, 0, model->gpu);
    });
}

int ppocr_model_profile(ppocr_model* model, size_t runs, double* op_ms) {
    return guard([&] {
        if (!model || !op_ms) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (runs == 0) fail(PPOCR_ERR_INVALID_INPUT, "runs must be positive");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        model->gpu->ensure_arena(model->m.plan.arena_bytes);
        const auto& ops = model->m.plan.ops;
        cudaStream_t s = model->gpu->stream;
        std::vector<cudaEvent_t> ev(ops.size() + 1);
        for (auto& e : ev) cuda_check(cudaEventCreate(&e), "event");
        std::vector<double> acc(ops.size(), 0.0);
        const Ctx c = model->ctx();
        try {
            for (size_t r = 0; r < runs; ++r) {
                cuda_check(cudaEventRecord(ev[0], s), "record");
                for (size_t i = 0; i < ops.size(); ++i) {
                    cuda_check(ops[i].fn(c, s), ops[i].name.c_str());
                    cuda_check(cudaEventRecord(ev[i + 1], s), "record");
                }
                wait_stream(s, 0, model->gpu);
                for (size_t i = 0; i < ops.size(); ++i) {
                    float ms = 0.f;
                    cuda_check(cudaEventElapsedTime(&ms, ev[i], ev[i + 1]), "elapsed");
                    acc[i] += ms;
                }
            }
        } catch (...) {
            for (auto& e : ev) cudaEventDestroy(e);
            throw;
        }
        for (auto& e : ev) cudaEventDestroy(e);
        for (size_t i = 0; i < ops.size(); ++i) op_ms[i] = acc[i] / (double)runs;
    });
}

int ppocr_selftest_wait_expiry(ppocr_gpu* gpu, int kernel, int wait_ms, int* code) {
    return guard([&] {
        if (!gpu || !code) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (kernel < 0 || kernel > 3) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: kernel must be 0..3");
        if (wait_ms < 1 || wait_ms > 2000) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: wait_ms outside 1..=2000");
        *code = 0;
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        // A 256 x 64 x 128 GEMM: two 128-row tiles, so CTA 1 runs normally while
        // CTA 0 waits for the first stage that its producer never loads.
        const int m = 256, n = 64, k = 128, planes = kernel >= 2 ? 3 : 1;
        ConvWeight cw;
        cw.cout = n; cw.cin = k; cw.kh = 1; cw.kw = 1;
        cw.w.assign((size_t)n * k, 0.5f);
        cw.b.assign(n, 0.f);
        WeightBlob blob;
        const int bn = kernel == 3 ? gemm_split_tile_n(n, k) : tc_engine_tile_n(n, planes);
        const int n_pad = kernel == 0 ? (n + 15) / 16 * 16 : (n + bn - 1) / bn * bn, k_pad = (k + 63) / 64 * 64;
        const size_t wo = kernel == 0 ? blob.add_bf16(pack_gemm_nk(cw, n_pad, k_pad)) : blob.add_bf16(pack_engine_kn(cw, planes, n_pad, k_pad));
        const std::vector<float> av((size_t)m * k, 0.25f);
        const size_t ao = planes == 1 ? blob.add_bf16(av) : blob.add_f32(av);
        const size_t co = blob.add_f32(std::vector<float>((size_t)m * n, 0.f));
        const size_t fo = blob.add_f32(std::vector<float>(64, 0.f));   // the wait-expiry flag
        const std::vector<uint8_t>& bytes = blob.bytes();
        char* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes.size()), "allocate wait test buffers");
        int* flag = reinterpret_cast<int*>(d + fo);
        cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
        const uint64_t limit = (uint64_t)wait_ms * 1000000ull;
        if (e == cudaSuccess) {
            if (kernel == 0) {
                GemmParams p;
                p.m = m; p.n = n; p.k = k; p.lda = k; p.k_pad = k_pad; p.n_pad = n_pad;
                p.a = d + ao; p.w_tc = d + wo; p.c = d + co; p.ldc = n; p.c_f32 = 1; p.dtype = DT_BF16;
                p.err = flag; p.wait_ns = limit; p.skip_load = 1;
                e = launch_gemm_tc(p, gpu->stream);
            } else if (kernel == 3) {
                SplitGemmParams p;
                p.m = m; p.n = n; p.k = k; p.lda = k; p.n_pad = n_pad; p.k_pad = k_pad;
                p.a = reinterpret_cast<const float*>(d + ao); p.w = d + wo; p.c = reinterpret_cast<float*>(d + co); p.ldc = n;
                p.err = flag; p.wait_ns = limit; p.skip_load = 1;
                e = launch_gemm_split(p, gpu->stream);
            } else {
                TcEngineParams p;
                p.mode = 0; p.planes = planes; p.m = m; p.n = n; p.k = k; p.n_pad = n_pad; p.k_pad = k_pad;
                p.w = d + wo; p.a = d + ao; p.lda = k; p.c = d + co; p.ldc = n;
                p.err = flag; p.wait_ns = limit; p.skip_load = 1;
                e = launch_tc_engine(p, gpu->stream);
            }
        }
        int h = 0;
        if (e == cudaSuccess) e = cudaMemcpyAsync(&h, flag, sizeof(int), cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        cuda_check(e, "wait-expiry self-test");
        *code = h;
        if (h) fail(PPOCR_ERR_GPU, "GPU error: a tensor-core pipeline wait ran out (code " + std::to_string(h) + ")");
    });
}

int ppocr_selftest_gemm(ppocr_gpu* gpu, int m, int n, int k, const float* a, const float* w, const float* bias, int act,
                        float* c, int* used_tensor_cores, int* wait_error) {
    return guard([&] {
        if (!gpu || !a || !w || !c) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (m <= 0 || n <= 0 || k <= 0 || k % 4) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: GEMM shape (k must be a multiple of 4)");
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        const int kp = (k + 63) / 64 * 64, np = (n + 15) / 16 * 16;
        ConvWeight cw;
        cw.cout = n; cw.cin = k; cw.kh = 1; cw.kw = 1;
        cw.w.assign(w, w + (size_t)n * k);
        cw.b = bias ? std::vector<float>(bias, bias + n) : std::vector<float>(n, 0.f);
        int n_pad4 = 0;
        WeightBlob blob;
        const size_t wf = blob.add_f32(pack_gemm_kn(cw, n_pad4));
        const size_t bo = blob.add_f32(cw.b);
        const size_t wt = blob.add_bf16(pack_gemm_nk(cw, np, kp));
        std::vector<float> av(a, a + (size_t)m * k);
        const size_t ao = blob.add_bf16(av);
        const std::vector<uint8_t>& bytes = blob.bytes();
        char* d = nullptr;
        const size_t cbytes = (size_t)m * n * 4;
        cuda_check(cudaMalloc(&d, bytes.size() + cbytes + 256), "allocate GEMM test buffers");
        cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(gpu->stream);
        GemmParams p;
        p.m = m; p.n = n; p.k = k; p.lda = k; p.n_pad = n_pad4; p.k_pad = kp;
        p.a = d + ao; p.w = reinterpret_cast<const float*>(d + wf); p.w_tc = d + wt;
        p.bias = reinterpret_cast<const float*>(d + bo); p.act = act;
        p.c = d + ((bytes.size() + 255) & ~(size_t)255); p.ldc = n; p.c_f32 = 1; p.dtype = DT_BF16;
        const bool tc = gemm_tc_supported(p);
        if (e == cudaSuccess) e = launch_gemm(p, gpu->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(c, p.c, cbytes, cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        cuda_check(e, "GEMM self-test");
        if (used_tensor_cores) *used_tensor_cores = tc ? 1 : 0;
        const int err = gemm_tc_error_and_clear();
        if (wait_error) *wait_error = err;
    });
}

int ppocr_selftest_gemm_ex(ppocr_gpu* gpu, int m, int n, int k, const float* a, const float* w, const float* bias, int act,
                           const float* residual, int out_bf16, int ldc, int coff, float* c, int* used_tensor_cores,
                           int* wait_error) {
    return guard([&] {
        if (!gpu || !a || !w || !c) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (m <= 0 || n <= 0 || k <= 0 || k % 4) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: GEMM shape (k must be a multiple of 4)");
        if (coff < 0 || ldc < coff + n) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: ldc must cover coff + n");
        if (act < ACT_NONE || act > ACT_SIGMOID) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: activation");
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        const int kp = (k + 63) / 64 * 64, np = (n + 15) / 16 * 16;
        ConvWeight cw;
        cw.cout = n; cw.cin = k; cw.kh = 1; cw.kw = 1;
        cw.w.assign(w, w + (size_t)n * k);
        cw.b = bias ? std::vector<float>(bias, bias + n) : std::vector<float>(n, 0.f);
        int n_pad4 = 0;
        WeightBlob blob;
        const size_t wf = blob.add_f32(pack_gemm_kn(cw, n_pad4));
        const size_t bo = blob.add_f32(cw.b);
        const size_t wt = blob.add_bf16(pack_gemm_nk(cw, np, kp));
        const size_t ao = blob.add_bf16(std::vector<float>(a, a + (size_t)m * k));
        const size_t ro = residual ? blob.add_bf16(std::vector<float>(residual, residual + (size_t)m * n)) : 0;
        const size_t celems = (size_t)m * ldc;
        const std::vector<float> cinit(c, c + celems);
        const size_t co = out_bf16 ? blob.add_bf16(cinit) : blob.add_f32(cinit);
        const std::vector<uint8_t>& bytes = blob.bytes();
        char* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes.size()), "allocate GEMM test buffers");
        cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(gpu->stream);
        GemmParams p;
        p.m = m; p.n = n; p.k = k; p.lda = k; p.n_pad = n_pad4; p.k_pad = kp;
        p.a = d + ao; p.w = reinterpret_cast<const float*>(d + wf); p.w_tc = d + wt;
        p.bias = reinterpret_cast<const float*>(d + bo); p.act = act;
        p.residual = residual ? d + ro : nullptr; p.ldr = n;
        p.c = d + co; p.ldc = ldc; p.coff = coff; p.c_f32 = out_bf16 ? 0 : 1; p.dtype = DT_BF16;
        const bool tc = gemm_tc_supported(p);
        std::vector<uint16_t> hb(out_bf16 ? celems : 0);
        if (e == cudaSuccess) e = launch_gemm(p, gpu->stream);
        if (e == cudaSuccess)
            e = out_bf16 ? cudaMemcpyAsync(hb.data(), p.c, celems * 2, cudaMemcpyDeviceToHost, gpu->stream)
                         : cudaMemcpyAsync(c, p.c, celems * 4, cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        cuda_check(e, "GEMM self-test");
        if (out_bf16)
            for (size_t i = 0; i < celems; ++i) {
                const uint32_t u = (uint32_t)hb[i] << 16;
                std::memcpy(c + i, &u, 4);
            }
        if (used_tensor_cores) *used_tensor_cores = tc ? 1 : 0;
        const int err = gemm_tc_error_and_clear();
        if (wait_error) *wait_error = err;
    });
}

int ppocr_selftest_pair_f32(ppocr_gpu* gpu, int m, int c_in, int c_out, const float* a, const float* w1,
                            const float* b1, const float* w2, const float* b2, const float* gate, int rows_per_image,
                            int residual, float* out) {
    return guard([&] {
        if (!gpu || !a || !w1 || !b1 || !w2 || !b2 || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (m <= 0 || !pair_rows_supported(c_in, c_out)) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: pair shape not covered");
        if (residual && c_out != c_in) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: the residual needs c_out == c_in");
        if (gate && (rows_per_image <= 0 || m % rows_per_image)) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: rows_per_image must divide m");
        const int h = 2 * c_in;
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        std::vector<float> w2t((size_t)h * c_out);   // [2 c_in][c_out], as the model packs it
        for (int o = 0; o < c_out; ++o)
            for (int j = 0; j < h; ++j) w2t[(size_t)j * c_out + o] = w2[(size_t)o * h + j];
        WeightBlob blob;
        const size_t o1 = blob.add_f32(std::vector<float>(w1, w1 + (size_t)h * c_in));
        const size_t o2 = blob.add_f32(w2t);
        const size_t ob1 = blob.add_f32(std::vector<float>(b1, b1 + h));
        const size_t ob2 = blob.add_f32(std::vector<float>(b2, b2 + c_out));
        const size_t ao = blob.add_f32(std::vector<float>(a, a + (size_t)m * c_in));
        const size_t go = gate ? blob.add_f32(std::vector<float>(gate, gate + (size_t)(m / rows_per_image) * c_in)) : 0;
        const size_t co = blob.add_f32(std::vector<float>((size_t)m * c_out, 0.f));
        const std::vector<uint8_t>& bytes = blob.bytes();
        char* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes.size()), "allocate pair test buffers");
        PairRowsParams p;
        p.m = m; p.c_in = c_in; p.c_out = c_out; p.rows_per_image = gate ? rows_per_image : 1;
        p.residual = residual ? 1 : 0; p.dtype = DT_F32;
        p.a = d + ao;
        p.gate = gate ? reinterpret_cast<const float*>(d + go) : nullptr;
        p.w1t = reinterpret_cast<const float*>(d + o1);
        p.w2 = reinterpret_cast<const float*>(d + o2);
        p.b1 = reinterpret_cast<const float*>(d + ob1);
        p.b2 = reinterpret_cast<const float*>(d + ob2);
        p.c = d + co;
        cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(gpu->stream);
        if (e == cudaSuccess) e = launch_pair_rows(p, gpu->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(out, p.c, (size_t)m * c_out * 4, cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        cuda_check(e, "pair self-test");
    });
}

int ppocr_selftest_dwconv(ppocr_gpu* gpu, int n, int hi, int wi, int c, int kh, int kw, int sh, int sw, int pt, int pl,
                          int pb, int pr, const float* x, const float* w, const float* bias, int act,
                          const float* residual, int bf16, int kernel, float* out, int* kernel_used) {
    return guard([&] {
        if (!gpu || !x || !w || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (n <= 0 || hi <= 0 || wi <= 0 || c <= 0 || c % (bf16 ? 8 : 4) || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 ||
            pt < 0 || pl < 0 || pb < 0 || pr < 0)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: depthwise shape");
        if (act < ACT_NONE || act > ACT_SIGMOID) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: activation");
        if (kernel < 0 || kernel > 2) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: kernel must be 0..2");
        const int ho = (hi + pt + pb - kh) / sh + 1, wo = (wi + pl + pr - kw) / sw + 1;
        if (hi + pt + pb < kh || wi + pl + pr < kw) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: kernel larger than the padded input");
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        ConvWeight cw;
        cw.cout = c; cw.cin = 1; cw.kh = kh; cw.kw = kw;
        cw.w.assign(w, w + (size_t)c * kh * kw);
        const size_t in_elems = (size_t)n * hi * wi * c, out_elems = (size_t)n * ho * wo * c;
        WeightBlob blob;
        const size_t wf = blob.add_f32(pack_depthwise(cw));
        const size_t bo = blob.add_f32(bias ? std::vector<float>(bias, bias + c) : std::vector<float>(c, 0.f));
        const std::vector<float> xin(x, x + in_elems);
        const size_t xo = bf16 ? blob.add_bf16(xin) : blob.add_f32(xin);
        size_t ro = 0;
        if (residual) {
            const std::vector<float> rin(residual, residual + out_elems);
            ro = bf16 ? blob.add_bf16(rin) : blob.add_f32(rin);
        }
        const size_t oo = blob.add_f32(std::vector<float>(out_elems, 0.f));   // room for either type
        const std::vector<uint8_t>& bytes = blob.bytes();
        DwParams p;
        p.n = n; p.hi = hi; p.wi = wi; p.c = c; p.in_cstride = c; p.in_coff = 0;
        p.ho = ho; p.wo = wo; p.kh = kh; p.kw = kw; p.sh = sh; p.sw = sw; p.pt = pt; p.pl = pl;
        p.act = act; p.dtype = bf16 ? DT_BF16 : DT_F32;
        char* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes.size()), "allocate depthwise test buffers");
        p.in = d + xo;
        p.weight = reinterpret_cast<const float*>(d + wf);
        p.bias = bias ? reinterpret_cast<const float*>(d + bo) : nullptr;
        p.residual = residual ? d + ro : nullptr;
        p.out = d + oo;
        const int used = kernel != 0 ? kernel : (kh == 3 && kw == 3 ? 2 : 1);
        std::vector<uint16_t> ob(bf16 ? out_elems : 0);
        cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(gpu->stream);
        if (e == cudaSuccess) e = launch_dwconv_kernel(p, gpu->stream, kernel);
        if (e == cudaSuccess)
            e = bf16 ? cudaMemcpyAsync(ob.data(), p.out, out_elems * 2, cudaMemcpyDeviceToHost, gpu->stream)
                     : cudaMemcpyAsync(out, p.out, out_elems * 4, cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        if (e == cudaErrorInvalidValue || e == cudaErrorInvalidConfiguration)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: the chosen depthwise kernel does not support this shape");
        cuda_check(e, "depthwise self-test");
        for (size_t i = 0; i < ob.size(); ++i) {
            const uint32_t u = (uint32_t)ob[i] << 16;
            std::memcpy(out + i, &u, 4);
        }
        if (kernel_used) *kernel_used = used;
    });
}

int ppocr_selftest_conv_split(ppocr_gpu* gpu, int n, int hi, int wi, int cin, int cout, int kh, int kw, int stride, int pad,
                              const float* x, const float* w, const float* bias, int act, const float* residual,
                              float* out) {
    return guard([&] {
        if (!gpu || !x || !w || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (n <= 0 || hi <= 0 || wi <= 0 || cin <= 0 || cout <= 0 || kh <= 0 || kw <= 0 || stride <= 0 || pad < 0)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: conv shape");
        if (act < ACT_NONE || act > ACT_SIGMOID) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: activation");
        const int ho = (hi + 2 * pad - kh) / stride + 1, wo = (wi + 2 * pad - kw) / stride + 1;
        if (ho <= 0 || wo <= 0) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: empty conv output");
        SplitGemmParams p;
        p.conv = 1;
        p.n_img = n; p.hi = hi; p.wi = wi; p.ho = ho; p.wo = wo; p.kh = kh; p.kw = kw; p.stride = stride; p.pt = pad; p.pl = pad;
        const int cpt = gemm_split_conv_cpt(cin);
        p.k = kh * kw * cpt; p.cin = cin; p.n = cout; p.lda = cin; p.ldc = cout; p.coff = 0; p.act = act;
        if (residual) {
            p.residual = residual;   // host pointer for the support check; replaced by the device copy below
            p.ldr = cout;
        }
        const int bn = gemm_split_tile_n(cout, p.k);
        p.n_pad = bn > 0 ? (cout + bn - 1) / bn * bn : 0;
        p.k_pad = (p.k + 63) / 64 * 64;
        p.m = n * ((ho + 7) / 8) * ((wo + 15) / 16) * 128;
        if (!cpt || !gemm_split_supported(p))
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: the split conv takes 32 input channels or more than 32 in multiples of 4");
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        ConvWeight cw;
        cw.cout = cout; cw.cin = cin; cw.kh = kh; cw.kw = kw;
        cw.w.assign(w, w + (size_t)cout * cin * kh * kw);
        cw.b = bias ? std::vector<float>(bias, bias + cout) : std::vector<float>(cout, 0.f);
        const size_t out_elems = (size_t)n * ho * wo * cout;
        WeightBlob blob;
        const size_t wo_ = blob.add_bf16(pack_engine_kn(cw, 3, p.n_pad, p.k_pad, cpt));
        const size_t bo = blob.add_f32(cw.b);
        const size_t xo = blob.add_f32(std::vector<float>(x, x + (size_t)n * hi * wi * cin));
        const size_t co = blob.add_f32(std::vector<float>(out_elems, 0.f));
        const size_t fo = blob.add_f32(std::vector<float>(64, 0.f));
        const size_t ro = residual ? blob.add_f32(std::vector<float>(residual, residual + out_elems)) : 0;
        const std::vector<uint8_t>& bytes = blob.bytes();
        char* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes.size()), "allocate conv test buffers");
        if (residual) p.residual = reinterpret_cast<const float*>(d + ro);
        p.a = reinterpret_cast<const float*>(d + xo); p.w = d + wo_; p.bias = reinterpret_cast<const float*>(d + bo);
        p.c = reinterpret_cast<float*>(d + co);
        p.err = reinterpret_cast<int*>(d + fo);
        int flag = 0;
        cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
        if (e == cudaSuccess) e = launch_gemm_split(p, gpu->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(out, p.c, out_elems * 4, cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(&flag, p.err, sizeof(int), cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        cuda_check(e, "split conv self-test");
        if (flag) fail(PPOCR_ERR_GPU, "GPU error: a tensor-core pipeline wait ran out (code " + std::to_string(flag) + ")");
    });
}

int ppocr_selftest_gemm_f32(ppocr_gpu* gpu, int m, int n, int k, const float* a, const float* w, const float* bias,
                            int act, const float* gate, int rows_per_image, const float* residual, int kernel, float* c,
                            int* kernel_used) {
    return guard([&] {
        if (!gpu || !a || !w || !c) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (m <= 0 || n <= 0 || k <= 0 || k % 4) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: GEMM shape (k must be a multiple of 4)");
        if (act < ACT_NONE || act > ACT_SIGMOID) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: activation");
        if (kernel < 0 || kernel > 5) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: kernel must be 0..5");
        if (gate && (rows_per_image <= 0 || m % rows_per_image)) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: rows_per_image must divide m");
        if (kernel == 4 || kernel == 5) {
            // The FP32-class tcgen05 split GEMM (5: A pre-split into its pieces by
            // its own kernel first).
            SplitGemmParams p;
            p.m = m; p.n = n; p.k = k; p.lda = k; p.ldc = n; p.ldr = n; p.act = act;
            p.rows_per_image = gate ? rows_per_image : 1;
            const int bn = gemm_split_tile_n(n, k);
            p.n_pad = bn > 0 ? (n + bn - 1) / bn * bn : 0;
            p.k_pad = (k + 63) / 64 * 64;
            if (!gemm_split_supported(p)) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: the split GEMM needs k % 16 == 0");
            std::lock_guard<std::mutex> lock(gpu->mu);
            gpu->bind();
            ConvWeight cw;
            cw.cout = n; cw.cin = k; cw.kh = 1; cw.kw = 1;
            cw.w.assign(w, w + (size_t)n * k);
            cw.b = bias ? std::vector<float>(bias, bias + n) : std::vector<float>(n, 0.f);
            WeightBlob blob;
            const size_t wo = blob.add_bf16(pack_engine_kn(cw, 3, p.n_pad, p.k_pad));
            const size_t bo = blob.add_f32(cw.b);
            const size_t ao = blob.add_f32(std::vector<float>(a, a + (size_t)m * k));
            const size_t go = gate ? blob.add_f32(std::vector<float>(gate, gate + (size_t)(m / rows_per_image) * k)) : 0;
            const size_t ro = residual ? blob.add_f32(std::vector<float>(residual, residual + (size_t)m * n)) : 0;
            const size_t co = blob.add_f32(std::vector<float>((size_t)m * n, 0.f));
            const size_t fo = blob.add_f32(std::vector<float>(64, 0.f));
            const size_t po = kernel == 5 ? blob.add_f32(std::vector<float>((size_t)3 * m * p.k_pad / 2, 0.f)) : 0;
            const std::vector<uint8_t>& bytes = blob.bytes();
            char* d = nullptr;
            cuda_check(cudaMalloc(&d, bytes.size()), "allocate GEMM test buffers");
            p.a = reinterpret_cast<const float*>(d + ao); p.w = d + wo; p.bias = reinterpret_cast<const float*>(d + bo);
            p.gate = gate ? reinterpret_cast<const float*>(d + go) : nullptr;
            p.residual = residual ? reinterpret_cast<const float*>(d + ro) : nullptr;
            p.c = reinterpret_cast<float*>(d + co);
            p.err = reinterpret_cast<int*>(d + fo);
            int flag = 0;
            cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
            if (e == cudaSuccess && kernel == 5) {
                e = launch_split_planes(p, d + po, gpu->stream);
                p.a_planes = d + po;
            }
            if (e == cudaSuccess) e = launch_gemm_split(p, gpu->stream);
            if (e == cudaSuccess) e = cudaMemcpyAsync(c, p.c, (size_t)m * n * 4, cudaMemcpyDeviceToHost, gpu->stream);
            if (e == cudaSuccess) e = cudaMemcpyAsync(&flag, p.err, sizeof(int), cudaMemcpyDeviceToHost, gpu->stream);
            if (e == cudaSuccess) {
                try {
                    wait_stream(gpu->stream, 0, gpu);
                } catch (...) {
                    cudaFree(d);
                    throw;
                }
            }
            cudaFree(d);
            cuda_check(e, "split GEMM self-test");
            if (flag) fail(PPOCR_ERR_GPU, "GPU error: a tensor-core pipeline wait ran out (code " + std::to_string(flag) + ")");
            if (kernel_used) *kernel_used = kernel;
            return;
        }
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        ConvWeight cw;
        cw.cout = n; cw.cin = k; cw.kh = 1; cw.kw = 1;
        cw.w.assign(w, w + (size_t)n * k);
        cw.b = bias ? std::vector<float>(bias, bias + n) : std::vector<float>(n, 0.f);
        int n_pad4 = 0;
        WeightBlob blob;
        const size_t wf = blob.add_f32(pack_gemm_kn(cw, n_pad4));
        const size_t bo = blob.add_f32(cw.b);
        const size_t ao = blob.add_f32(std::vector<float>(a, a + (size_t)m * k));
        const size_t go = gate ? blob.add_f32(std::vector<float>(gate, gate + (size_t)(m / rows_per_image) * k)) : 0;
        const size_t ro = residual ? blob.add_f32(std::vector<float>(residual, residual + (size_t)m * n)) : 0;
        const size_t co = blob.add_f32(std::vector<float>((size_t)m * n, 0.f));
        const std::vector<uint8_t>& bytes = blob.bytes();
        GemmParams p;
        p.m = m; p.n = n; p.k = k; p.lda = k; p.n_pad = n_pad4;
        p.act = act; p.ldr = n; p.ldc = n; p.coff = 0; p.c_f32 = 0; p.dtype = DT_F32;
        p.rows_per_image = gate ? rows_per_image : 1;
        char* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes.size()), "allocate GEMM test buffers");
        p.a = d + ao; p.w = reinterpret_cast<const float*>(d + wf);
        p.bias = reinterpret_cast<const float*>(d + bo);
        p.gate = gate ? reinterpret_cast<const float*>(d + go) : nullptr;
        p.residual = residual ? d + ro : nullptr;
        p.c = d + co;
        int used = kernel;
        if (kernel == 0) used = p.n <= 32 && gemm_stream_supported(p) ? 3 : 1;   // launch_gemm's FP32 choice
        const bool ok = used == 1 || (used == 2 && rows_gemm_supported(p)) || (used == 3 && gemm_stream_supported(p));
        if (!ok) {
            cudaFree(d);
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: the chosen GEMM kernel does not support this shape");
        }
        cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(gpu->stream);
        if (e == cudaSuccess)
            e = used == 3 ? launch_gemm_stream(p, gpu->stream) : used == 2 ? launch_rows_gemm(p, gpu->stream)
                                                                 : launch_gemm_simt(p, gpu->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(c, p.c, (size_t)m * n * 4, cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        cuda_check(e, "FP32 GEMM self-test");
        if (kernel_used) *kernel_used = used;
    });
}

int ppocr_measure_fp32_peak(ppocr_gpu* gpu, double* tflops_fma, double* tflops_fma2) {
    return guard([&] {
        if (!gpu || !tflops_fma || !tflops_fma2) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        int dev = 0, sms = 0;
        cuda_check(cudaGetDevice(&dev), "query device");
        cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "query SM count");
        float* sink = nullptr;
        cuda_check(cudaMalloc(&sink, sizeof(float)), "allocate probe sink");
        cudaEvent_t e0 = nullptr, e1 = nullptr;
        cudaError_t e = cudaEventCreate(&e0);
        if (e == cudaSuccess) e = cudaEventCreate(&e1);
        const int blocks = sms * 4, iters = 20000;
        const double flops = 2.0 * 16 * iters * 512.0 * blocks;
        double best[2] = {0.0, 0.0};
        for (int packed = 0; packed < 2 && e == cudaSuccess; ++packed)
            for (int rep = 0; rep < 3 && e == cudaSuccess; ++rep) {
                e = cudaEventRecord(e0, gpu->stream);
                if (e == cudaSuccess) e = launch_fp32_peak(sink, blocks, iters, packed != 0, gpu->stream);
                if (e == cudaSuccess) e = cudaEventRecord(e1, gpu->stream);
                if (e == cudaSuccess) e = cudaEventSynchronize(e1);
                float ms = 0.f;
                if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
                if (e == cudaSuccess && ms > 0.f) best[packed] = std::max(best[packed], flops / (ms * 1e-3) / 1e12);
            }
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        cudaFree(sink);
        cuda_check(e, "FP32 throughput probe");
        *tflops_fma = best[0];
        *tflops_fma2 = best[1];
    });
}

int ppocr_selftest_engine(ppocr_gpu* gpu, int planes, int n, int hi, int wi, int cin, int cout, int kh, int kw, int stride,
                          int pad, int second, const float* x, const float* x2, const float* w, const float* bias, int act,
                          float* out, int* used_tensor_cores, int* wait_error) {
    return guard([&] {
        if (!gpu || !x || !w || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (planes != 1 && planes != 3) fail(PPOCR_ERR_INVALID_INPUT, "planes must be 1 or 3");
        const int ch = planes == 1 ? 8 : 4;
        if (n <= 0 || hi <= 0 || wi <= 0 || cin <= 0 || cout <= 0 || kh <= 0 || kw <= 0 || stride <= 0 || pad < 0 ||
            cin % (second ? 2 * ch : ch) || second < 0 || second > 2 || (second == 2 && (!x2 || hi % 2 || wi % 2)))
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: engine test shape");
        const int ho = (hi + 2 * pad - kh) / stride + 1, wo = (wi + 2 * pad - kw) / stride + 1;
        if (ho <= 0 || wo <= 0) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: empty output");
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        ConvWeight cw;
        cw.cout = cout; cw.cin = cin; cw.kh = kh; cw.kw = kw;
        cw.w.assign(w, w + (size_t)cout * cin * kh * kw);
        cw.b = bias ? std::vector<float>(bias, bias + cout) : std::vector<float>(cout, 0.f);
        TcEngineParams p;
        p.planes = planes;
        p.mode = (kh == 1 && kw == 1 && stride == 1 && pad == 0 && !second) ? 0 : 1;
        p.m = n * ho * wo; p.n = cout; p.k = kh * kw * cin;
        const int bn = tc_engine_tile_n(cout, planes);
        p.n_pad = (cout + bn - 1) / bn * bn;
        p.k_pad = (p.k + 63) / 64 * 64;
        p.lda = cin; p.act = act; p.out_h = ho; p.out_w = wo; p.ldc = cout;
        ConvGather& g = p.conv;
        g.hi = hi; g.wi = wi; g.ho = ho; g.wo = wo; g.cin = cin; g.kh = kh; g.kw = kw; g.sh = stride; g.sw = stride;
        g.pt = pad; g.pl = pad;
        WeightBlob blob;
        const size_t wof = blob.add_bf16(pack_engine_kn(cw, planes, p.n_pad, p.k_pad));
        const size_t bo = blob.add_f32(cw.b);
        const size_t xn = (size_t)n * hi * wi * cin;
        std::vector<float> xv(x, x + xn);
        const size_t xo = planes == 1 ? blob.add_bf16(xv) : blob.add_f32(xv);
        size_t x2o = 0;
        if (second == 2) {
            std::vector<float> v2(x2, x2 + (size_t)n * (hi / 2) * (wi / 2) * (cin / 2));
            x2o = planes == 1 ? blob.add_bf16(v2) : blob.add_f32(v2);
        }
        const std::vector<uint8_t>& bytes = blob.bytes();
        const size_t esize = planes == 1 ? 2 : 4;
        const size_t cbytes = (size_t)p.m * cout * esize;
        char* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes.size() + cbytes + 256), "allocate engine test buffers");
        cudaError_t e = cudaMemcpyAsync(d, bytes.data(), bytes.size(), cudaMemcpyHostToDevice, gpu->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(gpu->stream);
        p.w = d + wof;
        p.bias = reinterpret_cast<const float*>(d + bo);
        p.a = d + xo;
        if (!second) {
            g.nsrc = 1;
            g.src[0] = ConvSource{d + xo, cin, cin, 0, 1, SRC_NHWC};
        } else if (second == 1) {
            // Both halves are views of the one [n, hi, wi, cin] tensor: channels
            // [0, cin/2) direct, [cin/2, cin) max-pooled.
            g.nsrc = 2;
            g.src[0] = ConvSource{d + xo, cin / 2, cin, 0, 1, SRC_NHWC};
            g.src[1] = ConvSource{d + xo, cin / 2, cin, cin / 2, 1, SRC_NHWC_MAXPOOL};
        } else {
            g.nsrc = 2;
            g.src[0] = ConvSource{d + xo, cin / 2, cin, 0, 1, SRC_NHWC};
            g.src[1] = ConvSource{d + x2o, cin / 2, cin / 2, 0, 2, SRC_NHWC};
        }
        p.c = d + ((bytes.size() + 255) & ~(size_t)255);
        const bool tc = tc_engine_supported(p);
        std::vector<uint16_t> hb(planes == 1 ? (size_t)p.m * cout : 0);
        if (e == cudaSuccess) e = launch_tc_engine(p, gpu->stream);
        if (e == cudaSuccess)
            e = planes == 1 ? cudaMemcpyAsync(hb.data(), p.c, cbytes, cudaMemcpyDeviceToHost, gpu->stream)
                            : cudaMemcpyAsync(out, p.c, cbytes, cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        cuda_check(e, "engine self-test");
        if (planes == 1)
            for (size_t i = 0; i < hb.size(); ++i) {
                const uint32_t u = (uint32_t)hb[i] << 16;
                std::memcpy(out + i, &u, 4);
            }
        if (used_tensor_cores) *used_tensor_cores = tc ? 1 : 0;
        const int err = tc_engine_error_and_clear();
        if (wait_error) *wait_error = err;
    });
}

int ppocr_recognizer_forward_logits(ppocr_model* model, const float* input, size_t input_len, float* logits,
                                    size_t logits_capacity) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (model->m.kind != Kind::Recognizer) fail(PPOCR_ERR_INVALID_INPUT, "logits output needs a recognizer");
        if (!logits || logits_capacity < model->m.output_elements) fail(PPOCR_ERR_INVALID_INPUT, "logits buffer is too small");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        upload_and_run(model, input, input_len);
        const size_t classes = (size_t)model->m.classes, ld = (size_t)model->m.logits_ld;
        const size_t rows = model->m.output_elements / classes;
        cuda_check(cudaMemcpy2DAsync(logits, classes * 4, model->tensor(model->m.logits), ld * 4, classes * 4, rows,
                                     cudaMemcpyDeviceToHost, model->gpu->stream),
                   "read logits");
        finish(model, model->m.logits, rows, classes, ld);
    });
}

int ppocr_preprocess(ppocr_gpu* gpu, const ppocr_image* image, const float corners[8], size_t content_width, size_t out_h,
                     size_t out_w, int kind, float* output) {
    return guard([&] {
        if (!gpu || !image || !corners || !output) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (image->gpu != gpu) fail(PPOCR_ERR_INVALID_INPUT, "image was uploaded to a different GPU");
        if (kind != 0 && kind != 1) fail(PPOCR_ERR_INVALID_INPUT, "kind must be 0 (detector) or 1 (recognizer)");
        if (out_h == 0 || out_w == 0 || content_width == 0 || content_width > out_w)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: content width outside 1..=output width");
        for (int i = 0; i < 8; ++i)
            if (!std::isfinite(corners[i])) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: corners must be finite");
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        PreprocessParams p = make_preprocess(image, corners, content_width, out_h, out_w, kind == 0);
        const size_t bytes = 3 * out_h * out_w * 4;
        float* d = nullptr;
        cuda_check(cudaMalloc(&d, bytes), "allocate preprocess output");
        p.out = d;
        cudaError_t e = launch_preprocess(p, gpu->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(output, d, bytes, cudaMemcpyDeviceToHost, gpu->stream);
        if (e == cudaSuccess) {
            try {
                wait_stream(gpu->stream, 0, gpu);
            } catch (...) {
                // After a wait that ran out the kernel may still write `d`: it is
                // left allocated rather than freed under it.
                if (!gpu->poisoned) cudaFree(d);
                throw;
            }
        }
        cudaFree(d);
        cuda_check(e, "preprocess");
    });
}

int ppocr_detector_forward_mask(ppocr_model* model, const float* input, size_t input_len, float threshold, float* probabilities,
                                uint8_t* mask) {
    return guard([&] {
        if (!model) fail(PPOCR_ERR_INVALID_INPUT, "model is null");
        if (model->m.kind != Kind::Detector) fail(PPOCR_ERR_INVALID_INPUT, "mask output needs a detector");
        if (!(threshold >= 0.f && threshold <= 1.f)) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: threshold must be in [0, 1]");
        std::lock_guard<std::mutex> lock(model->gpu->mu);
        model->gpu->bind();
        *model->m.mask_threshold = threshold;
        upload_and_run(model, input, input_len);
        if (probabilities) download(model, model->m.prob, probabilities, model->m.output_elements * 4);
        if (mask) download(model, model->m.mask, mask, model->m.output_elements);
        finish(model, model->m.prob, model->m.output_elements);
    });
}

}  // extern "C"
