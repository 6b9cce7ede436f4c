// Internal definitions shared by the C-ABI translation units: the device and
// image handles, the status/last-error plumbing and the bounded stream wait.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../kernels/kernels.h"
#include "common.hpp"
#include "ppocr_b200.h"

namespace ppocr {

// Message of the last failure on the calling thread (ppocr_last_error()).
std::string& last_error();

// Runs `f`, turning an Error into its status code and recording the message.
template <typename F>
int guard(F&& f) {
    try {
        f();
        last_error().clear();
        return PPOCR_OK;
    } catch (const Error& e) {
        last_error() = e.what();
        return e.code;
    } catch (const std::bad_alloc&) {
        last_error() = "out of host memory";
        return PPOCR_ERR_GPU;
    } catch (const std::exception& e) {
        last_error() = e.what();
        return PPOCR_ERR_GPU;
    }
}

// Waits for `s` with a deadline (<= 0: 60 s); Error::Gpu on expiry or a device
// error.  On expiry `owner` (if given) is marked poisoned: its queued work may
// still write the caller's buffers, so every later call on it fails at once.
void wait_stream(cudaStream_t s, int timeout_ms, ppocr_gpu* owner = nullptr);

}  // namespace ppocr

struct ppocr_gpu {
    // References: the caller's handle plus every model, image and engine made
    // on this device (the reference's Gpu is Clone over an Arc, so its models
    // keep it alive, src/gpu/runtime.rs:88-92).  The device resources are freed
    // when the last one is released.
    std::atomic<int> refs{1};
    std::atomic<bool> poisoned{false};   // a wait on this device ran out (see wait_stream)
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaStream_t side = nullptr;                            // concurrent regions' second stream
    cudaEvent_t fork = nullptr, join = nullptr;             // their fork / join events
    std::mutex mu;
    void* arena = nullptr;
    size_t arena_bytes = 0;
    uint64_t arena_gen = 0;
    std::string name;

    void bind() const {
        if (poisoned)
            ppocr::fail(PPOCR_ERR_GPU, "GPU error: an earlier call's device work did not finish within the wait limit; "
                                       "this handle accepts no further work");
        ppocr::cuda_check(cudaSetDevice(device), "cudaSetDevice");
    }
    void ensure_arena(size_t bytes) {
        if (bytes <= arena_bytes) return;
        ppocr::cuda_check(cudaStreamSynchronize(stream), "synchronize before arena growth");
        if (arena) cudaFree(arena);
        arena = nullptr;
        arena_bytes = 0;
        ppocr::cuda_check(cudaMalloc(&arena, bytes), "allocate activation arena");
        arena_bytes = bytes;
        ++arena_gen;
    }
};

struct ppocr_image {
    ppocr_gpu* gpu = nullptr;
    uint8_t* rgb = nullptr;
    uint32_t width = 0, height = 0;
    size_t capacity = 0;   // bytes allocated at rgb (a reused engine page buffer may hold a smaller page)
};

namespace ppocr {
void gpu_retain(ppocr_gpu* gpu);
void gpu_release(ppocr_gpu* gpu);

// Quad-resample parameters for `image` (Normalization::new, src/preprocess/kernels.rs:9-18).
PreprocessParams make_preprocess(const ppocr_image* image, const float corners[8], size_t content_width, size_t out_h,
                                 size_t out_w, bool detector);

// Guards a caller's input memory for work that may outlive the call (an engine
// pool worker that missed the call's deadline): the memory is read only
// between a successful enter() and leave(); close() (the call returning)
// refuses later entries and waits for the readers inside.
class CallGate {
public:
    bool enter() {
        std::lock_guard<std::mutex> lock(mu_);
        if (!open_) return false;
        ++readers_;
        return true;
    }
    void leave() {
        std::lock_guard<std::mutex> lock(mu_);
        --readers_;
        cv_.notify_all();
    }
    void close() {
        std::unique_lock<std::mutex> lock(mu_);
        open_ = false;
        cv_.wait(lock, [&] { return readers_ == 0; });
    }

private:
    std::mutex mu_;
    std::condition_variable cv_;
    bool open_ = true;
    int readers_ = 0;
};

// Recognizer crop forwards enqueued back to back on one device's stream and
// waited for once (the engine's recognition stage: one forward per chunk
// canvas width).  add() enqueues what ppocr_recognizer_forward_crops_ex runs,
// with the greedy-CTC rows copied to `indices` / `probabilities`, which must be
// page-locked host memory valid until wait(); wait() synchronises, then raises
// the models' errors as the single-forward call would.  A model's device
// flags are reset at its first forward of the batch and read back once.
class CropBatch {
public:
    CropBatch() = default;
    CropBatch(const CropBatch&) = delete;
    CropBatch& operator=(const CropBatch&) = delete;
    // An unfinished batch (an error between add() and wait()) still waits for
    // its copies before the host buffers can be reused.
    ~CropBatch() {
        try {
            wait();
        } catch (...) {
        }
    }
    void add(ppocr_model* model, const ppocr_image* const* images, size_t count, const float* corners,
             const size_t* content_widths, int32_t* indices, float* probabilities);
    void wait();

private:
    struct Rows {
        const ppocr_model* model;
        const int32_t* idx;
        const float* prob;
        size_t rows;
    };
    ppocr_gpu* gpu_ = nullptr;
    std::vector<ppocr_model*> models_;
    std::vector<Rows> rows_;
};

// ppocr_engine_recognize_batch with the results as strings; the page bytes
// are read only inside `gate` (null: no gate).  Error::InvalidInput when the
// gate has closed before the pages were read.
std::vector<std::string> engine_recognize(ppocr_engine* engine, size_t count, const uint8_t* const* rgb,
                                          const size_t* rgb_lengths, const uint32_t* widths, const uint32_t* heights,
                                          int format, CallGate* gate);
}  // namespace ppocr
