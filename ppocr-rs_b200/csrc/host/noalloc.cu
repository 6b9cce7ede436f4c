// Device preprocessing for callers that cannot allocate GPU memory.
//
// ppocr_preprocess stages the resampled image in a device buffer it
// allocates with cudaMalloc on every call before copying it to the caller's
// host array.  Some callers cannot allow that: code running under a fixed
// device-memory budget or a custom allocator that owns all device memory, and
// hosts that forbid allocation calls while they are serving (cudaMalloc
// synchronises the device and may fail late under memory pressure).
// ppocr_preprocess_noalloc runs the same kernel but stages its output in the
// file-scope array below, so it makes no allocation call at all.
//
// The array is a fixed 4 MiB (1 Mi floats) on every GPU that loads this
// library, held until the process exits; outputs larger than that are
// rejected.  All calls on a device share it: two calls whose GPU work
// overlaps (different threads, or different streams of the same device)
// race on it and must be serialised by the caller.  It keeps the last call's
// contents; nothing needs clearing because the kernel writes every element
// of the output, including the zero padding past content_width.
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "../kernels/kernels.h"
#include "handles.hpp"

namespace {

constexpr size_t kNoAllocFloats = size_t(1) << 20;   // 3 * out_h * out_w must not exceed this
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats];

std::mutex g_addr_mu;
float* g_addr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device.  In host code
// the array's name is only a host-side stand-in, so the address is looked up
// once per device (with that device current) and cached.
float* scratch_address(int device) {
    if (device < 0 || device >= kMaxDevices) ppocr::fail(PPOCR_ERR_GPU, "device index out of range for the scratch table");
    std::lock_guard<std::mutex> lock(g_addr_mu);
    if (!g_addr[device]) {
        void* p = nullptr;
        ppocr::cuda_check(cudaGetSymbolAddress(&p, g_noalloc_scratch), "look up the preprocessing scratch address");
        g_addr[device] = static_cast<float*>(p);
    }
    return g_addr[device];
}

}  // namespace

extern "C" int ppocr_preprocess_noalloc(ppocr_gpu* gpu, const ppocr_image* image, const float corners[8],
                                        size_t content_width, size_t out_h, size_t out_w, int kind, float* output) {
    using namespace ppocr;
    return guard([&] {
        if (!gpu || !image || !corners || !output) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (image->gpu != gpu) fail(PPOCR_ERR_INVALID_INPUT, "image was uploaded to a different GPU");
        if (kind != 0 && kind != 1) fail(PPOCR_ERR_INVALID_INPUT, "kind must be 0 (detector) or 1 (recognizer)");
        if (out_h == 0 || out_w == 0 || content_width == 0 || content_width > out_w)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: content width outside 1..=output width");
        if (out_h > kNoAllocFloats || out_w > kNoAllocFloats || 3 * out_h * out_w > kNoAllocFloats)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: 3 x " + std::to_string(out_h) + " x " + std::to_string(out_w) +
                                              " floats exceed the no-allocation preprocessing limit of " +
                                              std::to_string(kNoAllocFloats) + " floats");
        for (int i = 0; i < 8; ++i)
            if (!std::isfinite(corners[i])) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: corners must be finite");
        std::lock_guard<std::mutex> lock(gpu->mu);
        gpu->bind();
        PreprocessParams p = make_preprocess(image, corners, content_width, out_h, out_w, kind == 0);
        p.out = scratch_address(gpu->device);
        cuda_check(launch_preprocess(p, gpu->stream), "preprocess");
        cuda_check(cudaMemcpyAsync(output, p.out, 3 * out_h * out_w * sizeof(float), cudaMemcpyDeviceToHost, gpu->stream),
                   "read preprocess output");
        wait_stream(gpu->stream, 0, gpu);
    });
}
