// Error model of the host runtime.  Every failure is an Error carrying one of
// the ppocr_status codes (one per `gpu::Error` variant, ppocr-rs
// src/gpu/error.rs:8-45) and a message in the reference's wording.
#pragma once

#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "ppocr_b200.h"

namespace ppocr {

struct Error : std::runtime_error {
    int code;
    Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

[[noreturn]] inline void fail(int code, const std::string& message) { throw Error(code, message); }

inline void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) fail(PPOCR_ERR_GPU, std::string(what) + ": " + cudaGetErrorString(e));
}

}  // namespace ppocr
