// Static execution plan of one (model, input shape): activation tensors,
// the op list, and an offline arena layout.
//
// Tensors live in one per-device arena; the planner assigns offsets by
// greedy interval colouring over op-index lifetimes (largest first, lowest
// offset that does not overlap a tensor alive at the same time), the same
// job as ppocr-rs's ArenaAllocator / compact_layout (src/gpu/runtime.rs:414-557).
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <string>
#include <vector>

#include "../kernels/kernels.h"

namespace ppocr {

struct TensorDesc {
    int n = 0, h = 0, w = 0, c = 0;
    DType dt = DT_F32;
    size_t bytes = 0;
    int first = -1, last = -1;   // op indices of first write / last read
    bool pinned = false;         // live for the whole plan (inputs / outputs)
    size_t offset = 0;
    std::string name;
};

// Resolves tensor ids and weight offsets to device pointers at launch time.
struct Ctx {
    char* arena = nullptr;
    const char* weights = nullptr;
    const std::vector<TensorDesc>* tensors = nullptr;
    void* act(int tid) const { return tid < 0 ? nullptr : arena + (*tensors)[tid].offset; }
    const float* wf(size_t off) const { return reinterpret_cast<const float*>(weights + off); }
    const void* wb(size_t off) const { return weights + off; }
};

using OpFn = std::function<cudaError_t(const Ctx&, cudaStream_t)>;

struct OpRec {
    std::string name;
    OpFn fn;
    std::vector<int> reads, writes;
    std::string kind;          // kernel family: conv, dwconv, gemm, se, gate, head, ...
    double weight_bytes = 0;   // parameter bytes the kernel reads
    double flops = 0;          // algorithmic multiply-adds x 2
};

struct Plan {
    std::vector<TensorDesc> tensors;
    std::vector<OpRec> ops;
    size_t arena_bytes = 0;

    int add_tensor(const std::string& name, int n, int h, int w, int c, DType dt, bool pinned = false);
    int add_raw(const std::string& name, size_t bytes, bool pinned = false);
    void add_op(const std::string& name, std::vector<int> reads, std::vector<int> writes, OpFn fn,
                const std::string& kind = "misc", double weight_bytes = 0, double flops = 0);
    // Algorithmic bytes of op i: every tensor it reads and writes once, plus its weights.
    double op_bytes(size_t i) const;
    // Computes lifetimes and offsets; returns the arena size in bytes.
    size_t finalize();
    // Enqueues every op on `stream`; throws Error(GPU) on a launch failure.
    void run(const Ctx& ctx, cudaStream_t stream) const;
};

}  // namespace ppocr
