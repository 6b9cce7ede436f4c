// Static execution plan of one (model, input shape): activation tensors,
// the op list, and an offline arena layout.
//
// Tensors live in one per-device arena; the planner assigns offsets by
// greedy interval colouring over op-index lifetimes (largest first, lowest
// offset that does not overlap a tensor alive at the same time), the same
// job as ppocr-rs's ArenaAllocator / compact_layout (src/gpu/runtime.rs:414-557).
// A tensor touched inside a concurrent region is live for the whole region,
// so ops that may run at the same time never share memory.
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
    // Second stream and the fork / join events of concurrent regions (null:
    // every op on the launch stream).
    cudaStream_t side = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
    // Device flag the tensor-core kernels set when a pipeline wait runs out
    // (read back with the forward's other flags); null: their own globals.
    int* err = nullptr;
    // Per-model arrival counters of the fused SE kernels (zero between launches).
    int* counters = nullptr;
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
    int lane = 0;              // inside a concurrent region: 0 the launch stream, 1 the side stream
};

// Ops [begin, end) whose lane-1 ops run on a second stream, concurrently with
// the region's lane-0 ops: the side stream waits for everything enqueued
// before the region, and the launch stream waits for the side stream at its
// end.  Lane-1 ops must not depend on the region's lane-0 ops or vice versa.
struct Region {
    int begin = 0, end = 0;
};

struct Plan {
    std::vector<TensorDesc> tensors;
    std::vector<OpRec> ops;
    std::vector<Region> regions;
    int lane = 0;               // lane of the ops added next
    size_t arena_bytes = 0;

    // Concurrent regions: ops added between begin_region and end_region with
    // set_lane(1) form the side lane.  Regions do not nest.
    void begin_region() { regions.push_back({(int)ops.size(), -1}); }
    void end_region() { regions.back().end = (int)ops.size(); lane = 0; }
    void set_lane(int l) { lane = l; }

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
