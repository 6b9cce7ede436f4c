#include "graph.hpp"

#include <algorithm>

#include "common.hpp"

namespace ppocr {

int Plan::add_tensor(const std::string& name, int n, int h, int w, int c, DType dt, bool pinned) {
    TensorDesc t;
    t.n = n; t.h = h; t.w = w; t.c = c; t.dt = dt; t.pinned = pinned; t.name = name;
    t.bytes = (size_t)n * h * w * c * dtype_size(dt);
    tensors.push_back(t);
    return (int)tensors.size() - 1;
}

int Plan::add_raw(const std::string& name, size_t bytes, bool pinned) {
    TensorDesc t;
    t.bytes = bytes; t.pinned = pinned; t.name = name; t.c = 1;
    tensors.push_back(t);
    return (int)tensors.size() - 1;
}

double Plan::op_bytes(size_t i) const {
    const OpRec& op = ops[i];
    double b = op.weight_bytes;
    for (int t : op.reads) b += (double)tensors[t].bytes;
    for (int t : op.writes) b += (double)tensors[t].bytes;
    return b;
}

void Plan::add_op(const std::string& name, std::vector<int> reads, std::vector<int> writes, OpFn fn, const std::string& kind,
                  double weight_bytes, double flops) {
    OpRec r;
    r.name = name;
    r.kind = kind;
    r.weight_bytes = weight_bytes;
    r.flops = flops;
    r.fn = std::move(fn);
    reads.erase(std::remove(reads.begin(), reads.end(), -1), reads.end());
    writes.erase(std::remove(writes.begin(), writes.end(), -1), writes.end());
    r.reads = std::move(reads);
    r.writes = std::move(writes);
    r.lane = lane;
    ops.push_back(std::move(r));
}

size_t Plan::finalize() {
    const int nops = (int)ops.size();
    for (auto& t : tensors) { t.first = -1; t.last = -1; }
    for (int i = 0; i < nops; ++i) {
        for (int tid : ops[i].writes) {
            auto& t = tensors[tid];
            if (t.first < 0) t.first = i;
            t.last = std::max(t.last, i);
        }
        for (int tid : ops[i].reads) {
            auto& t = tensors[tid];
            if (t.first < 0) t.first = i;   // read before any write: an input filled outside the plan
            t.last = std::max(t.last, i);
        }
    }
    for (const Region& g : regions)
        for (auto& t : tensors)
            if (t.first >= 0 && t.first < g.end && t.last >= g.begin) {
                t.first = std::min(t.first, g.begin);
                t.last = std::max(t.last, g.end - 1);
            }
    for (auto& t : tensors)
        if (t.pinned || t.first < 0) { t.first = -1; t.last = nops; }

    std::vector<int> order(tensors.size());
    for (size_t i = 0; i < order.size(); ++i) order[i] = (int)i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return tensors[a].bytes > tensors[b].bytes; });
    struct Placed { size_t off, end; int first, last; };
    std::vector<Placed> placed;
    size_t total = 0;
    for (int id : order) {
        auto& t = tensors[id];
        const size_t size = (t.bytes + 255) & ~(size_t)255;
        std::vector<std::pair<size_t, size_t>> busy;
        for (auto& p : placed)
            if (!(p.last < t.first || t.last < p.first)) busy.push_back({p.off, p.end});
        std::sort(busy.begin(), busy.end());
        size_t off = 0;
        for (auto& b : busy) {
            if (off + size <= b.first) break;
            off = std::max(off, b.second);
        }
        t.offset = off;
        placed.push_back({off, off + size, t.first, t.last});
        total = std::max(total, off + size);
    }
    arena_bytes = std::max<size_t>(total, 256);
    return arena_bytes;
}

void Plan::run(const Ctx& ctx, cudaStream_t stream) const {
    const bool conc = ctx.side && ctx.fork && ctx.join;
    size_t r = 0;
    for (int i = 0; i < (int)ops.size(); ++i) {
        const OpRec& op = ops[i];
        const bool in_region = conc && r < regions.size() && i >= regions[r].begin && i < regions[r].end;
        if (in_region && i == regions[r].begin) {
            cuda_check(cudaEventRecord(ctx.fork, stream), "fork concurrent region");
            cuda_check(cudaStreamWaitEvent(ctx.side, ctx.fork, 0), "fork concurrent region");
        }
        cudaError_t e = op.fn(ctx, in_region && op.lane == 1 ? ctx.side : stream);
        if (e != cudaSuccess) fail(PPOCR_ERR_GPU, "launch " + op.name + ": " + cudaGetErrorString(e));
        if (in_region && i + 1 == regions[r].end) {
            cuda_check(cudaEventRecord(ctx.join, ctx.side), "join concurrent region");
            cuda_check(cudaStreamWaitEvent(stream, ctx.join, 0), "join concurrent region");
            ++r;
        }
    }
}

}  // namespace ppocr
