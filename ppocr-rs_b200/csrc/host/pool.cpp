// Multi-GPU OCR through the product API: one engine per device, each driven
// by its own host worker thread (its own ppocr_gpu, stream set, model cache
// and page staging), pages dealt round-robin across the devices and the
// results gathered in page order.  The pages of a worker that does not answer
// within the call's deadline are dealt again to the workers that did; the
// late worker sits out until its task returns.  No device-to-device traffic:
// every page's detector -> DB -> rectify -> recognizer -> CTC runs on one GPU.
// (The reference's OcrEngine drives one backend, src/ocr.rs:365-604.)
#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <functional>
#include <future>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.hpp"
#include "handles.hpp"
#include "ppocr_b200.h"

using namespace ppocr;

namespace ppocr {

// A worker: one host thread running the tasks queued to it, in order.
class Worker {
public:
    Worker() : thread_([this] { loop(); }) {}
    ~Worker() {
        {
            std::lock_guard<std::mutex> lock(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        thread_.join();
    }
    void submit(std::function<void()> task) {
        {
            std::lock_guard<std::mutex> lock(mu_);
            queue_.push_back(std::move(task));
        }
        cv_.notify_all();
    }

private:
    void loop() {
        while (true) {
            std::function<void()> task;
            {
                std::unique_lock<std::mutex> lock(mu_);
                cv_.wait(lock, [&] { return stop_ || !queue_.empty(); });
                if (queue_.empty()) return;
                task = std::move(queue_.front());
                queue_.pop_front();
            }
            task();
        }
    }
    std::mutex mu_;
    std::condition_variable cv_;
    std::deque<std::function<void()>> queue_;
    bool stop_ = false;
    std::thread thread_;
};

// Deals `items` round-robin over the workers, runs fn(worker, its items) on
// each worker's thread, and collects one result per item, in item order.
//  - A worker whose result is not in by `timeout_ms` (<= 0: no limit) is
//    late: its items are dealt again to the others, and it gets no work (in
//    this call or a later one) until its task has returned; that task's
//    results are dropped.
//  - A worker that fails with Error::Gpu is left out for the rest of the call
//    and its items are dealt again; any other error is the call's error.
//  - Error::Gpu when no worker is left.
template <typename R>
class ShardDispatcher {
public:
    using Run = std::function<std::vector<R>(size_t worker, const std::vector<size_t>& items)>;

    explicit ShardDispatcher(size_t workers) : busy_(workers) {
        for (size_t i = 0; i < workers; ++i) workers_.emplace_back(new Worker());
        for (auto& b : busy_) b = std::make_shared<std::atomic<bool>>(false);
    }

    std::vector<R> run(size_t items, const Run& fn, int timeout_ms, std::vector<int>* owner = nullptr) {
        std::vector<R> out(items);
        if (owner) owner->assign(items, -1);
        std::vector<size_t> pending(items);
        for (size_t i = 0; i < items; ++i) pending[i] = i;
        std::vector<bool> failed(workers_.size(), false);
        std::string last_gpu_error;
        while (!pending.empty()) {
            std::vector<size_t> ready;
            for (size_t w = 0; w < workers_.size(); ++w)
                if (!failed[w] && !*busy_[w]) ready.push_back(w);
            if (ready.empty())
                fail(PPOCR_ERR_GPU, last_gpu_error.empty() ? "GPU error: no device answered within the wait limit"
                                                           : last_gpu_error);
            std::vector<std::vector<size_t>> shard(ready.size());
            for (size_t k = 0; k < pending.size(); ++k) shard[k % ready.size()].push_back(pending[k]);
            struct Job {
                size_t worker;
                std::vector<size_t> items;
                std::future<std::vector<R>> result;
            };
            std::vector<Job> jobs;
            for (size_t s = 0; s < ready.size(); ++s) {
                if (shard[s].empty()) continue;
                const size_t w = ready[s];
                auto task = std::make_shared<std::packaged_task<std::vector<R>()>>(
                    [fn, w, its = shard[s], flag = busy_[w]]() {
                        struct Clear {
                            std::shared_ptr<std::atomic<bool>> f;
                            ~Clear() { *f = false; }
                        } clear{flag};
                        return fn(w, its);
                    });
                *busy_[w] = true;
                jobs.push_back(Job{w, shard[s], task->get_future()});
                workers_[w]->submit([task] { (*task)(); });
            }
            const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms > 0 ? timeout_ms : 0);
            pending.clear();
            for (Job& j : jobs) {
                if (timeout_ms > 0 && j.result.wait_until(deadline) != std::future_status::ready) {
                    pending.insert(pending.end(), j.items.begin(), j.items.end());
                    continue;
                }
                std::vector<R> r;
                try {
                    r = j.result.get();
                } catch (const Error& e) {
                    if (e.code != PPOCR_ERR_GPU) throw;
                    failed[j.worker] = true;
                    last_gpu_error = e.what();
                    pending.insert(pending.end(), j.items.begin(), j.items.end());
                    continue;
                }
                if (r.size() != j.items.size()) fail(PPOCR_ERR_GPU, "GPU error: a worker returned the wrong number of results");
                for (size_t k = 0; k < j.items.size(); ++k) {
                    out[j.items[k]] = std::move(r[k]);
                    if (owner) (*owner)[j.items[k]] = (int)j.worker;
                }
            }
            std::sort(pending.begin(), pending.end());
        }
        return out;
    }

    size_t size() const { return workers_.size(); }

private:
    std::vector<std::unique_ptr<Worker>> workers_;
    std::vector<std::shared_ptr<std::atomic<bool>>> busy_;
};

}  // namespace ppocr

struct ppocr_engine_pool {
    std::vector<ppocr_gpu*> gpus;
    std::vector<ppocr_engine*> engines;
    std::unique_ptr<ShardDispatcher<std::string>> dispatch;
    ~ppocr_engine_pool() {
        dispatch.reset();   // joins the worker threads (a late task finishes first)
        for (ppocr_engine* e : engines) ppocr_engine_destroy(e);
        for (ppocr_gpu* g : gpus) ppocr_gpu_destroy(g);
    }
};

extern "C" {

int ppocr_engine_pool_create(const int* devices, size_t count, const char* detector_model, const char* recognizer_model,
                             const char* dictionary, const ppocr_engine_options* options, ppocr_engine_pool** out) {
    return guard([&] {
        if (!devices || !out || count == 0) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: no devices");
        *out = nullptr;
        std::unique_ptr<ppocr_engine_pool> pool(new ppocr_engine_pool());
        for (size_t i = 0; i < count; ++i) {
            ppocr_gpu* g = nullptr;
            if (ppocr_gpu_create(devices[i], &g) != PPOCR_OK) fail(PPOCR_ERR_GPU, last_error());
            pool->gpus.push_back(g);
            ppocr_engine* e = nullptr;
            const int st = ppocr_engine_create(g, detector_model, recognizer_model, dictionary, options, &e);
            if (st != PPOCR_OK) fail(st, last_error());
            pool->engines.push_back(e);
        }
        pool->dispatch.reset(new ShardDispatcher<std::string>(count));
        *out = pool.release();
    });
}

void ppocr_engine_pool_destroy(ppocr_engine_pool* pool) {
    try {
        delete pool;
    } catch (...) {
    }
}

int ppocr_engine_pool_size(const ppocr_engine_pool* pool, size_t* count) {
    return guard([&] {
        if (!pool || !count) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        *count = pool->engines.size();
    });
}

int ppocr_engine_pool_recognize_batch(ppocr_engine_pool* pool, size_t count, const uint8_t* const* rgb,
                                      const size_t* rgb_lengths, const uint32_t* widths, const uint32_t* heights,
                                      int format, int timeout_ms, char** results, size_t* result_lengths,
                                      int* devices_used) {
    return guard([&] {
        if (!pool || !rgb || !rgb_lengths || !widths || !heights || !results) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (format != 0 && format != 1) fail(PPOCR_ERR_INVALID_INPUT, "format must be 0 (JSON) or 1 (text)");
        for (size_t i = 0; i < count; ++i) results[i] = nullptr;
        // A late worker may still be running when this call returns: it reads
        // the caller's arrays and pages only inside the gate, which closes
        // before the call returns.
        auto gate = std::make_shared<CallGate>();
        struct Close {
            std::shared_ptr<CallGate> g;
            ~Close() { g->close(); }
        } close{gate};
        auto fn = [pool, gate, rgb, rgb_lengths, widths, heights, format](size_t w, const std::vector<size_t>& items) {
            std::vector<const uint8_t*> r(items.size());
            std::vector<size_t> l(items.size());
            std::vector<uint32_t> ww(items.size()), hh(items.size());
            if (!gate->enter()) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: the call returned before its pages were read");
            for (size_t k = 0; k < items.size(); ++k) {
                r[k] = rgb[items[k]];
                l[k] = rgb_lengths[items[k]];
                ww[k] = widths[items[k]];
                hh[k] = heights[items[k]];
            }
            gate->leave();
            return engine_recognize(pool->engines[w], items.size(), r.data(), l.data(), ww.data(), hh.data(), format,
                                    gate.get());
        };
        std::vector<int> owner;
        std::vector<std::string> text = pool->dispatch->run(count, fn, timeout_ms, &owner);
        for (size_t i = 0; i < count; ++i) {
            char* s = static_cast<char*>(std::malloc(text[i].size() + 1));
            if (!s) {
                for (size_t k = 0; k < i; ++k) ppocr_string_free(results[k]);
                fail(PPOCR_ERR_GPU, "out of host memory");
            }
            std::memcpy(s, text[i].data(), text[i].size());
            s[text[i].size()] = 0;
            results[i] = s;
            if (result_lengths) result_lengths[i] = text[i].size();
            if (devices_used) devices_used[i] = pool->gpus[owner[i]]->device;
        }
    });
}

int ppocr_selftest_dispatch(size_t workers, size_t items, uint32_t stall_mask, uint32_t fail_mask, int stall_ms,
                            int timeout_ms, int* owner, int* values) {
    return guard([&] {
        if (workers == 0 || workers > 32 || !owner || !values) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: dispatch test arguments");
        ShardDispatcher<int> d(workers);
        auto fn = [stall_mask, fail_mask, stall_ms](size_t w, const std::vector<size_t>& its) {
            // A fake device: a stalling worker answers after stall_ms, a failing
            // one raises a device error; the others answer item * 10.
            if (fail_mask >> w & 1) fail(PPOCR_ERR_GPU, "GPU error: fake device " + std::to_string(w) + " failed");
            std::this_thread::sleep_for(std::chrono::milliseconds((stall_mask >> w & 1) ? stall_ms : 2));
            std::vector<int> r(its.size());
            for (size_t k = 0; k < its.size(); ++k) r[k] = (int)its[k] * 10;
            return r;
        };
        std::vector<int> own;
        const std::vector<int> v = d.run(items, fn, timeout_ms, &own);
        for (size_t i = 0; i < items; ++i) {
            owner[i] = own[i];
            values[i] = v[i];
        }
    });
}

}  // extern "C"
