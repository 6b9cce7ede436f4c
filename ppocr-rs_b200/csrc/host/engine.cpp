// C ABI of the end-to-end pipeline: the host steps of pipeline.cpp and an
// OcrEngine (src/ocr.rs:364-540) over this library's models.
//
// The engine follows recognize_with (src/ocr.rs:573-621): the page is
// uploaded once; the detector runs on it with device preprocessing; the
// probability map comes back to the host for the DB postprocess; crops are
// ordered by aspect ratio and recognized six at a time on a canvas of the
// chunk's width, each chunk rectified on the device straight into the
// recognizer's input; only the per-step arg-max classes and probabilities
// come back for the CTC text assembly.  Models are cached per input shape,
// the recognizer's packed weights shared between shapes.
//
// The batch entry point gives every page the same result as the one-page
// call: a crop's recognizer output depends only on its own canvas width and
// pixels (every kernel treats batch entries independently and chooses its
// configuration from per-image shapes), so crops of all pages that share a
// canvas width run in shared batches, with unused slots zero-filled.
#include <algorithm>
#include <chrono>
#include <array>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <sstream>
#include <map>
#include <string>
#include <thread>
#include <vector>

#include "common.hpp"
#include "handles.hpp"
#include "pipeline.hpp"
#include "ppocr_b200.h"

using namespace ppocr;

struct ppocr_dictionary {
    std::vector<std::string> entries;
};

namespace {

void check(int status) {
    if (status != PPOCR_OK) fail(status, last_error());
}

PostOptions post_options(const ppocr_postprocess_options* o) {
    PostOptions p;
    if (o) {
        p.binary_threshold = o->binary_threshold;
        p.box_threshold = o->box_threshold;
        p.min_area = o->min_area;
        p.unclip_ratio = o->unclip_ratio;
        p.max_boxes = o->max_boxes;
    }
    return p;
}

void write_text(const Decoded& d, char* text, size_t capacity, size_t* length, float* score) {
    if (length) *length = d.text.size();
    if (score) *score = d.score;
    if (text) {
        if (capacity < d.text.size() + 1) fail(PPOCR_ERR_INVALID_INPUT, "text buffer is too small");
        std::memcpy(text, d.text.c_str(), d.text.size() + 1);
    }
}

std::string read_file(const char* path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) fail(PPOCR_ERR_READ_FILE, std::string("read recognition dictionary ") + path);
    std::ostringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

using Shape = std::array<size_t, 4>;

// Cached model shapes: a few detector page sizes and batch sizes, and one
// recognizer per (batch, canvas width) in use.  A page's text chunks span
// hundreds of canvas widths, each a model shape (plan, graph); the recognizer
// cache holds them all so repeated calls rebuild nothing (a cached shape keeps
// its plan and graph on the host and 8 bytes of flags on the device; the
// weights are shared).
constexpr size_t kDetectorCache = 4, kRecognizerCache = 1024;
constexpr size_t kDetectorBatch = 8;     // pages per detector forward
constexpr size_t kRecognizerBatch = 64;  // crops per recognizer forward
// Batch shapes for a width's remaining crops: the smallest that holds them.
constexpr size_t kTailBatches[] = {8, 16, 32};

struct ImageHandle {
    ppocr_image* p = nullptr;
    ImageHandle() = default;
    ImageHandle(const ImageHandle&) = delete;
    ImageHandle& operator=(const ImageHandle&) = delete;
    ImageHandle(ImageHandle&& o) noexcept : p(o.p) { o.p = nullptr; }
    ~ImageHandle() { ppocr_image_destroy(p); }
};


}  // namespace

struct ppocr_engine {
    ppocr_gpu* gpu = nullptr;
    bool owns_gpu_ref = false;   // the engine holds a reference on `gpu` (released by ppocr_engine_destroy)
    std::string det_path, rec_path;
    int det_size = PPOCR_TINY, rec_size = PPOCR_TINY;
    ppocr_load_options load{}, rec_load{};
    PostOptions post;
    uint32_t max_side = 736;
    std::vector<std::string> dict;
    size_t classes = 0;
    std::vector<std::pair<Shape, ppocr_model*>> det_cache, rec_cache;
    ppocr_model* rec_weights = nullptr;   // keeps the shared packed recognizer weights alive
    // Wall time of the last batch call per stage (ms): upload, detector,
    // DB postprocess, recognizer forwards (model loads included), assembly.
    double stage_ms[5] = {0, 0, 0, 0, 0};
    // Page staging reused across batch calls: device RGB buffers (grown, never
    // shrunk) and one pinned host buffer the pages are copied through, so a
    // call makes no allocation once the sizes have been seen (a cudaMalloc /
    // cudaFree pair per page per call stalled whole calls for up to a second).
    std::vector<ppocr_image*> page_pool;
    uint8_t* pinned = nullptr;
    size_t pinned_bytes = 0;
    // Page-locked staging of the recognition stage's greedy-CTC rows
    // (indices, then probabilities), grown as needed.
    uint8_t* ctc_host = nullptr;
    size_t ctc_bytes = 0;

    ~ppocr_engine() {
        for (auto& e : det_cache) ppocr_model_destroy(e.second);
        for (auto& e : rec_cache) ppocr_model_destroy(e.second);
        if (rec_weights) ppocr_model_destroy(rec_weights);
        for (ppocr_image* im : page_pool) ppocr_image_destroy(im);
        if (pinned) cudaFreeHost(pinned);
        if (ctc_host) cudaFreeHost(ctc_host);
    }


    ppocr_model* detector(const Shape& shape) {
        for (auto& e : det_cache)
            if (e.first == shape) return e.second;
        if (det_cache.size() == kDetectorCache) {
            ppocr_model_destroy(det_cache.front().second);
            det_cache.erase(det_cache.begin());
        }
        ppocr_model* m = nullptr;
        check(ppocr_detector_load_ex(gpu, det_path.c_str(), det_size, shape.data(), &load, &m));
        det_cache.emplace_back(shape, m);
        return m;
    }

    // The session of `shape` (loaded on first use).  A full cache drops its
    // oldest session that is not in `keep` (the sessions a pending batch uses).
    ppocr_model* recognizer(const Shape& shape, const std::vector<ppocr_model*>& keep = {}) {
        for (auto& e : rec_cache)
            if (e.first == shape) return e.second;
        if (rec_cache.size() >= kRecognizerCache) {
            for (auto it = rec_cache.begin(); it != rec_cache.end(); ++it)
                if (std::find(keep.begin(), keep.end(), it->second) == keep.end()) {
                    ppocr_model_destroy(it->second);
                    rec_cache.erase(it);
                    break;
                }
        }
        ppocr_model* m = nullptr;
        check(ppocr_recognizer_load_ex(gpu, rec_path.c_str(), rec_size, shape.data(), &rec_load, rec_weights, &m));
        if (!rec_weights) {
            // A second session on the same weights owns nothing but keeps them loaded.
            check(ppocr_recognizer_load_ex(gpu, rec_path.c_str(), rec_size, shape.data(), &rec_load, m, &rec_weights));
        }
        rec_cache.emplace_back(shape, m);
        return m;
    }

    struct Page {
        const uint8_t* rgb;
        size_t len;
        uint32_t width, height;
    };

    // Uploads the pages into the reused device buffers: one host copy into
    // pinned memory, one asynchronous copy per page, one stream wait.  The page
    // bytes are read inside `gate` only (null: no gate).
    void upload_pages(const std::vector<Page>& pages, CallGate* gate);

    std::vector<OcrResult> recognize_batch(const std::vector<Page>& pages, CallGate* gate = nullptr) {
        using clock = std::chrono::steady_clock;
        auto t_prev = clock::now();
        auto lap = [&](int stage) {
            const auto t = clock::now();
            stage_ms[stage] = std::chrono::duration<double, std::milli>(t - t_prev).count();
            t_prev = t;
        };
        const size_t np = pages.size();
        std::vector<OcrResult> res(np);
        for (size_t i = 0; i < np; ++i) {
            if (!pages[i].rgb) fail(PPOCR_ERR_INVALID_INPUT, "image pixels are null");
            res[i].source_w = pages[i].width;
            res[i].source_h = pages[i].height;
            detector_input_size(pages[i].width, pages[i].height, max_side, &res[i].input_w, &res[i].input_h);
        }
        upload_pages(pages, gate);
        struct PageRef {
            ppocr_image* p;
        };
        std::vector<PageRef> imgs(np);
        for (size_t i = 0; i < np; ++i) imgs[i].p = page_pool[i];
        lap(0);
        // Detector: pages of one input size, kDetectorBatch per forward.
        std::vector<std::vector<float>> probs(np);
        std::map<std::pair<uint32_t, uint32_t>, std::vector<size_t>> by_size;
        for (size_t i = 0; i < np; ++i) by_size[{res[i].input_h, res[i].input_w}].push_back(i);
        for (const auto& [hw, idx] : by_size) {
            for (size_t s = 0; s < idx.size(); s += kDetectorBatch) {
                const size_t n = std::min(kDetectorBatch, idx.size() - s);
                ppocr_model* det = detector(Shape{n, 3, hw.first, hw.second});
                std::vector<const ppocr_image*> batch(n);
                for (size_t k = 0; k < n; ++k) batch[k] = imgs[idx[s + k]].p;
                const size_t per = (size_t)hw.first * hw.second;
                std::vector<float> out(n * per);
                check(ppocr_detector_forward_images(det, batch.data(), n, out.data()));
                for (size_t k = 0; k < n; ++k) probs[idx[s + k]].assign(out.begin() + k * per, out.begin() + (k + 1) * per);
            }
        }
        lap(1);
        // DB postprocess on host threads.
        std::vector<std::vector<Detection>> dets(np);
        std::vector<std::string> errors(np);
        std::atomic<size_t> next{0};
        const size_t workers = std::max<size_t>(1, std::min<size_t>(np, std::thread::hardware_concurrency()));
        std::vector<std::thread> pool;
        for (size_t t = 0; t < workers; ++t)
            pool.emplace_back([&] {
                for (size_t i = next++; i < np; i = next++) {
                    try {
                        dets[i] = extract_detections(probs[i].data(), res[i].input_h, res[i].input_w, pages[i].width,
                                                     pages[i].height, res[i].input_w, res[i].input_h, post);
                    } catch (const std::exception& e) {
                        errors[i] = e.what();
                    }
                }
            });
        for (auto& t : pool) t.join();
        for (size_t i = 0; i < np; ++i)
            if (!errors[i].empty()) fail(PPOCR_ERR_INVALID_INPUT, errors[i]);
        lap(2);
        // Crops of every page, grouped by their chunk's canvas width.
        struct Crop {
            size_t page, det, content;
        };
        std::map<size_t, std::vector<Crop>> by_width;
        std::vector<std::vector<Decoded>> decoded(np);
        for (size_t i = 0; i < np; ++i) {
            decoded[i].resize(dets[i].size());
            for (const RecBatch& b : recognition_batches(dets[i]))
                for (size_t k = 0; k < b.index.size(); ++k) by_width[b.width].push_back(Crop{i, b.index[k], b.content[k]});
        }
        // One forward per (canvas width, up to kRecognizerBatch crops), all
        // enqueued back to back and waited for once; the greedy-CTC rows land
        // in the engine's page-locked staging.
        struct Forward {
            ppocr_model* rec;
            const std::vector<Crop>* crops;
            size_t first, n, width, steps, row0;
        };
        std::vector<Forward> forwards;
        std::vector<ppocr_model*> in_use;
        size_t total_rows = 0;
        for (const auto& [width, crops] : by_width) {
            for (size_t s = 0; s < crops.size(); s += kRecognizerBatch) {
                const size_t n = std::min(kRecognizerBatch, crops.size() - s);
                size_t shape_n = kRecognizerBatch;
                for (size_t b : kTailBatches)
                    if (n <= b) { shape_n = b; break; }
                ppocr_model* rec = recognizer(Shape{shape_n, 3, 48, width}, in_use);
                in_use.push_back(rec);
                size_t out_shape[4] = {0, 0, 0, 0};
                check(ppocr_model_output_shape(rec, out_shape, nullptr, nullptr));
                forwards.push_back(Forward{rec, &crops, s, n, width, out_shape[1], total_rows});
                total_rows += n * out_shape[1];
            }
        }
        if (total_rows * 8 > ctc_bytes) {
            std::lock_guard<std::mutex> lock(gpu->mu);
            gpu->bind();
            if (ctc_host) cudaFreeHost(ctc_host);
            ctc_host = nullptr;
            ctc_bytes = 0;
            cuda_check(cudaHostAlloc(reinterpret_cast<void**>(&ctc_host), total_rows * 8, cudaHostAllocPortable),
                       "allocate CTC staging");
            ctc_bytes = total_rows * 8;
        }
        int32_t* all_idx = reinterpret_cast<int32_t*>(ctc_host);
        float* all_prob = reinterpret_cast<float*>(ctc_host + total_rows * 4);
        CropBatch batch;
        for (const Forward& f : forwards) {
            std::vector<const ppocr_image*> ims(f.n);
            std::vector<float> corners(f.n * 8);
            std::vector<size_t> contents(f.n);
            for (size_t k = 0; k < f.n; ++k) {
                const Crop& c = (*f.crops)[f.first + k];
                ims[k] = imgs[c.page].p;
                contents[k] = c.content;
                for (int q = 0; q < 4; ++q) {
                    corners[k * 8 + 2 * q] = dets[c.page][c.det].poly[q].x;
                    corners[k * 8 + 2 * q + 1] = dets[c.page][c.det].poly[q].y;
                }
            }
            batch.add(f.rec, ims.data(), f.n, corners.data(), contents.data(), all_idx + f.row0, all_prob + f.row0);
        }
        batch.wait();
        for (const Forward& f : forwards)
            for (size_t k = 0; k < f.n; ++k) {
                const Crop& c = (*f.crops)[f.first + k];
                const size_t r = f.row0 + k * f.steps;
                decoded[c.page][c.det] = decode_ctc_steps(all_idx + r, all_prob + r, f.steps, classes, dict, c.content, f.width);
            }
        lap(3);
        for (size_t i = 0; i < np; ++i)
            for (size_t d = 0; d < dets[i].size(); ++d) {
                OcrLine l;
                std::copy(dets[i][d].poly, dets[i][d].poly + 4, l.poly);
                l.detection_score = dets[i][d].score;
                l.text = decoded[i][d].text;
                l.recognition_score = decoded[i][d].score;
                res[i].lines.push_back(std::move(l));
            }
        lap(4);
        return res;
    }

    OcrResult recognize(const uint8_t* rgb, size_t len, uint32_t width, uint32_t height) {
        if (!rgb) fail(PPOCR_ERR_INVALID_INPUT, "image pixels are null");
        OcrResult r;
        r.source_w = width;
        r.source_h = height;
        detector_input_size(width, height, max_side, &r.input_w, &r.input_h);
        ppocr_image* img = nullptr;
        check(ppocr_upload_rgb(gpu, width, height, rgb, len, &img));
        struct ImageGuard {
            ppocr_image* p;
            ~ImageGuard() { ppocr_image_destroy(p); }
        } guard_img{img};

        ppocr_model* det = detector(Shape{1, 3, r.input_h, r.input_w});
        std::vector<float> prob((size_t)r.input_h * r.input_w);
        const float full[8] = {0.f, 0.f, (float)width, 0.f, (float)width, (float)height, 0.f, (float)height};
        check(ppocr_model_forward_image(det, img, full, r.input_w, prob.data(), prob.size()));
        const std::vector<Detection> dets =
            extract_detections(prob.data(), r.input_h, r.input_w, width, height, r.input_w, r.input_h, post);

        std::vector<Decoded> decoded(dets.size());
        for (const RecBatch& b : recognition_batches(dets)) {
            const size_t n = b.index.size();
            ppocr_model* rec = recognizer(Shape{n, 3, 48, b.width});
            size_t out_shape[4] = {0, 0, 0, 0};
            check(ppocr_model_output_shape(rec, out_shape, nullptr, nullptr));
            const size_t steps = out_shape[1];
            std::vector<float> corners(n * 8);
            for (size_t k = 0; k < n; ++k)
                for (int c = 0; c < 4; ++c) {
                    corners[k * 8 + 2 * c] = dets[b.index[k]].poly[c].x;
                    corners[k * 8 + 2 * c + 1] = dets[b.index[k]].poly[c].y;
                }
            std::vector<int32_t> idx(n * steps);
            std::vector<float> p(n * steps);
            check(ppocr_recognizer_forward_crops(rec, img, n, corners.data(), b.content.data(), idx.data(), p.data(),
                                                 nullptr));
            for (size_t k = 0; k < n; ++k)
                decoded[b.index[k]] = decode_ctc_steps(idx.data() + k * steps, p.data() + k * steps, steps, classes, dict,
                                                       b.content[k], b.width);
        }
        for (size_t i = 0; i < dets.size(); ++i) {
            OcrLine l;
            std::copy(dets[i].poly, dets[i].poly + 4, l.poly);
            l.detection_score = dets[i].score;
            l.text = decoded[i].text;
            l.recognition_score = decoded[i].score;
            r.lines.push_back(std::move(l));
        }
        return r;
    }
};

namespace ppocr {

std::vector<std::string> engine_recognize(ppocr_engine* engine, size_t count, const uint8_t* const* rgb,
                                          const size_t* rgb_lengths, const uint32_t* widths, const uint32_t* heights,
                                          int format, CallGate* gate) {
    if (format != 0 && format != 1) fail(PPOCR_ERR_INVALID_INPUT, "format must be 0 (JSON) or 1 (text)");
    std::vector<ppocr_engine::Page> pages(count);
    for (size_t i = 0; i < count; ++i) pages[i] = ppocr_engine::Page{rgb[i], rgb_lengths[i], widths[i], heights[i]};
    const std::vector<OcrResult> r = engine->recognize_batch(pages, gate);
    std::vector<std::string> out(count);
    for (size_t i = 0; i < count; ++i) out[i] = format == 0 ? result_json(r[i]) : result_text(r[i]);
    return out;
}

}  // namespace ppocr

void ppocr_engine::upload_pages(const std::vector<Page>& pages, CallGate* gate) {
    size_t total = 0;
    for (const Page& pg : pages) {
        const size_t expected = (size_t)pg.width * pg.height * 3;
        // Gpu::upload_rgb checks (src/gpu/runtime.rs:175-197)
        if (pg.width == 0 || pg.height == 0) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: source image dimensions must be non-zero");
        if (pg.len != expected)
            fail(PPOCR_ERR_INVALID_INPUT, "invalid input: source image has " + std::to_string(pg.len) + " RGB bytes; expected " +
                                              std::to_string(expected) + " for " + std::to_string(pg.width) + "x" +
                                              std::to_string(pg.height));
        total += (expected + 255) & ~(size_t)255;
    }
    std::lock_guard<std::mutex> lock(gpu->mu);
    gpu->bind();
    if (total > pinned_bytes) {
        if (pinned) cudaFreeHost(pinned);
        pinned = nullptr;
        pinned_bytes = 0;
        cuda_check(cudaHostAlloc(reinterpret_cast<void**>(&pinned), total, cudaHostAllocPortable), "allocate page staging");
        pinned_bytes = total;
    }
    struct Lease {
        CallGate* g;
        ~Lease() {
            if (g) g->leave();
        }
    } lease{nullptr};
    if (gate) {
        if (!gate->enter()) fail(PPOCR_ERR_INVALID_INPUT, "invalid input: the call returned before its pages were read");
        lease.g = gate;
    }
    size_t off = 0;
    for (size_t i = 0; i < pages.size(); ++i) {
        const Page& pg = pages[i];
        if (i == page_pool.size()) page_pool.push_back(nullptr);
        ppocr_image*& im = page_pool[i];
        if (!im) {
            im = new ppocr_image();
            im->gpu = gpu;
            gpu_retain(gpu);
        }
        if (im->capacity < pg.len) {
            if (im->rgb) cudaFree(im->rgb);
            im->rgb = nullptr;
            im->capacity = 0;
            cuda_check(cudaMalloc(&im->rgb, pg.len), "allocate page buffer");
            im->capacity = pg.len;
        }
        im->width = pg.width;
        im->height = pg.height;
        std::memcpy(pinned + off, pg.rgb, pg.len);
        cuda_check(cudaMemcpyAsync(im->rgb, pinned + off, pg.len, cudaMemcpyHostToDevice, gpu->stream), "upload page");
        off += (pg.len + 255) & ~(size_t)255;
    }
    if (lease.g) {
        lease.g->leave();
        lease.g = nullptr;
    }
    // The pinned staging is rewritten by the next call: the copies land first.
    wait_stream(gpu->stream, 0, gpu);
}

extern "C" {

void ppocr_postprocess_options_default(ppocr_postprocess_options* o) {
    if (!o) return;
    const PostOptions d;
    o->binary_threshold = d.binary_threshold;
    o->box_threshold = d.box_threshold;
    o->min_area = d.min_area;
    o->unclip_ratio = d.unclip_ratio;
    o->max_boxes = d.max_boxes;
}

int ppocr_db_postprocess(const float* probabilities, size_t height, size_t width, uint32_t source_w, uint32_t source_h,
                         uint32_t content_w, uint32_t content_h, const ppocr_postprocess_options* options,
                         ppocr_detection* detections, size_t capacity, size_t* count) {
    return guard([&] {
        if (!probabilities) fail(PPOCR_ERR_INVALID_INPUT, "probability map is null");
        if (capacity && !detections) fail(PPOCR_ERR_INVALID_INPUT, "detection buffer is null");
        const std::vector<Detection> d =
            extract_detections(probabilities, height, width, source_w, source_h, content_w, content_h, post_options(options));
        if (count) *count = d.size();
        for (size_t i = 0; i < d.size() && i < capacity; ++i) {
            for (int c = 0; c < 4; ++c) {
                detections[i].polygon[2 * c] = d[i].poly[c].x;
                detections[i].polygon[2 * c + 1] = d[i].poly[c].y;
            }
            detections[i].score = d[i].score;
        }
    });
}

int ppocr_dictionary_parse(const char* contents, size_t length, ppocr_dictionary** out) {
    return guard([&] {
        if (!contents || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        auto d = std::make_unique<ppocr_dictionary>();
        d->entries = parse_dictionary(std::string(contents, length));
        *out = d.release();
    });
}

int ppocr_dictionary_load(const char* path, ppocr_dictionary** out) {
    return guard([&] {
        if (!path || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        auto d = std::make_unique<ppocr_dictionary>();
        d->entries = parse_dictionary(read_file(path));
        *out = d.release();
    });
}

int ppocr_dictionary_size(const ppocr_dictionary* dictionary, size_t* size) {
    return guard([&] {
        if (!dictionary || !size) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        *size = dictionary->entries.size();
    });
}

int ppocr_dictionary_entry(const ppocr_dictionary* dictionary, size_t index, char* text, size_t capacity, size_t* length) {
    return guard([&] {
        if (!dictionary) fail(PPOCR_ERR_INVALID_INPUT, "dictionary is null");
        if (index >= dictionary->entries.size()) fail(PPOCR_ERR_INVALID_INPUT, "dictionary index out of range");
        const std::string& e = dictionary->entries[index];
        if (length) *length = e.size();
        if (text && capacity > e.size()) std::memcpy(text, e.c_str(), e.size() + 1);
    });
}

void ppocr_dictionary_destroy(ppocr_dictionary* dictionary) { delete dictionary; }

int ppocr_ctc_decode(const ppocr_dictionary* dictionary, const float* probabilities, size_t steps, size_t classes,
                     size_t content_width, size_t input_width, char* text, size_t text_capacity, size_t* text_length,
                     float* score) {
    return guard([&] {
        if (!dictionary || !probabilities) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        write_text(decode_ctc_rows(probabilities, steps, classes, dictionary->entries, content_width, input_width), text,
                   text_capacity, text_length, score);
    });
}

int ppocr_ctc_decode_steps(const ppocr_dictionary* dictionary, const int32_t* indices, const float* probabilities,
                           size_t steps, size_t classes, size_t content_width, size_t input_width, char* text,
                           size_t text_capacity, size_t* text_length, float* score) {
    return guard([&] {
        if (!dictionary || !indices || !probabilities) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        write_text(decode_ctc_steps(indices, probabilities, steps, classes, dictionary->entries, content_width, input_width),
                   text, text_capacity, text_length, score);
    });
}

void ppocr_engine_options_default(ppocr_engine_options* o) {
    if (!o) return;
    std::memset(o, 0, sizeof(*o));
    o->detector_size = PPOCR_TINY;
    o->recognizer_size = PPOCR_TINY;
    o->precision = PPOCR_PRECISION_FP32;
    o->detector_max_side = 736;
    ppocr_postprocess_options_default(&o->postprocess);
}

int ppocr_engine_create(ppocr_gpu* gpu, const char* detector_model, const char* recognizer_model, const char* dictionary,
                        const ppocr_engine_options* options, ppocr_engine** out) {
    return guard([&] {
        if (!gpu || !detector_model || !recognizer_model || !dictionary || !out) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        ppocr_engine_options o;
        ppocr_engine_options_default(&o);
        if (options) o = *options;
        auto e = std::make_unique<ppocr_engine>();
        e->gpu = gpu;
        gpu_retain(gpu);
        e->owns_gpu_ref = true;
        e->det_path = detector_model;
        e->rec_path = recognizer_model;
        e->det_size = o.detector_size;
        e->rec_size = o.recognizer_size;
        e->post = post_options(&o.postprocess);
        e->post.validate();
        e->max_side = o.detector_max_side;
        ppocr_load_options_default(&e->load);
        e->load.precision = o.precision;
        e->rec_load = e->load;
        if (o.recognizer_precision) e->rec_load.precision = o.recognizer_precision - 1;
        if (e->rec_load.precision != PPOCR_PRECISION_FP32 && e->rec_load.precision != PPOCR_PRECISION_BF16 &&
            e->rec_load.precision != PPOCR_PRECISION_FP32_TC)
            fail(PPOCR_ERR_INVALID_INPUT, "unknown recognizer precision");
        e->dict = parse_dictionary(read_file(dictionary));
        // validate_recognizer_dictionary (src/ocr.rs:689-700), against the file's classifier.
        const size_t shape[4] = {1, 3, 48, 320};
        size_t out_shape[4] = {0, 0, 0, 0};
        check(ppocr_inspect_model(recognizer_model, 1, o.recognizer_size, shape, e->rec_load.precision, nullptr, nullptr,
                                  nullptr, out_shape));
        e->classes = out_shape[2];
        if (e->classes != e->dict.size() + 1 && e->classes != e->dict.size() + 2)
            fail(PPOCR_ERR_INVALID_INPUT, "recognizer has " + std::to_string(e->classes) +
                                              " output classes, but the dictionary has " + std::to_string(e->dict.size()) +
                                              " entries");
        *out = e.release();
    });
}

void ppocr_engine_destroy(ppocr_engine* engine) {
    if (!engine) return;
    ppocr_gpu* gpu = engine->owns_gpu_ref ? engine->gpu : nullptr;
    try {
        delete engine;
    } catch (...) {
    }
    if (gpu) gpu_release(gpu);
}

int ppocr_engine_recognize(ppocr_engine* engine, const uint8_t* rgb, size_t rgb_length, uint32_t width, uint32_t height,
                           int format, char** result, size_t* result_length) {
    return guard([&] {
        if (!engine || !result) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        if (format != 0 && format != 1) fail(PPOCR_ERR_INVALID_INPUT, "format must be 0 (JSON) or 1 (text)");
        const OcrResult r = engine->recognize(rgb, rgb_length, width, height);
        const std::string s = format == 0 ? result_json(r) : result_text(r);
        char* buf = static_cast<char*>(std::malloc(s.size() + 1));
        if (!buf) fail(PPOCR_ERR_GPU, "out of host memory");
        std::memcpy(buf, s.c_str(), s.size() + 1);
        *result = buf;
        if (result_length) *result_length = s.size();
    });
}

int ppocr_engine_stage_times(const ppocr_engine* engine, double* ms, size_t count) {
    return guard([&] {
        if (!engine || !ms) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        for (size_t i = 0; i < count && i < 5; ++i) ms[i] = engine->stage_ms[i];
    });
}

int ppocr_engine_recognize_batch(ppocr_engine* engine, size_t count, const uint8_t* const* rgb, const size_t* rgb_lengths,
                                 const uint32_t* widths, const uint32_t* heights, int format, char** results,
                                 size_t* result_lengths) {
    return guard([&] {
        if (!engine || !rgb || !rgb_lengths || !widths || !heights || !results) fail(PPOCR_ERR_INVALID_INPUT, "null argument");
        const std::vector<std::string> r = engine_recognize(engine, count, rgb, rgb_lengths, widths, heights, format, nullptr);
        std::vector<char*> out(count, nullptr);
        try {
            for (size_t i = 0; i < count; ++i) {
                const std::string& s = r[i];
                out[i] = static_cast<char*>(std::malloc(s.size() + 1));
                if (!out[i]) fail(PPOCR_ERR_GPU, "out of host memory");
                std::memcpy(out[i], s.c_str(), s.size() + 1);
                if (result_lengths) result_lengths[i] = s.size();
            }
        } catch (...) {
            for (char* p : out) std::free(p);
            throw;
        }
        for (size_t i = 0; i < count; ++i) results[i] = out[i];
    });
}

void ppocr_string_free(char* text) { std::free(text); }

}  // extern "C"
