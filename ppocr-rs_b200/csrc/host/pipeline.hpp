// Host-side steps of the end-to-end pipeline around the two models
// (ppocr-rs src/ocr.rs): DB postprocess of the probability map, recognition
// planning, dictionary parsing, greedy-CTC text assembly and the JSON result.
//
// Geometry is computed in f32 with every operation rounded in the
// reference's order (the library is built with -ffp-contract=off), so boxes
// and scores come out bit-identical to the reference's for the same map.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ppocr {

struct Pt {
    float x = 0.f, y = 0.f;
};

struct Detection {
    Pt poly[4];
    float score = 0.f;
};

// DetectorPostprocessOptions (src/ocr.rs:231-271).
struct PostOptions {
    float binary_threshold = 0.2f;
    float box_threshold = 0.4f;
    size_t min_area = 3;
    float unclip_ratio = 1.4f;
    size_t max_boxes = 1000;
    void validate() const;   // Error(INVALID_INPUT) on a bad option
};

// extract_detections (src/ocr.rs:723-782) over a [height, width] map whose
// content area is content_w x content_h of a source_w x source_h image.
std::vector<Detection> extract_detections(const float* values, size_t height, size_t width, uint32_t source_w,
                                          uint32_t source_h, uint32_t content_w, uint32_t content_h,
                                          const PostOptions& opts);

// DetectorInputPlan::new (src/ocr.rs:86-101): detector input (width, height);
// max_side == 0 selects the released model's resize policy.
void detector_input_size(uint32_t width, uint32_t height, uint32_t max_side, uint32_t* in_w, uint32_t* in_h);

// Recognition planning (src/ocr.rs:154-219, 1128-1156).
float polygon_aspect_ratio(const Pt (&poly)[4]);
size_t crop_content_width(const Pt (&poly)[4]);
size_t recognizer_batch_width(const std::vector<const Pt*>& polys);

// One chunk of recognize_with (src/ocr.rs:573-621): detection indices in
// aspect-ratio order, the canvas width and each crop's content width.
struct RecBatch {
    std::vector<size_t> index;
    size_t width = 0;
    std::vector<size_t> content;
};
std::vector<RecBatch> recognition_batches(const std::vector<Detection>& dets);

// parse_dictionary (src/ocr.rs:892-965): PaddleX `character_dict:` list or one
// entry per line; Error(INVALID_INPUT) on an empty dictionary or entry.
std::vector<std::string> parse_dictionary(const std::string& contents);

struct Decoded {
    std::string text;
    float score = 0.f;
};

// decode_ctc_greedy_for_input (src/ocr.rs:800-853) from full probability rows.
Decoded decode_ctc_rows(const float* probs, size_t steps, size_t classes, const std::vector<std::string>& dict,
                        size_t content_width, size_t input_width);
// The same from per-step arg-max classes and their probabilities (the device's
// softmax statistics; rows of a softmax sum to one, so row_probability is the
// clamped maximum).
Decoded decode_ctc_steps(const int32_t* index, const float* prob, size_t steps, size_t classes,
                         const std::vector<std::string>& dict, size_t content_width, size_t input_width);

// join_decoded_texts (src/ocr.rs:702-721).
Decoded join_decoded_texts(const std::vector<Decoded>& parts);

struct OcrLine {
    Pt poly[4];
    float detection_score = 0.f;
    std::string text;
    float recognition_score = 0.f;
};

struct OcrResult {
    uint32_t source_w = 0, source_h = 0;
    uint32_t input_w = 0, input_h = 0;
    std::vector<OcrLine> lines;
};

// The reference's serialised OcrResult (pretty JSON) and its text() form.
std::string result_json(const OcrResult& r);
std::string result_text(const OcrResult& r);

}  // namespace ppocr
