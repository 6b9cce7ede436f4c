// Detector / recognizer graph construction for the B200 kernels.
#pragma once

#include <memory>
#include <string>
#include <vector>

#include "graph.hpp"
#include "ppocr_b200.h"
#include "weights.hpp"

namespace ppocr {

enum class Kind { Detector, Recognizer };

struct BuiltModel {
    Kind kind = Kind::Detector;
    int size = PPOCR_TINY;
    DType dtype = DT_F32;
    Plan plan;
    WeightBlob blob;
    int n = 0, h = 0, w = 0;          // input NCHW [n, 3, h, w]
    int input = -1;                   // FP32 NCHW input tensor
    // detector
    int prob = -1, mask = -1;         // FP32 [n, h, w]; u8 [n, h, w]
    // recognizer
    int probs = -1;                   // FP32 [n, t, classes]
    int logits = -1;                  // FP32 [n, t, logits_ld]: rows padded to 16 bytes
    int logits_ld = 0;
    int index = -1, max_prob = -1, margin = -1;   // [n, t]
    int t = 0, classes = 0;
    std::shared_ptr<float> mask_threshold = std::make_shared<float>(0.2f);   // DB binarisation threshold
    std::vector<size_t> output_shape;
    size_t output_elements = 0;
    int tensor_count = 0;             // tensors in the source file
};

// Validates, reads and packs the checkpoint, and builds the plan.  Errors
// follow gpu::Detector::load / gpu::Recognizer::load (src/gpu/model.rs:50-93, 156-220).
BuiltModel build_detector(const SafeTensors& st, int size, const size_t shape[4], DType dt, bool tensor_cores);
BuiltModel build_recognizer(const SafeTensors& st, int size, const size_t shape[4], DType dt, bool tensor_cores);

const char* size_name(int size);

}  // namespace ppocr
