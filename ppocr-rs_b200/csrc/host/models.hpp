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
    int counter_slots = 0;            // per-model device counters (fused SE pool + MLP), zeroed at load
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

// Which contractions run on the tensor cores (tcgen05):
//   TC_NONE      every GEMM and conv on CUDA cores (FP32 exact FMA / BF16 SIMT);
//   TC_GEMMS     pointwise convs / linears on tcgen05: BF16 operands in BF16
//                mode, FP32 operands as three BF16 pieces in FP32 mode (split
//                GEMM); BF16 single-source convs as implicit tcgen05 GEMMs;
//   TC_ALL       as TC_GEMMS, plus the FP32 mode's dense convs through the
//                tensor-core engine (three-piece operands gathered per tap).
enum TcMode : int { TC_NONE = 0, TC_GEMMS = 1, TC_ALL = 2 };

// Validates, reads and packs the checkpoint, and builds the plan.  Errors
// follow gpu::Detector::load / gpu::Recognizer::load (src/gpu/model.rs:50-93, 156-220).
BuiltModel build_detector(const SafeTensors& st, int size, const size_t shape[4], DType dt, int tc_mode);
BuiltModel build_recognizer(const SafeTensors& st, int size, const size_t shape[4], DType dt, int tc_mode);

const char* size_name(int size);

}  // namespace ppocr
