// Safetensors reader with the reference's checks (ppocr-rs src/gpu/weights.rs:28-155):
// the file is read once, the JSON header indexed, and every tensor access
// checks dtype (F32 only), element count and byte range.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace ppocr {

struct TensorInfo {
    std::string dtype;
    std::vector<size_t> shape;
    size_t begin = 0, end = 0;   // absolute byte offsets in the file
};

class SafeTensors {
public:
    static SafeTensors load(const std::string& path);            // Error::ReadFile / Error::Safetensors
    static SafeTensors from_bytes(std::vector<uint8_t> bytes);    // Error::Safetensors / InvalidTensorRange

    size_t size() const { return tensors_.size(); }
    bool contains(const std::string& name) const { return tensors_.count(name) != 0; }
    const std::map<std::string, TensorInfo>& tensors() const { return tensors_; }

    // Little-endian F32 values of `name`; TensorNotFound, UnsupportedDtype,
    // TensorSizeOverflow, TensorByteLength, InvalidTensorRange.
    std::vector<float> f32(const std::string& name) const;
    // As f32() plus a shape check (ShapeMismatch).
    std::vector<float> f32(const std::string& name, const std::vector<size_t>& shape) const;
    const std::vector<size_t>& shape(const std::string& name) const;

    // A recorder holds no file: every f32(name, shape) request succeeds with
    // values of 1 and is remembered, so running a model builder against it
    // lists the tensors (names and shapes) of that model's checkpoint.
    static SafeTensors recorder();
    bool recording() const { return recording_; }
    const std::map<std::string, std::vector<size_t>>& requested() const { return requested_; }

private:
    std::vector<uint8_t> bytes_;
    std::map<std::string, TensorInfo> tensors_;
    bool recording_ = false;
    mutable std::map<std::string, std::vector<size_t>> requested_;
};

// Writes a checkpoint of random-init weights for the detector (detector =
// true) or recognizer of tier `size` in the reference's tensor layout, drawn
// from the benchmark configs' distributions: detector conv weights
// N(0, sqrt(2 / fan_in)), recognizer conv / linear weights N(0, 0.02), batch
// norm gamma 1, beta 0, mean 0, var 1, layer norm weight 1 and bias 0, every
// bias 0, and the medium detector's 9x9 neck kernels in the rank-one form
// p[o, i] d[i, :] (|d[i]| = 1) its factorisation accepts.  Each tensor draws
// from its own generator seeded by (seed, crc32(name)).
void write_seeded_weights(const std::string& path, bool detector, int size, uint64_t seed);

}  // namespace ppocr
