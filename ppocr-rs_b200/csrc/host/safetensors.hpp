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

private:
    std::vector<uint8_t> bytes_;
    std::map<std::string, TensorInfo> tensors_;
};

}  // namespace ppocr
