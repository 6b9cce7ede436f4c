// Safetensors file reader.  Format: u64 little-endian header length, a JSON
// object {name: {"dtype", "shape", "data_offsets": [begin, end]}, "__metadata__": {...}},
// then the tensor bytes.  Error classes follow ppocr-rs src/gpu/weights.rs:28-155.
#include "safetensors.hpp"

#include <cstring>
#include <fstream>
#include <sstream>

#include "common.hpp"

namespace ppocr {
namespace {

// Minimal JSON reader: only what a safetensors header can hold.
struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
};

class Parser {
public:
    Parser(const char* s, size_t n) : s_(s), n_(n) {}
    Json parse() {
        Json v = value();
        ws();
        if (i_ != n_) bad("trailing characters after the header object");
        return v;
    }

private:
    const char* s_;
    size_t n_, i_ = 0;
    [[noreturn]] void bad(const std::string& why) {
        fail(PPOCR_ERR_SAFETENSORS, "decode safetensors: invalid header JSON (" + why + ")");
    }
    void ws() { while (i_ < n_ && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_; }
    char peek() { ws(); if (i_ >= n_) bad("unexpected end"); return s_[i_]; }
    void expect(char c) { if (peek() != c) bad(std::string("expected '") + c + "'"); ++i_; }
    Json value() {
        char c = peek();
        if (c == '{') return object();
        if (c == '[') return array();
        if (c == '"') { Json j; j.kind = Json::String; j.str = string(); return j; }
        if (c == 't' || c == 'f' || c == 'n') return literal();
        return number();
    }
    Json literal() {
        Json j;
        auto match = [&](const char* w) { size_t l = strlen(w); if (i_ + l <= n_ && !strncmp(s_ + i_, w, l)) { i_ += l; return true; } return false; };
        if (match("true")) { j.kind = Json::Bool; j.b = true; }
        else if (match("false")) { j.kind = Json::Bool; }
        else if (match("null")) { j.kind = Json::Null; }
        else bad("bad literal");
        return j;
    }
    Json number() {
        size_t st = i_;
        if (i_ < n_ && (s_[i_] == '-' || s_[i_] == '+')) ++i_;
        while (i_ < n_ && (isdigit((unsigned char)s_[i_]) || s_[i_] == '.' || s_[i_] == 'e' || s_[i_] == 'E' || s_[i_] == '-' || s_[i_] == '+')) ++i_;
        if (st == i_) bad("bad value");
        Json j;
        j.kind = Json::Number;
        j.num = std::stod(std::string(s_ + st, i_ - st));
        return j;
    }
    std::string string() {
        expect('"');
        std::string out;
        while (true) {
            if (i_ >= n_) bad("unterminated string");
            char c = s_[i_++];
            if (c == '"') break;
            if (c == '\\') {
                if (i_ >= n_) bad("bad escape");
                char e = s_[i_++];
                switch (e) {
                    case '"': out += '"'; break;
                    case '\\': out += '\\'; break;
                    case '/': out += '/'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u': {
                        if (i_ + 4 > n_) bad("bad unicode escape");
                        unsigned cp = std::stoul(std::string(s_ + i_, 4), nullptr, 16);
                        i_ += 4;
                        if (cp < 0x80) out += (char)cp;
                        else if (cp < 0x800) { out += (char)(0xC0 | (cp >> 6)); out += (char)(0x80 | (cp & 63)); }
                        else { out += (char)(0xE0 | (cp >> 12)); out += (char)(0x80 | ((cp >> 6) & 63)); out += (char)(0x80 | (cp & 63)); }
                        break;
                    }
                    default: bad("bad escape");
                }
            } else {
                out += c;
            }
        }
        return out;
    }
    Json array() {
        expect('[');
        Json j;
        j.kind = Json::Array;
        if (peek() == ']') { ++i_; return j; }
        while (true) {
            j.arr.push_back(value());
            char c = peek();
            ++i_;
            if (c == ']') break;
            if (c != ',') bad("expected ',' in array");
        }
        return j;
    }
    Json object() {
        expect('{');
        Json j;
        j.kind = Json::Object;
        if (peek() == '}') { ++i_; return j; }
        while (true) {
            std::string k = string();
            expect(':');
            j.obj.emplace_back(std::move(k), value());
            char c = peek();
            ++i_;
            if (c == '}') break;
            if (c != ',') bad("expected ',' in object");
        }
        return j;
    }
};

const Json* member(const Json& o, const char* key) {
    for (auto& kv : o.obj)
        if (kv.first == key) return &kv.second;
    return nullptr;
}

std::string shape_str(const std::vector<size_t>& s) {
    std::ostringstream o;
    o << "[";
    for (size_t i = 0; i < s.size(); ++i) o << (i ? ", " : "") << s[i];
    o << "]";
    return o.str();
}

}  // namespace

SafeTensors SafeTensors::load(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) fail(PPOCR_ERR_READ_FILE, "read weights " + path + ": " + std::strerror(errno));
    std::vector<uint8_t> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    if (f.bad()) fail(PPOCR_ERR_READ_FILE, "read weights " + path + ": I/O error");
    return from_bytes(std::move(bytes));
}

SafeTensors SafeTensors::from_bytes(std::vector<uint8_t> bytes) {
    SafeTensors st;
    if (bytes.size() < 8) fail(PPOCR_ERR_SAFETENSORS, "decode safetensors: header too small");
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | bytes[i];
    if (n > bytes.size() - 8 || n > (uint64_t)100 * 1024 * 1024)
        fail(PPOCR_ERR_SAFETENSORS, "decode safetensors: invalid header length");
    Json root = Parser(reinterpret_cast<const char*>(bytes.data() + 8), (size_t)n).parse();
    if (root.kind != Json::Object) fail(PPOCR_ERR_SAFETENSORS, "decode safetensors: header is not an object");
    const size_t data_start = 8 + (size_t)n;
    for (auto& kv : root.obj) {
        if (kv.first == "__metadata__") continue;
        const Json& t = kv.second;
        const Json* dt = member(t, "dtype");
        const Json* sh = member(t, "shape");
        const Json* off = member(t, "data_offsets");
        if (t.kind != Json::Object || !dt || dt->kind != Json::String || !sh || sh->kind != Json::Array || !off ||
            off->kind != Json::Array || off->arr.size() != 2)
            fail(PPOCR_ERR_SAFETENSORS, "decode safetensors: invalid tensor entry " + kv.first);
        TensorInfo info;
        info.dtype = dt->str;
        for (auto& d : sh->arr) {
            if (d.kind != Json::Number || d.num < 0) fail(PPOCR_ERR_SAFETENSORS, "decode safetensors: invalid shape of " + kv.first);
            info.shape.push_back((size_t)d.num);
        }
        if (off->arr[0].kind != Json::Number || off->arr[1].kind != Json::Number || off->arr[0].num < 0 || off->arr[1].num < 0)
            fail(PPOCR_ERR_SAFETENSORS, "decode safetensors: invalid data offsets of " + kv.first);
        const size_t b = (size_t)off->arr[0].num, e = (size_t)off->arr[1].num;
        info.begin = data_start + b;
        info.end = data_start + e;
        if (b > e || info.end > bytes.size()) {
            std::ostringstream o;
            o << "tensor \"" << kv.first << "\" byte range " << info.begin << ".." << info.end << " is outside a "
              << bytes.size() << "-byte file";
            fail(PPOCR_ERR_INVALID_TENSOR_RANGE, o.str());
        }
        st.tensors_[kv.first] = info;
    }
    st.bytes_ = std::move(bytes);
    return st;
}

const std::vector<size_t>& SafeTensors::shape(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) fail(PPOCR_ERR_TENSOR_NOT_FOUND, "tensor \"" + name + "\" was not found");
    return it->second.shape;
}

std::vector<float> SafeTensors::f32(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) fail(PPOCR_ERR_TENSOR_NOT_FOUND, "tensor \"" + name + "\" was not found");
    const TensorInfo& info = it->second;
    if (info.dtype != "F32")
        fail(PPOCR_ERR_UNSUPPORTED_DTYPE, "tensor \"" + name + "\" has dtype " + info.dtype + "; expected F32");
    size_t count = 1;
    for (size_t d : info.shape) {
        if (d != 0 && count > SIZE_MAX / 4 / d)
            fail(PPOCR_ERR_TENSOR_SIZE_OVERFLOW, "tensor \"" + name + "\" shape " + shape_str(info.shape) + " overflows the platform address space");
        count *= d;
    }
    const size_t expected = count * 4, found = info.end - info.begin;
    if (found != expected) {
        std::ostringstream o;
        o << "tensor \"" << name << "\" contains " << found << " bytes; expected " << expected << " bytes for F32";
        fail(PPOCR_ERR_TENSOR_BYTE_LENGTH, o.str());
    }
    std::vector<float> out(count);
    if (count) std::memcpy(out.data(), bytes_.data() + info.begin, expected);
    return out;
}

SafeTensors SafeTensors::recorder() {
    SafeTensors st;
    st.recording_ = true;
    return st;
}

std::vector<float> SafeTensors::f32(const std::string& name, const std::vector<size_t>& shape) const {
    if (recording_) {
        requested_[name] = shape;
        size_t count = 1;
        for (size_t d : shape) count *= d;
        return std::vector<float>(count, 1.f);
    }
    const std::vector<size_t>& found = this->shape(name);
    if (found != shape)
        fail(PPOCR_ERR_SHAPE_MISMATCH, "tensor \"" + name + "\" has shape " + shape_str(found) + "; expected " + shape_str(shape));
    return f32(name);
}

}  // namespace ppocr
