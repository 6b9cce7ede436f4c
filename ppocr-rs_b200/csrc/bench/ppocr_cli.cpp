// ppocr: end-to-end OCR of one image (the reference's `ppocr` binary,
// ppocr-rs src/bin/ppocr.rs:12-133) over the C ABI's engine.
//
// Same options and defaults (--model-size, --detector-model,
// --recognizer-model, --dictionary, --detector-max-side, the postprocess
// thresholds, --format json|text, --output).  Only the GPU backend exists in
// this build; models are given as files (there is no model store or
// network).  Images are decoded here: PNG (8/16-bit gray, gray+alpha, RGB,
// RGBA and palette, non-interlaced; zlib inflate) and binary PPM/PGM.
// Alpha is dropped, as converting to RGB8 does in the reference.
#include <zlib.h>

#include <cctype>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "ppocr_b200.h"

namespace {

[[noreturn]] void die(const std::string& m) {
    std::fprintf(stderr, "Error: %s\n", m.c_str());
    std::exit(1);
}

void check(int status, const char* what) {
    if (status != PPOCR_OK) die(std::string(what) + ": " + ppocr_last_error());
}

std::vector<uint8_t> read_all(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) die("read image " + path);
    return std::vector<uint8_t>(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
}

struct Image {
    uint32_t width = 0, height = 0;
    std::vector<uint8_t> rgb;
};

uint32_t be32(const uint8_t* p) { return (uint32_t)p[0] << 24 | (uint32_t)p[1] << 16 | (uint32_t)p[2] << 8 | p[3]; }

uint8_t paeth(int a, int b, int c) {
    const int p = a + b - c, pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
    return (uint8_t)((pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c));
}

Image decode_png(const std::vector<uint8_t>& d) {
    static const uint8_t sig[8] = {0x89, 'P', 'N', 'G', 0x0d, 0x0a, 0x1a, 0x0a};
    if (d.size() < 8 || std::memcmp(d.data(), sig, 8) != 0) die("not a PNG file");
    Image img;
    int depth = 0, color = 0, interlace = 0;
    std::vector<uint8_t> idat, palette;
    size_t pos = 8;
    while (pos + 12 <= d.size()) {
        const uint32_t len = be32(&d[pos]);
        const std::string type(reinterpret_cast<const char*>(&d[pos + 4]), 4);
        if (pos + 12 + (size_t)len > d.size()) die("truncated PNG chunk " + type);
        const uint8_t* body = &d[pos + 8];
        if (type == "IHDR") {
            if (len < 13) die("bad PNG header");
            img.width = be32(body);
            img.height = be32(body + 4);
            depth = body[8];
            color = body[9];
            interlace = body[12];
        } else if (type == "PLTE") {
            palette.assign(body, body + len);
        } else if (type == "IDAT") {
            idat.insert(idat.end(), body, body + len);
        } else if (type == "IEND") {
            break;
        }
        pos += 12 + (size_t)len;
    }
    if (img.width == 0 || img.height == 0) die("PNG has no image");
    if (interlace != 0) die("interlaced PNG is not supported; re-save without interlacing");
    int channels = 0;
    switch (color) {
        case 0: channels = 1; break;
        case 2: channels = 3; break;
        case 3: channels = 1; break;
        case 4: channels = 2; break;
        case 6: channels = 4; break;
        default: die("unsupported PNG color type");
    }
    if (!(depth == 8 || depth == 16) || (color == 3 && depth != 8)) die("unsupported PNG bit depth");
    const size_t bpp = (size_t)channels * (depth / 8);
    const size_t stride = (size_t)img.width * bpp;
    std::vector<uint8_t> raw((stride + 1) * img.height);
    z_stream zs{};
    if (inflateInit(&zs) != Z_OK) die("zlib init");
    zs.next_in = idat.data();
    zs.avail_in = (uInt)idat.size();
    zs.next_out = raw.data();
    zs.avail_out = (uInt)raw.size();
    const int zr = inflate(&zs, Z_FINISH);
    inflateEnd(&zs);
    if (zr != Z_STREAM_END || zs.total_out != raw.size()) die("corrupt PNG image data");
    std::vector<uint8_t> px(stride * img.height);
    for (uint32_t y = 0; y < img.height; ++y) {
        const uint8_t filter = raw[y * (stride + 1)];
        const uint8_t* in = &raw[y * (stride + 1) + 1];
        uint8_t* out = &px[y * stride];
        const uint8_t* up = y ? &px[(y - 1) * stride] : nullptr;
        for (size_t x = 0; x < stride; ++x) {
            const int a = x >= bpp ? out[x - bpp] : 0, b = up ? up[x] : 0, c = (up && x >= bpp) ? up[x - bpp] : 0;
            int v = in[x];
            switch (filter) {
                case 0: break;
                case 1: v += a; break;
                case 2: v += b; break;
                case 3: v += (a + b) / 2; break;
                case 4: v += paeth(a, b, c); break;
                default: die("bad PNG filter");
            }
            out[x] = (uint8_t)v;
        }
    }
    img.rgb.resize((size_t)img.width * img.height * 3);
    const size_t step = depth / 8;   // 16-bit samples: keep the high byte
    for (size_t i = 0; i < (size_t)img.width * img.height; ++i) {
        const uint8_t* s = &px[i * bpp];
        uint8_t r, g, b;
        if (color == 3) {
            const size_t k = (size_t)s[0] * 3;
            if (k + 2 >= palette.size()) die("PNG palette index out of range");
            r = palette[k]; g = palette[k + 1]; b = palette[k + 2];
        } else if (channels <= 2) {
            r = g = b = s[0];
        } else {
            r = s[0]; g = s[step]; b = s[2 * step];
        }
        img.rgb[i * 3] = r; img.rgb[i * 3 + 1] = g; img.rgb[i * 3 + 2] = b;
    }
    return img;
}

Image decode_pnm(const std::vector<uint8_t>& d) {
    std::string s(d.begin(), d.end());
    size_t p = 0;
    auto token = [&]() {
        while (p < s.size()) {
            if (std::isspace((unsigned char)s[p])) ++p;
            else if (s[p] == '#') { while (p < s.size() && s[p] != '\n') ++p; }
            else break;
        }
        const size_t b = p;
        while (p < s.size() && !std::isspace((unsigned char)s[p])) ++p;
        return s.substr(b, p - b);
    };
    const std::string magic = token();
    if (magic != "P6" && magic != "P5") die("unsupported PNM type (P5 / P6 only)");
    Image img;
    img.width = (uint32_t)std::stoul(token());
    img.height = (uint32_t)std::stoul(token());
    const unsigned long maxval = std::stoul(token());
    if (maxval != 255) die("PNM maxval must be 255");
    ++p;   // the single whitespace after the header
    const size_t ch = magic == "P6" ? 3 : 1, n = (size_t)img.width * img.height;
    if (p + n * ch > d.size()) die("truncated PNM image");
    img.rgb.resize(n * 3);
    for (size_t i = 0; i < n; ++i)
        for (int c = 0; c < 3; ++c) img.rgb[i * 3 + c] = d[p + i * ch + (ch == 3 ? c : 0)];
    return img;
}

Image decode(const std::string& path) {
    const std::vector<uint8_t> d = read_all(path);
    if (d.size() >= 8 && d[0] == 0x89 && d[1] == 'P') return decode_png(d);
    if (d.size() >= 2 && d[0] == 'P' && (d[1] == '6' || d[1] == '5')) return decode_pnm(d);
    if (d.size() >= 3 && d[0] == 0xff && d[1] == 0xd8) die("JPEG decoding is not part of this build; convert the image to PNG");
    die("unrecognised image format (PNG or binary PPM/PGM expected)");
}

int size_code(const std::string& s) {
    if (s == "tiny") return PPOCR_TINY;
    if (s == "small") return PPOCR_SMALL;
    if (s == "medium") return PPOCR_MEDIUM;
    die("unknown model size " + s);
}

void usage() {
    std::printf(
        "usage: ppocr IMAGE --detector-model FILE --recognizer-model FILE [--dictionary FILE] [--backend gpu]\n"
        "             [--model-size tiny|small|medium] [--detector-max-side 736] [--binary-threshold 0.2]\n"
        "             [--box-threshold 0.4] [--min-area 3] [--unclip-ratio 1.4] [--max-boxes 1000]\n"
        "             [--format json|text] [--output FILE] [--device 0] [--precision fp32|bf16]\n");
}

}  // namespace

int main(int argc, char** argv) {
    std::string image, det, rec, dict, format = "json", output, backend = "gpu", size = "tiny", precision = "fp32";
    ppocr_engine_options o;
    ppocr_engine_options_default(&o);
    int device = 0;
    for (int i = 1; i < argc; ++i) {
        const std::string k = argv[i];
        auto val = [&]() -> std::string {
            if (i + 1 >= argc) die("missing value for " + k);
            return argv[++i];
        };
        if (k == "-h" || k == "--help") { usage(); return 0; }
        else if (k == "--backend") backend = val();
        else if (k == "--model-size") size = val();
        else if (k == "--model-dir") val();
        else if (k == "--offline") {}
        else if (k == "--detector-model") det = val();
        else if (k == "--recognizer-model") rec = val();
        else if (k == "--dictionary") dict = val();
        else if (k == "--threads") val();   // CPU backend option; the GPU backend does not use it
        else if (k == "--detector-max-side") o.detector_max_side = (uint32_t)std::stoul(val());
        else if (k == "--binary-threshold") o.postprocess.binary_threshold = std::stof(val());
        else if (k == "--box-threshold") o.postprocess.box_threshold = std::stof(val());
        else if (k == "--min-area") o.postprocess.min_area = std::stoul(val());
        else if (k == "--unclip-ratio") o.postprocess.unclip_ratio = std::stof(val());
        else if (k == "--max-boxes") o.postprocess.max_boxes = std::stoul(val());
        else if (k == "--format") format = val();
        else if (k == "--output") output = val();
        else if (k == "--device") device = std::stoi(val());
        else if (k == "--precision") precision = val();
        else if (!k.empty() && k[0] == '-') die("unknown option " + k);
        else if (image.empty()) image = k;
        else die("unexpected argument " + k);
    }
    if (image.empty()) { usage(); return 2; }
    if (backend != "gpu") die("only the GPU backend is part of this build (--backend gpu)");
    if (format != "json" && format != "text") die("--format must be json or text");
    if (det.empty() || rec.empty()) die("--detector-model and --recognizer-model are required (no model store in this build)");
    if (dict.empty()) {
        const size_t slash = rec.find_last_of('/');
        dict = (slash == std::string::npos ? std::string(".") : rec.substr(0, slash)) + "/inference.yml";
    }
    o.detector_size = o.recognizer_size = size_code(size);
    o.precision = precision == "bf16" ? PPOCR_PRECISION_BF16 : PPOCR_PRECISION_FP32;
    if (o.detector_max_side == 0) die("detector maximum side must be positive");

    const Image img = decode(image);
    ppocr_gpu* gpu = nullptr;
    check(ppocr_gpu_create(device, &gpu), "initialize GPU backend");
    ppocr_engine* engine = nullptr;
    check(ppocr_engine_create(gpu, det.c_str(), rec.c_str(), dict.c_str(), &o, &engine), "load OCR engine");
    char* result = nullptr;
    size_t len = 0;
    check(ppocr_engine_recognize(engine, img.rgb.data(), img.rgb.size(), img.width, img.height, format == "json" ? 0 : 1,
                                 &result, &len),
          "run OCR");
    if (!output.empty()) {
        std::ofstream f(output, std::ios::binary);
        if (!f) die("write OCR result " + output);
        f.write(result, (std::streamsize)len);
    } else {
        std::fwrite(result, 1, len, stdout);
        std::fputc('\n', stdout);
    }
    ppocr_string_free(result);
    ppocr_engine_destroy(engine);
    ppocr_gpu_destroy(gpu);
    return 0;
}
