// Weight access with the reference loader's semantics, the algebraic
// rewrites the reference CPU path applies at load time, and packers into the
// layouts the kernels read.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "safetensors.hpp"

namespace ppocr {

struct ConvWeight {
    std::vector<float> w;   // OIHW
    std::vector<float> b;   // [O] (zeros when the source has no bias)
    int cout = 0, cin = 0, kh = 0, kw = 0;   // cin = channels per group
};

class WeightReader {
public:
    explicit WeightReader(const SafeTensors& st) : st_(st) {}
    std::vector<float> get(const std::string& name, const std::vector<size_t>& shape) const { return st_.f32(name, shape); }
    // Conv2d::load (src/cpu/model.rs:87-106)
    ConvWeight conv(const std::string& prefix, int cout, int cin_per_group, int kh, int kw, bool bias) const;
    // Conv2d::load_bn: conv + BN folded (src/cpu/model.rs:108-133, 371-407)
    ConvWeight conv_bn(const std::string& prefix, int cout, int cin_per_group, int kh, int kw, bool bias,
                       const std::string& norm = "normalization") const;
    // Fold an already-read OI.. weight with the BN stored under `norm_prefix`.
    void fold_bn(ConvWeight& cw, const std::string& norm_prefix) const;
    // Linear: weight [out, in], bias [out] (src/cpu/model.rs:1681-1686)
    ConvWeight linear(const std::string& prefix, int in, int out) const;

private:
    const SafeTensors& st_;
};

// Rank-one split of a dense [O, I, k, k] kernel into depthwise [I][k*k] and
// pointwise [O][I] (power iteration, src/cpu/model.rs:221-369).  Throws
// InvalidModel when the kernel is not rank-one separable.
void factor_rank_one(const std::vector<float>& weight, int cin, int cout, int k, std::vector<float>& depthwise,
                     std::vector<float>& pointwise);

// Intraclass branch fusion (src/cpu/model.rs:811-888).
ConvWeight fuse_intraclass(const ConvWeight& sym, const ConvWeight& ver, const ConvWeight& hor);

// Transposed-conv BN fold over the output axis of IOHW (src/cpu/model.rs:1440-1477).
void fold_transpose_bn(std::vector<float>& w_iohw, std::vector<float>& b, int cin, int cout, const WeightReader& r,
                       const std::string& norm_prefix);

// Device weight image: FP32 and BF16 sections appended with 256-byte alignment.
class WeightBlob {
public:
    size_t add_f32(const std::vector<float>& v);
    size_t add_bf16(const std::vector<float>& v);   // round-to-nearest-even
    const std::vector<uint8_t>& bytes() const { return data_; }

private:
    std::vector<uint8_t> data_;
    size_t reserve(size_t bytes);
};

// Packers (all from OIHW / [out][in] sources)
std::vector<float> pack_conv_tiles(const ConvWeight& cw, int tile);       // [ceil(O/tile)][kh][kw][I][tile]
std::vector<float> pack_conv_kn(const ConvWeight& cw, int& n_pad);        // [kh][kw][I][O_pad4] (implicit GEMM)
std::vector<float> pack_conv_halo(const ConvWeight& cw, int bn);          // [ceil(I/4)][kh*kw][4][bn], zero padded
// Tensor-core engine weights: [planes][n_pad][k_pad] with k = (ky, kx, i); plane
// p holds the p-th BF16 piece of each value (planes 1: bf16(w); planes 3: the
// three-way split w = w0 + w1 + w2), every value exactly representable in BF16.
// cin_pad > cin: each tap takes cin_pad K columns, the last cin_pad - cin zero.
std::vector<float> pack_engine_kn(const ConvWeight& cw, int planes, int n_pad, int k_pad, int cin_pad = 0);
float bf16_round(float f);                                                // round to nearest even
// tcgen05 conv weights: [n_pad][kh][kw][cin_pad], channels past cin zero.
std::vector<float> pack_conv_tc(const ConvWeight& cw, int n_pad, int cin_pad);
std::vector<float> pack_depthwise(const ConvWeight& cw);                  // [kh*kw][C]
std::vector<float> pack_gemm_kn(const ConvWeight& cw, int& n_pad);        // [K][N_pad4]
std::vector<float> pack_gemm_nk(const ConvWeight& cw, int n_pad, int k_pad);  // [N_pad][K_pad] (BF16 source)
}  // namespace ppocr
