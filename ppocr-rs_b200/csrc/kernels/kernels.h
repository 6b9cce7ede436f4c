// Launch interface of the sm_100a kernels.  Plain structs of device pointers
// and sizes; every launcher enqueues on `stream` and returns the launch error.
//
// Tensor layout: NHWC, channels contiguous, `cstride` elements between pixels
// and `coff` the first channel of the view (concatenation is a channel offset
// into a wider buffer).  DType selects the storage type of activations.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace ppocr {

enum DType : int { DT_F32 = 0, DT_BF16 = 1 };

// Fused activations (src/cpu/kernels/mod.rs:2365-2403).
enum Act : int {
    ACT_NONE = 0,
    ACT_RELU = 1,
    ACT_SILU = 2,
    ACT_GELU = 3,      // 0.5 x (1 + erf(x / sqrt 2)), erf by Abramowitz-Stegun 7.1.26
    ACT_HSWISH = 4,    // x * clamp(x / 6 + 0.5, 0, 1)
    ACT_SIGMOID = 5,
};

inline size_t dtype_size(DType t) { return t == DT_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------
// Direct convolution (groups = 1): stems, 3x3 / 2x2 / k x k convs, detector
// head conv_down.  The input is a virtual concatenation of up to four
// sources, each read with nearest-neighbour upsampling by `scale` and
// optionally through a 2x2 stride-1 "same-upper" max pool (the stem's pool
// branch, src/cpu/ops.rs:1520-1535), so neither the concat nor the upsample
// nor the pool is materialised.
// ---------------------------------------------------------------------------
enum SourceMode : int { SRC_NHWC = 0, SRC_NHWC_MAXPOOL = 1, SRC_NCHW_F32 = 2 };

struct ConvSource {
    const void* ptr = nullptr;
    int channels = 0;   // channels this source contributes (multiple of 4 for NHWC)
    int cstride = 0;    // pixel stride of the source buffer in elements
    int coff = 0;       // first channel of the view
    int scale = 1;      // nearest-neighbour upsampling factor
    int mode = SRC_NHWC;
};

struct ConvParams {
    int n = 0, hi = 0, wi = 0, cin = 0;   // logical input (after upsampling)
    ConvSource src[4];
    int nsrc = 0;
    int ho = 0, wo = 0, cout = 0;
    int kh = 0, kw = 0, sh = 1, sw = 1, pt = 0, pl = 0;
    int co_tile = 8;                      // output channels per thread: 8, 16, 32 or 64
    const float* weight = nullptr;        // [ceil(cout/co_tile)][kh][kw][cin][co_tile]
    const float* weight_kn = nullptr;     // implicit-GEMM layout [kh][kw][cin][n_pad] (or null)
    int n_pad = 0;
    const void* w_tc = nullptr;           // tcgen05 conv: BF16 [tc_n_pad][kh*kw*tc_cin_pad] (or null)
    int tc_n_pad = 0, tc_cin_pad = 0;
    int halo = 0;                         // 1: `weight` is the halo-tiled layout [ceil(cin/4)][kh*kw][4][conv_halo_bn(cout)]
    int halo_order = 0;                   // halo kernel: 0 blocked per-quad sums, 1 the direct kernel's (tap, channel) order,
                                          // 2 one running sum quad by quad
    const float* bias = nullptr;          // [cout] (padded to conv_halo_bn(cout) for the halo kernel)
    int act = 0;
    const void* residual = nullptr;       // NHWC [n, ho/res_scale, wo/res_scale, cout], added after act
    int res_scale = 1;
    void* out = nullptr;
    int out_cstride = 0, out_coff = 0;
    DType dtype = DT_F32;
    // tcgen05 kernels: a pipeline wait that runs out stores its code here
    // (null: the kernel file's own flag) and gives up after wait_ns (0: 2 s).
    int* err = nullptr;
    uint64_t wait_ns = 0;
};
cudaError_t launch_conv(const ConvParams& p, cudaStream_t stream);

// tcgen05 implicit-GEMM conv of one NHWC BF16 source (gemm_tc.cu): 8 x 16
// output-pixel tiles, each K step a strided 4D TMA box of 64 channels at one
// tap, TMA stores of the output tile.  Needs w_tc.
bool conv_tc_supported(const ConvParams& p);
cudaError_t launch_conv_tc(const ConvParams& p, cudaStream_t stream);

// Halo-tiled SIMT conv (conv_halo.cu): 3x3 at stride 1 or 2 and 2x2 at
// stride 1, cout a multiple of 8 up to 64, NHWC sources (power-of-two
// upsampled views) or the 3-channel NCHW FP32 image at stride 2.  Sums each
// output per input quad (blocked) or, with halo_order = 1, in the direct
// kernel's (ky, kx, channel) order when the tile's whole input fits a stage.
bool conv_halo_supported(const ConvParams& p);
int conv_halo_bn(int cout);   // output channels the packed weights and bias are padded to
cudaError_t launch_conv_halo(const ConvParams& p, cudaStream_t stream);

// Implicit-GEMM view of a dense conv for the SIMT GEMM kernel (gemm_simt.cu).
struct ConvGather {
    int hi = 0, wi = 0, ho = 0, wo = 0, cin = 0, kh = 0, kw = 0, sh = 1, sw = 1, pt = 0, pl = 0;
    int nsrc = 0;
    ConvSource src[4];
    int shift[4] = {0, 0, 0, 0};          // log2 of each source's upsampling factor
};
// True when the conv can run as a SIMT implicit GEMM: NHWC sources with whole
// channel quads, power-of-two upsampling, cout >= 16.
bool conv_gemm_supported(const ConvParams& p);
// Runs the conv through the implicit-GEMM SIMT kernel (needs weight_kn).
cudaError_t launch_conv_gemm(const ConvParams& p, cudaStream_t stream);

// ---------------------------------------------------------------------------
// Depthwise convolution, any k x k / stride, fused bias + activation +
// residual (residual added after the activation, same shape as the output).
// ---------------------------------------------------------------------------
struct DwParams {
    int n = 0, hi = 0, wi = 0, c = 0;
    const void* in = nullptr;
    int in_cstride = 0, in_coff = 0;
    int ho = 0, wo = 0;
    int kh = 0, kw = 0, sh = 1, sw = 1, pt = 0, pl = 0;
    const float* weight = nullptr;   // [kh*kw][c]
    const float* bias = nullptr;     // [c] or null
    int act = 0;
    const void* residual = nullptr;  // [n, ho, wo, c] tight, or null
    void* out = nullptr;             // [n, ho, wo, c] tight
    DType dtype = DT_F32;
};
cudaError_t launch_dwconv(const DwParams& p, cudaStream_t stream);
// kernel: 0 the default choice, 1 the tiled kernel, 2 the rolling-row 3x3 kernel.
cudaError_t launch_dwconv_kernel(const DwParams& p, cudaStream_t stream, int kernel);

// ---------------------------------------------------------------------------
// Pointwise GEMM  C[m, n] = act(A[m, k] * W + bias) (+ residual)
//   A rows are NHWC pixels (or sequence steps); optionally every A element
//   is multiplied by a per-(image, channel) SE gate first.  The residual may
//   be read through the same gate (LCNet pair: the residual is the gated
//   token output) and through nearest upsampling of the pixel grid.
// ---------------------------------------------------------------------------
struct GemmParams {
    int m = 0, n = 0, k = 0;
    const void* a = nullptr;
    int lda = 0;
    const float* gate = nullptr;      // [images][k], A *= gate[m / rows_per_image]
    int rows_per_image = 1;
    const float* w = nullptr;         // FP32 path: [k][n_pad4]
    const void* w_tc = nullptr;       // tensor-core path: BF16 [n_pad][k_pad] K-major
    int n_pad = 0, k_pad = 0;
    const float* bias = nullptr;      // [n]
    int act = 0;
    const void* residual = nullptr;   // [rows][ldr] added after act
    int ldr = 0;
    const float* res_gate = nullptr;  // residual *= res_gate[img][col] (stride n)
    int res_scale = 1, h = 1, w_px = 1;  // residual via nearest upsample of an h x w grid per image
    void* c = nullptr;
    int ldc = 0, coff = 0;
    DType dtype = DT_F32;             // storage of A, residual and C
    int c_f32 = 0;                    // 1: C is FP32 regardless of dtype
    // tcgen05 GEMM: wait-expiry flag (null: g_tc_error) and bound (0: 2 s);
    // skip_load = 1 (self-test only) leaves CTA 0's first stage unloaded so
    // that the waits on it run out.
    int* err = nullptr;
    uint64_t wait_ns = 0;
    int skip_load = 0;
};
cudaError_t launch_gemm(const GemmParams& p, cudaStream_t stream);

// Pointwise pair out = W2 GELU(W1 (A*gate) + b1) + b2 (+ A*gate), one pixel
// row per thread with the 2C hidden units kept in registers (LCNet
// channel_conv1 / channel_conv2, src/cpu/backend.rs:443-695).  rowgemm.cu.
struct PairRowsParams {
    long long m = 0;
    int c_in = 0, c_out = 0;
    const void* a = nullptr;          // [m][c_in]
    const float* gate = nullptr;      // [images][c_in] or null
    int rows_per_image = 1;
    const float* w1t = nullptr;       // [2 c_in][c_in]
    const float* w2 = nullptr;        // [2 c_in][c_out]
    const float* b1 = nullptr;        // [2 c_in]
    const float* b2 = nullptr;        // [c_out]
    int residual = 0;                 // add the gated input (c_out == c_in)
    void* c = nullptr;                // [m][c_out]
    DType dtype = DT_F32;
};
bool pair_rows_supported(int c_in, int c_out);
cudaError_t launch_pair_rows(const PairRowsParams& p, cudaStream_t stream);
// Row-per-thread pointwise GEMM for N <= 128 (rowgemm.cu).
bool rows_gemm_supported(const GemmParams& p);
cudaError_t launch_rows_gemm(const GemmParams& p, cudaStream_t stream);
// FP32 SIMT GEMMs (gemm_simt.cu: any shape; gemm_stream.cu: persistent,
// double-buffered, K <= 128 and N <= 128).  All FP32 GEMM kernels sum each
// output in k order and add bias, activation and residual in the same order,
// so they give bit-identical results.
cudaError_t launch_gemm_simt(const GemmParams& p, cudaStream_t stream);
bool gemm_stream_supported(const GemmParams& p);
cudaError_t launch_gemm_stream(const GemmParams& p, cudaStream_t stream);

// Tensor-core (tcgen05) GEMM availability: BF16 storage, k_pad % 64 == 0, n_pad % 16 == 0.
bool gemm_tc_supported(const GemmParams& p);
cudaError_t launch_gemm_tc(const GemmParams& p, cudaStream_t stream);
// Reads and clears the tensor-core kernel's wait-expiry code (0 = none; host sync).
int gemm_tc_error_and_clear();

// ---------------------------------------------------------------------------
// tcgen05 GEMM / implicit-GEMM conv over BF16 operands (tc_engine.cu).
// planes 1: BF16 A (activations), W and C; planes 3: FP32 A, W and C, each
// operand split into three BF16 pieces and the six leading products
// accumulated (FP32-class products).  K order of a conv: (ky, kx, channel).
struct TcEngineParams {
    int mode = 0;                     // 0: dense A rows; 1: conv window gather (conv)
    int planes = 1;
    int m = 0, n = 0, k = 0;
    int n_pad = 0, k_pad = 0;         // W is BF16 [planes][n_pad][k_pad], k_pad % 64 == 0
    const void* w = nullptr;
    const void* a = nullptr;          // mode 0: [m][lda]
    int lda = 0;
    const float* gate = nullptr;      // mode 0: A *= gate[row / rows_per_image][k]
    int rows_per_image = 1;
    ConvGather conv;                  // mode 1: geometry, sources (channel counts per source)
    const float* bias = nullptr;      // [n]
    int act = 0;
    const void* residual = nullptr;   // same dtype as C, [rows][ldr], nearest-upsampled by res_scale
    int ldr = 0, res_scale = 1, out_h = 1, out_w = 1;
    void* c = nullptr;                // BF16 (planes 1) or FP32 (planes 3) [m][ldc] at column coff
    int ldc = 0, coff = 0;
    int* err = nullptr;               // wait-expiry flag (null: g_tce_error)
    uint64_t wait_ns = 0;             // pipeline wait bound (0: 2 s)
    int skip_load = 0;                // self-test only: CTA 0's first W load is never issued
};
// FP32-class tcgen05 GEMM over FP32 activations (gemm_split.cu): A is loaded
// as FP32 by TMA and split into three BF16 pieces in shared memory, W comes
// pre-split ([3][n_pad][k_pad] BF16, pack_engine_kn with planes 3), the six
// leading products accumulate in FP32 in TMEM.  The SE gate scales A (and
// res_gate the residual) inside the kernel.
struct SplitGemmParams {
    int m = 0, n = 0, k = 0;          // k % 16 == 0
    const float* a = nullptr;         // [m][lda], lda % 4 == 0, 16-byte aligned
    int lda = 0;
    const float* gate = nullptr;      // A *= gate[row / rows_per_image][k] (or null)
    int rows_per_image = 1;
    const void* w = nullptr;          // BF16 [3][n_pad][k_pad], k_pad % 64 == 0
    int n_pad = 0, k_pad = 0;
    const float* bias = nullptr;      // [n] or null
    int act = 0;
    const float* residual = nullptr;  // [rows][ldr] FP32 added after act, nearest-upsampled by res_scale
    int ldr = 0;
    const float* res_gate = nullptr;  // residual *= res_gate[row / rows_per_image][col] (or null)
    int res_scale = 1, out_h = 1, out_w = 1;
    float* c = nullptr;               // [m][ldc] at column coff (16-byte aligned rows)
    int ldc = 0, coff = 0;
    int* err = nullptr;               // wait-expiry flag (null: g_split_error)
    uint64_t wait_ns = 0;             // pipeline wait bound (0: 2 s)
    int skip_load = 0;                // self-test only: CTA 0's first stage is never loaded
    // Pre-split A (dense mode only): BF16 [3][m][k_pad], the three pieces of
    // the gated A as launch_split_planes writes them.  The GEMM then loads the
    // pieces like W instead of splitting A in shared memory for every N tile
    // (`a` and `gate` unused); the products, and so C, are bit-identical.
    const void* a_planes = nullptr;
    // Implicit-GEMM convolution (conv = 1): A is the NHWC FP32 input
    // [n_img][hi][wi] with pixel pitch lda and `cin` channels; K order (ky,
    // kx, channel) with each tap's channels padded to cpt = k / (kh * kw) =
    // gemm_split_conv_cpt(cin) (the padding reads zeros: outside the TMA
    // map); a tile is 8 x 16 output pixels of one image, each 64-wide K block
    // one or two taps in strided 4D TMA boxes; C is NHWC [n_img][ho][wo] with
    // pixel pitch ldc at channel coff; the residual (res_scale 1, no gate) is
    // NHWC [n_img][ho][wo] with pixel pitch ldr.  No gate or pre-split A in
    // this mode.
    int conv = 0;
    int n_img = 0, hi = 0, wi = 0, ho = 0, wo = 0, kh = 0, kw = 0, stride = 1, pt = 0, pl = 0;
    int cin = 0;                      // conv mode: input channels (0: cpt)
};
// Channels per tap of the split conv for `cin` input channels: 32 for 32, else
// cin rounded up to a multiple of 64 (cin > 32, cin % 4 == 0); 0 when the
// mode does not take cin.
int gemm_split_conv_cpt(int cin);
int gemm_split_tile_n(int n, int k);  // output channels per tile for K = k (n_pad is a multiple of it; 0: K too long)
// The three BF16 pieces of A (gated as the GEMM would gate it) into
// planes [3][m][k_pad], zeros past column k: p.a, p.lda, p.gate,
// p.rows_per_image, p.m, p.k, p.k_pad of a dense SplitGemmParams.
cudaError_t launch_split_planes(const SplitGemmParams& p, void* planes, cudaStream_t stream);
// Whether pre-splitting A pays for this shape: A would otherwise be split once
// per N tile, and four or more tiles cost more than the pieces' round trip.
bool gemm_split_presplit_pays(int m, int n, int k);
bool gemm_split_supported(const SplitGemmParams& p);
cudaError_t launch_gemm_split(const SplitGemmParams& p, cudaStream_t stream);

// Raises `func`'s dynamic shared memory limit to `bytes` on the current
// device, once per device (the attribute is per device context).
cudaError_t allow_dynamic_smem(const void* func, int bytes);

int tc_engine_tile_n(int n, int planes);
bool tc_engine_supported(const TcEngineParams& p);
cudaError_t launch_tc_engine(const TcEngineParams& p, cudaStream_t stream);
int tc_engine_error_and_clear();

// ---------------------------------------------------------------------------
// Squeeze-excitation
// ---------------------------------------------------------------------------
// partial[img][chunk][c] = sum over the chunk's pixels of x[img, :, :, c].
// Fixed chunking and fixed summation order: results are bit-reproducible.
struct PoolParams {
    int n = 0, hw = 0, c = 0;
    const void* in = nullptr;
    int in_cstride = 0;
    int chunks = 1;
    float* sum = nullptr;      // [n][chunks][c]
    DType dtype = DT_F32;
};
int channel_sum_chunks(int hw, int c);
cudaError_t launch_channel_sum(const PoolParams& p, cudaStream_t stream);

// gate[img][c] = hard_sigmoid(W2 relu(W1 mean + b1) + b2; alpha, 0.5),
// mean = (sum of the chunk partials in chunk order) / hw.
struct SeMlpParams {
    int n = 0, c = 0, r = 0, hw = 0, chunks = 1;
    const float* sum = nullptr;
    const float* w1 = nullptr;  // [r][c]
    const float* b1 = nullptr;  // [r]
    const float* w2 = nullptr;  // [c][r]
    const float* b2 = nullptr;  // [c]
    float alpha = 1.f / 6.f;
    float* gate = nullptr;      // [n][c]
    int f64 = 0;                // 1: mean and dot products accumulated in double (FP32 mode)
};
cudaError_t launch_se_mlp(const SeMlpParams& p, cudaStream_t stream);

// channel_sum and se_mlp in one launch: the last block to finish its chunk of
// an image (a per-image arrival counter) runs that image's MLP from the chunk
// partials, in chunk order, so the gate is the same as the two-launch form's.
// counters: n ints, zero before the launch; the kernel leaves them zero.
struct SePoolParams {
    PoolParams pool;
    SeMlpParams mlp;                  // n, c, r, hw, chunks, sum as in `pool`
    int* counters = nullptr;
};
cudaError_t launch_se_pool_mlp(const SePoolParams& p, cudaStream_t stream);

// out = x * g (mode 0) or x + x * g (mode 1), then + upsample(addend, add_scale)
struct GateApplyParams {
    int n = 0, h = 0, w = 0, c = 0;
    const void* x = nullptr;
    const float* gate = nullptr;
    int mode = 0;
    const void* addend = nullptr;    // [n, h/add_scale, w/add_scale, c] or null
    int add_scale = 1;
    void* out = nullptr;
    int out_cstride = 0, out_coff = 0;
    DType dtype = DT_F32;
};
cudaError_t launch_gate_apply(const GateApplyParams& p, cudaStream_t stream);

// ---------------------------------------------------------------------------
// Detector head tail: ConvT 2x2 s2 (+folded BN) ReLU -> ConvT 2x2 s2 -> sigmoid,
// one thread per input pixel writing its 4x4 output patch, plus the DB
// binarisation mask (src/cpu/model.rs:1516-1520, src/ocr.rs:745).
// ---------------------------------------------------------------------------
struct HeadParams {
    int n = 0, h = 0, w = 0, ch = 0;
    const void* in = nullptr;     // [n, h, w, ch]
    const float* w_up = nullptr;  // [4 taps][ch in][ch out]
    const float* b_up = nullptr;  // [ch]
    const float* w_fin = nullptr; // [4 taps][ch]
    float b_fin = 0.f;
    float* prob = nullptr;        // [n, 4h, 4w] or null
    float* logits = nullptr;      // [n, 4h, 4w] or null
    uint8_t* mask = nullptr;      // [n, 4h, 4w] or null
    float threshold = 0.2f;
    DType dtype = DT_F32;
};
cudaError_t launch_det_head(const HeadParams& p, cudaStream_t stream);

// 2x2 stride-1 max pool padded at the bottom / right (pads never win;
// src/cpu/ops.rs:1520-1535), written into a channel slice of `out`.
struct MaxPoolParams {
    int n = 0, h = 0, w = 0, c = 0;
    const void* in = nullptr;       // [n, h, w, c] tight
    void* out = nullptr;
    int out_cstride = 0, out_coff = 0;
    DType dtype = DT_F32;
};
cudaError_t launch_maxpool_same_upper(const MaxPoolParams& p, cudaStream_t stream);


// ---------------------------------------------------------------------------
// Recognizer ops
// ---------------------------------------------------------------------------
// 3x2 stride-(3,2) average pool (src/cpu/ops.rs:1536-1566)
struct AvgPoolParams {
    int n = 0, h = 0, w = 0, c = 0;
    const void* in = nullptr;
    void* out = nullptr;          // [n, h/3, w/2, c]
    DType dtype = DT_F32;
};
cudaError_t launch_avgpool_3x2(const AvgPoolParams& p, cudaStream_t stream);

// Row LayerNorm, two-pass, eps (src/cpu/kernels/mod.rs:2288-2310); optional
// residual added after the affine transform.
struct LayerNormParams {
    int rows = 0, c = 0;
    const void* in = nullptr;
    const float* weight = nullptr;
    const float* bias = nullptr;
    float eps = 1e-6f;
    const void* residual = nullptr;
    void* out = nullptr;
    DType dtype = DT_F32;
};
cudaError_t launch_layernorm(const LayerNormParams& p, cudaStream_t stream);

// Multi-head self-attention over a [n, t, 3, heads, d] QKV buffer
// (src/cpu/model.rs:1705-1725); output [n, t, heads * d].
struct AttentionParams {
    int n = 0, t = 0, heads = 0, d = 0;
    const void* qkv = nullptr;
    void* out = nullptr;
    float scale = 1.f;
    DType dtype = DT_F32;
};
cudaError_t launch_attention(const AttentionParams& p, cudaStream_t stream);

// Row softmax + greedy-CTC statistics over FP32 logits [rows, classes]:
// probabilities, arg-max (last index among equal maxima), its probability and
// the top-2 logit margin.  Any output may be null.
struct SoftmaxParams {
    int rows = 0, classes = 0;
    int ld = 0;                       // logits row stride in floats (0: classes)
    const float* logits = nullptr;
    float* prob = nullptr;
    int32_t* index = nullptr;
    float* max_prob = nullptr;
    float* margin = nullptr;
};
cudaError_t launch_softmax_ctc(const SoftmaxParams& p, cudaStream_t stream);

// ---------------------------------------------------------------------------
// Image preprocessing: quad -> rectangle bilinear resample of packed RGB8,
// rounded to integers, BGR order, (x * scale + bias) per channel, zero past
// content_width (src/preprocess/kernels.rs:94-165).  Output NCHW FP32.
// ---------------------------------------------------------------------------
struct PreprocessParams {
    const uint8_t* rgb = nullptr;   // [src_h][src_w][3]
    int src_w = 0, src_h = 0;
    float corners[8] = {0};
    int out_w = 0, out_h = 0, content_w = 0;
    float scale[3] = {0}, bias[3] = {0};   // per output channel (B, G, R)
    float* out = nullptr;           // [3][out_h][out_w]
};
cudaError_t launch_preprocess(const PreprocessParams& p, cudaStream_t stream);

// Elementwise conversion between storage types / layouts.
cudaError_t launch_nchw_to_nhwc(const float* in, void* out, int n, int c, int h, int w, DType dt, cudaStream_t stream);
cudaError_t launch_to_f32(const void* in, float* out, size_t count, DType dt, cudaStream_t stream);
cudaError_t launch_check_finite(const float* in, size_t count, int* flag, cudaStream_t stream);
// dst[0, count) = src[0, count), *flag = 1 if any value is not finite (16-byte aligned buffers).
cudaError_t launch_copy_check(const float* src, float* dst, size_t count, int* flag, cudaStream_t stream);
// Copies `count` 32-bit words on `stream` as a kernel (a copy-engine copy
// would queue behind the copies of other streams).
cudaError_t launch_copy_words(const void* src, void* dst, size_t count, cudaStream_t stream);
// Same over `rows` rows of `cols` values at row stride `ld`.
cudaError_t launch_check_finite_rows(const float* in, size_t rows, size_t cols, size_t ld, int* flag, cudaStream_t stream);
// FP32 CUDA-core throughput probe (fp32_peak.cu): blocks x 512 threads, each
// 16 FMA chains x iters steps (2 * 16 * iters * 512 * blocks flops).
cudaError_t launch_fp32_peak(float* sink, int blocks, int iters, bool packed, cudaStream_t stream);

}  // namespace ppocr
