/*
 * ppocr_b200.h - C ABI of the B200-native PP-OCRv6 detector / recognizer backend.
 *
 * This is the drop-in boundary for ppocr-rs's direct-model GPU API
 * (`ppocr_rs::gpu`, src/gpu/mod.rs:1-13).  Each entry point replaces one Rust
 * item, cited beside it.  Conventions:
 *   - every call returns an `int` status: PPOCR_OK (0) or one of the error
 *     codes below, which map 1:1 onto the variants of `gpu::Error`
 *     (src/gpu/error.rs:8-45); the message of the last failure on the calling
 *     thread is returned by ppocr_last_error();
 *   - handles are opaque; a handle is used by one thread at a time;
 *   - host pointers are plain arrays owned by the caller; nothing crosses the
 *     ABI as a C++ exception or a framework tensor type;
 *   - shapes are NCHW [n, c, h, w] for inputs, [n, 1, h, w] for detector
 *     outputs and [n, t, classes] for recognizer outputs, as in
 *     `ModelOutput` (src/gpu/model.rs:38-42).
 */
#ifndef PPOCR_B200_H
#define PPOCR_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: one per `gpu::Error` variant (src/gpu/error.rs:8-45). */
enum ppocr_status {
    PPOCR_OK = 0,
    PPOCR_ERR_READ_FILE = 1,            /* Error::ReadFile */
    PPOCR_ERR_SAFETENSORS = 2,          /* Error::Safetensors */
    PPOCR_ERR_TENSOR_NOT_FOUND = 3,     /* Error::TensorNotFound */
    PPOCR_ERR_UNSUPPORTED_DTYPE = 4,    /* Error::UnsupportedDtype */
    PPOCR_ERR_SHAPE_MISMATCH = 5,       /* Error::ShapeMismatch */
    PPOCR_ERR_TENSOR_SIZE_OVERFLOW = 6, /* Error::TensorSizeOverflow */
    PPOCR_ERR_TENSOR_BYTE_LENGTH = 7,   /* Error::TensorByteLength */
    PPOCR_ERR_INVALID_TENSOR_RANGE = 8, /* Error::InvalidTensorRange */
    PPOCR_ERR_INVALID_MODEL = 9,        /* Error::InvalidModel */
    PPOCR_ERR_INVALID_INPUT = 10,       /* Error::InvalidInput */
    PPOCR_ERR_GPU = 11                  /* Error::Gpu */
};

/* Model tiers: `ModelSize` (src/models.rs:62-69). */
enum ppocr_model_size { PPOCR_MEDIUM = 0, PPOCR_SMALL = 1, PPOCR_TINY = 2 };

/* Activation storage / GEMM precision of a loaded model.
 * FP32:   FP32 activations and FP32-class arithmetic (the parity mode): the
 *         1x1 convs and the dense convs over 32 or 64 k input channels on tcgen05 with both
 *         operands carried as three BF16 pieces (the six leading products
 *         accumulated in FP32, the dominant sum in its own accumulators); the
 *         other convs, depthwise, head and SE on CUDA-core FP32 FMA.
 * BF16:   BF16 activations in HBM, tcgen05 BF16 tensor-core GEMMs with FP32
 *         accumulation; all other arithmetic FP32 in registers.
 * FP32_TC: FP32 activations; pointwise and dense convs on tcgen05 with each
 *         FP32 operand split into three BF16 pieces (x = x0 + x1 + x2) and
 *         the six leading products accumulated in FP32 (FP32-class products,
 *         tensor-core accumulation order). */
enum ppocr_precision { PPOCR_PRECISION_FP32 = 0, PPOCR_PRECISION_BF16 = 1, PPOCR_PRECISION_FP32_TC = 2 };

typedef struct ppocr_gpu ppocr_gpu;
typedef struct ppocr_image ppocr_image;
typedef struct ppocr_model ppocr_model;

/* Options of ppocr_*_load_ex.  Zero-initialise, then set the fields. */
typedef struct ppocr_load_options {
    int precision;   /* enum ppocr_precision; default FP32 */
    int use_graph;   /* 1: replay each forward as one captured CUDA graph */
    int simt_only;   /* 1: CUDA-core kernels only (no tcgen05); for A/B checks */
    int keep_tensors; /* 1: every activation keeps its own arena range, so
                         ppocr_model_read_tensor sees each op's output after a
                         forward (diagnostics; the arena grows to their sum) */
    int reserved[4];
} ppocr_load_options;

/* Fills `options` with the defaults (FP32, CUDA graphs on). */
void ppocr_load_options_default(ppocr_load_options* options);

/* Message of the last failed call on this thread ("" if none). */
const char* ppocr_last_error(void);

/* Number of visible CUDA devices. New: ppocr-rs picks one wgpu adapter
 * (src/gpu/runtime.rs:99-104); the B200 build shards across devices. */
int ppocr_gpu_count(int* count);

/* Gpu::new() (src/gpu/runtime.rs:94-167): binds `device`, creates its stream
 * set and the per-device activation arena. */
int ppocr_gpu_create(int device, ppocr_gpu** out);
void ppocr_gpu_destroy(ppocr_gpu* gpu);

/* Gpu::info() (src/gpu/runtime.rs:169-171): adapter name into `name`. */
int ppocr_gpu_info(const ppocr_gpu* gpu, char* name, size_t capacity);

/* Gpu::upload_rgb(width, height, &[u8]) (src/gpu/runtime.rs:174-229):
 * interleaved RGB8, `len` must equal width*height*3. */
int ppocr_upload_rgb(ppocr_gpu* gpu, uint32_t width, uint32_t height,
                     const uint8_t* pixels, size_t len, ppocr_image** out);
void ppocr_image_destroy(ppocr_image* image);

/* gpu::Detector::load(&Gpu, path, ModelSize, [n,c,h,w]) (src/gpu/model.rs:50-93).
 * Validates the shape (src/gpu/model.rs:268-276) and the tier's tensor count
 * (src/gpu/model.rs:58-65), packs the safetensors weights. */
int ppocr_detector_load(ppocr_gpu* gpu, const char* path, int size,
                        const size_t input_shape[4], ppocr_model** out);
int ppocr_detector_load_ex(ppocr_gpu* gpu, const char* path, int size,
                           const size_t input_shape[4],
                           const ppocr_load_options* options, ppocr_model** out);

/* gpu::Recognizer::load (src/gpu/model.rs:156-220), shape rules at
 * src/gpu/model.rs:278-286.  `shared_weights_from` (may be NULL) reuses the
 * device weights of an already-loaded recognizer of the same file and tier,
 * as `load_with_shared_weights` does (src/gpu/model.rs:168-218). */
int ppocr_recognizer_load(ppocr_gpu* gpu, const char* path, int size,
                          const size_t input_shape[4], ppocr_model** out);
int ppocr_recognizer_load_ex(ppocr_gpu* gpu, const char* path, int size,
                             const size_t input_shape[4],
                             const ppocr_load_options* options,
                             const ppocr_model* shared_weights_from,
                             ppocr_model** out);
void ppocr_model_destroy(ppocr_model* model);

/* Device-free load check (new): runs every check of Detector::load /
 * Recognizer::load (src/gpu/model.rs:50-93, 156-220: input shape, tensor
 * count, names, shapes, dtypes, rank-one separability) and builds the plan
 * without touching a GPU.  kind: 0 detector, 1 recognizer.  Any output
 * pointer may be NULL. */
int ppocr_inspect_model(const char* path, int kind, int size, const size_t input_shape[4], int precision,
                        size_t* ops, size_t* arena_bytes, size_t* weight_bytes, size_t output_shape[4]);

/* Seeded random-init checkpoint (new; the reference downloads the released
 * weights, src/models.rs:200-222, which needs a network): writes a
 * safetensors file holding every tensor of the kind (0 detector,
 * 1 recognizer) / size tier in the reference's names and shapes, drawn from
 * the benchmark configs' distributions (detector conv weights
 * N(0, sqrt(2 / fan_in)), recognizer conv / linear weights N(0, 0.02), batch
 * norm gamma 1 / beta 0 / mean 0 / var 1, layer norm weight 1 / bias 0,
 * biases 0).  Each tensor has its own generator seeded by (seed, name), so the
 * file depends only on (kind, size, seed).  Needs no GPU.  Backs
 * ppocr-gpu-bench --seed-weights. */
int ppocr_write_seeded_weights(const char* path, int kind, int size, uint64_t seed);

/* ModelOutput::shape: writes the output shape (rank 4 for the detector,
 * rank 3 for the recognizer) and the element count. */
int ppocr_model_output_shape(const ppocr_model* model, size_t shape[4],
                             size_t* rank, size_t* elements);
/* Input shape the model was loaded for. */
int ppocr_model_input_shape(const ppocr_model* model, size_t shape[4]);

/* Detector::forward / Recognizer::forward(&[f32]) (src/gpu/model.rs:95-114,
 * 222-238): NCHW F32 host input of `input_len` values, host output of
 * `output_capacity` values (>= ppocr_model_output_shape's element count).
 * Detector output: probability map.  Recognizer output: per-step class
 * probabilities (softmax), as the reference returns. */
int ppocr_model_forward(ppocr_model* model, const float* input, size_t input_len,
                        float* output, size_t output_capacity);

/* New: the host-buffer forward of `images` inputs (a multiple of the model's
 * batch), run as images / batch chunks of the model's batch with each chunk's
 * host-to-device copy, forward and device-to-host copy on their own streams,
 * so copies of one chunk overlap the forward of the next.  `input` holds
 * images x 3 x H x W values and `output` receives images x (per-image output)
 * values, exactly what ppocr_model_forward returns chunk by chunk (the
 * kernels are batch-invariant).  Page-locked host buffers let the copies run
 * asynchronously; pageable ones still work.  Errors as ppocr_model_forward. */
int ppocr_model_forward_pipelined(ppocr_model* model, const float* input, size_t images, float* output,
                                  size_t output_capacity);
/* New, recognizer only: ppocr_model_forward_pipelined that returns, per
 * (image, step), only the greedy-CTC arg-max class and its probability (what
 * decode_ctc_greedy_for_input reads, src/ocr.rs:800-853), in the layout of
 * ppocr_recognizer_forward_ctc: `indices` and `probabilities` receive
 * images x T entries each (capacity = entries each array holds).  The full
 * probability rows stay on the device (their finiteness is still checked), so
 * 8 bytes per step cross to the host instead of 4 x classes. */
int ppocr_recognizer_forward_pipelined_ctc(ppocr_model* model, const float* input, size_t images, int32_t* indices,
                                           float* probabilities, size_t capacity);

/* forward_image(&GpuImage, ImagePreprocess) (src/gpu/model.rs:116-138,
 * 240-259; ImagePreprocess::{detector, recognizer} src/gpu/runtime.rs:50-69):
 * device-side quad resample, BGR swap, normalisation and right zero-padding
 * past `content_width` (the detector passes the input width).  `corners`
 * holds four (x, y) source points: top-left, top-right, bottom-right,
 * bottom-left.  Batch must be 1. */
int ppocr_model_forward_image(ppocr_model* model, const ppocr_image* image,
                              const float corners[8], size_t content_width,
                              float* output, size_t output_capacity);

/* Detector::benchmark / Recognizer::benchmark(&[f32], warmup, runs)
 * (src/gpu/model.rs:140-148, 261-266; timed region src/gpu/runtime.rs:1798-1830):
 * uploads once, then times `runs` forwards on the device (submit + wait, no
 * readback).  `samples_ms` receives `runs` values in milliseconds. */
int ppocr_model_benchmark(ppocr_model* model, const float* input, size_t input_len,
                          size_t warmup, size_t runs, double* samples_ms);

/* Batched device-resident forward (new; the reference has no batched
 * device API).  `device_input` is a device pointer to NCHW F32 input,
 * `device_output` a device pointer receiving the F32 output, `stream` a
 * cudaStream_t (NULL = the model's own stream).  Asynchronous: returns
 * after enqueueing. */
int ppocr_model_forward_device(ppocr_model* model, const float* device_input,
                               float* device_output, void* stream);

/* Zero-copy device residency (new): the device addresses of the model's own
 * input slot (NCHW F32) and output (detector probability map / recognizer
 * probabilities, F32) inside the activation arena.  Valid until another
 * model on the same ppocr_gpu grows the arena (a later load); re-query after
 * loading.  ppocr_model_run enqueues one forward over whatever the input
 * slot holds on `stream` (NULL = the model's stream) and returns. */
int ppocr_model_device_buffers(ppocr_model* model, float** device_input, float** device_output);
int ppocr_model_run(ppocr_model* model, void* stream);

/* Waits (bounded by `timeout_ms`; <= 0 means 60 s) for the model's stream;
 * Error::Gpu on a timeout or an asynchronous device error, and Error::Gpu
 * when a tensor-core pipeline wait of the last device-resident run ran out.
 *
 * Every call that waits for the device does so for at most 60 s.  When that
 * limit runs out the call fails with PPOCR_ERR_GPU while work it queued may
 * still be running: that work may still write the call's output buffers
 * afterwards, and the ppocr_gpu handle (with its models and images) refuses
 * every further call with PPOCR_ERR_GPU.  Destroying the handles stays safe. */
int ppocr_model_synchronize(ppocr_model* model, int timeout_ms);

/* Recognizer only: greedy CTC on the device (replaces the argmax scan of
 * decode_ctc_greedy_for_input, src/ocr.rs:800-853).  For every (n, t) writes
 * the arg-max class (ties resolve to the highest index, as Rust's
 * Iterator::max_by does), its probability, and the top-2 logit margin.
 * All three are host arrays of n*t entries; any may be NULL. */
int ppocr_recognizer_forward_ctc(ppocr_model* model, const float* input, size_t input_len,
                                 int32_t* indices, float* probabilities, float* margins);

/* Per-op profile: the counterpart of PPOCR_GPU_PROFILE's per-dispatch
 * timestamps (src/gpu/runtime.rs:1815-1817, 1832-1933).  op_info describes
 * op `index` of the plan: name, kernel family, algorithmic bytes (every
 * tensor read and written once plus weights) and FLOPs.  profile runs the
 * plan op by op `runs` times over the current input slot, bracketing every op
 * with CUDA events on the model's stream, and writes each op's mean time in
 * milliseconds to op_ms[count]. */
int ppocr_model_op_count(const ppocr_model* model, size_t* count);
int ppocr_model_op_info(const ppocr_model* model, size_t index, char* name, size_t name_capacity,
                        char* kind, size_t kind_capacity, double* bytes, double* flops);
int ppocr_model_profile(ppocr_model* model, size_t runs, double* op_ms);

/* Diagnostic (new): the plan's activation tensors.  tensor_info gives the
 * name of tensor `index` (the op or weight prefix that writes it), its NHWC
 * shape (n, h, w, c; raw buffers report n = h = w = 1 and c = their element
 * count) and its storage type (0 F32, 1 BF16).  read_tensor copies the
 * tensor's current arena contents to `out` as F32 (BF16 widened).  An
 * intermediate tensor holds its op's output after a forward only when the
 * model was loaded with keep_tensors = 1; otherwise later ops may reuse its
 * memory. */
int ppocr_model_tensor_count(const ppocr_model* model, size_t* count);
int ppocr_model_tensor_info(const ppocr_model* model, size_t index, char* name, size_t name_capacity, size_t shape[4],
                            int* dtype);
int ppocr_model_read_tensor(ppocr_model* model, size_t index, float* out, size_t capacity);

/* Diagnostic (new): C[m, n] = act(A[m, k] W[n, k]^T + bias) through the
 * BF16 GEMM path of this library on `gpu`.  A and W are host F32 arrays
 * rounded to BF16 on upload; C is returned in F32.  used_tensor_cores is set
 * to 1 when the tcgen05 kernel ran (k % 8 == 0), wait_error to the kernel's
 * wait-expiry code (0 = none).  act: 0 none, 1 ReLU, 2 SiLU, 3 GELU. */
int ppocr_selftest_gemm(ppocr_gpu* gpu, int m, int n, int k, const float* a, const float* w, const float* bias,
                        int act, float* c, int* used_tensor_cores, int* wait_error);

/* Diagnostic (new): ppocr_selftest_gemm writing into a channel slice of a
 * wider output, with an optional residual, as the model's concat and
 * residual epilogues do.  C is [m][ldc] (ldc >= coff + n); its initial
 * contents come from `c` and columns outside [coff, coff + n) must come back
 * unchanged.  residual (may be NULL) is [m][n], added after the activation.
 * out_bf16 = 1 stores C (and reads the residual) as BF16, 0 as F32 output
 * with a BF16 residual.  act as for ppocr_selftest_gemm, plus 4 HardSwish,
 * 5 sigmoid. */
int ppocr_selftest_gemm_ex(ppocr_gpu* gpu, int m, int n, int k, const float* a, const float* w, const float* bias,
                           int act, const float* residual, int out_bf16, int ldc, int coff, float* c,
                           int* used_tensor_cores, int* wait_error);

/* Diagnostic (new): the split GEMM's implicit-conv mode (FP32 operands in
 * three BF16 pieces on tcgen05) on an NHWC FP32 input x [n, hi, wi, cin]
 * (cin 32, or above 32 in multiples of 4: each tap's channels are read
 * zero-padded to a multiple of 64) with OIHW weights w [cout, cin, kh, kw], symmetric zero
 * padding `pad` and stride 1 or 2; out receives [n, ho, wo, cout] NHWC,
 * act as for ppocr_selftest_gemm_ex, then + residual (may be NULL; NHWC
 * [n, ho, wo, cout]).  The model's dense FP32 convs over one
 * such source use this path. */
int ppocr_selftest_conv_split(ppocr_gpu* gpu, int n, int hi, int wi, int cin, int cout, int kh, int kw, int stride,
                              int pad, const float* x, const float* w, const float* bias, int act,
                              const float* residual, float* out);
/* Diagnostic (new): the FP32 pointwise GEMM of the FP32 mode,
 * C[m, n] = act((A * gate) W[n, k]^T + bias) + residual, all in F32, through
 * one chosen kernel: kernel 0 = the model's dispatch, 1 = the register-tiled
 * SIMT kernel, 2 = the row kernel (n <= 128), 3 = the streaming kernel
 * (k <= 128, n <= 128).  gate (may be NULL) is [m / rows_per_image][k] and
 * scales A; residual (may be NULL) is [m][n].  kernel_used returns the kernel
 * that ran (1..3).  k must be a multiple of 4; a kernel that does not
 * support the shape fails with PPOCR_ERR_INVALID_INPUT.  kernel 4 = the
 * tcgen05 split GEMM of the FP32 mode (k a multiple of 16): A and W carried
 * as three BF16 pieces each, the six leading products accumulated in FP32 in
 * TMEM (FP32-class rounding, not bit-identical to the CUDA-core kernels);
 * kernel 5 = the same with A split into its pieces by a kernel of its own
 * first (the model's choice when A would otherwise be split once per output
 * tile of four or more): bit-identical to kernel 4. */
int ppocr_selftest_gemm_f32(ppocr_gpu* gpu, int m, int n, int k, const float* a, const float* w, const float* bias,
                            int act, const float* gate, int rows_per_image, const float* residual, int kernel, float* c,
                            int* kernel_used);

/* Diagnostic (new): the fused FP32 LCNet channel pair of the FP32 mode,
 * out = W2 GELU(W1 (a * gate) + b1) + b2 (+ a * gate when residual is 1),
 * a [m][c_in], w1 [2 c_in][c_in], w2 [c_out][2 c_in], b1 [2 c_in], b2 [c_out],
 * gate (may be NULL) [m / rows_per_image][c_in], out [m][c_out].  The model
 * runs it on maps of at least 98,304 pixel rows; on the same inputs it must
 * equal two ppocr_selftest_gemm_f32 calls (GELU, then the residual) bit for
 * bit.  (c_in, c_out) must be one of the LCNet pairs the kernel covers. */
int ppocr_selftest_pair_f32(ppocr_gpu* gpu, int m, int c_in, int c_out, const float* a, const float* w1,
                            const float* b1, const float* w2, const float* b2, const float* gate, int rows_per_image,
                            int residual, float* out);

/* Diagnostic (new): one depthwise convolution (the models' LCNet token convs,
 * RepLkFpn / rank-one depthwise, recognizer head convs) through one chosen
 * kernel: kernel 0 = the models' dispatch, 1 = the tiled kernel (every
 * geometry), 2 = the rolling-row kernel (3x3 and 5x5; the dispatch uses it
 * for 3x3).  x is NHWC [n, hi, wi, c],
 * w is [c][kh * kw], bias (may be NULL) [c], residual (may be NULL) and out
 * NHWC [n, ho, wo, c] with ho = (hi + pt + pb - kh) / sh + 1 and wo likewise.
 * act as for ppocr_selftest_gemm_ex.  bf16 = 1 runs the BF16 mode: x and
 * residual are rounded to BF16 and out holds the BF16 results widened to F32.
 * c must be a multiple of 4 (8 with bf16).  kernel_used returns 1 or 2. */
int ppocr_selftest_dwconv(ppocr_gpu* gpu, int n, int hi, int wi, int c, int kh, int kw, int sh, int sw, int pt, int pl,
                          int pb, int pr, const float* x, const float* w, const float* bias, int act,
                          const float* residual, int bf16, int kernel, float* out, int* kernel_used);

/* Diagnostic (new): one convolution through the tcgen05 engine of the BF16
 * and FP32-class modes.  planes 1: input rounded to BF16, BF16 weights and
 * output; planes 3: FP32 input / weights split into three BF16 pieces each,
 * FP32 output.  NHWC input [n, hi, wi, cin] (cin a multiple of 8 / 4), OIHW
 * weight, symmetric padding, output NHWC [n, ho, wo, cout] in F32.  When
 * `second` is 1 the input's channels are split into two sources: the first
 * half direct, the second half read through a 2x2 same-upper max pool
 * (second == 2: through a x2 nearest upsampling of a half-size tensor given
 * as x2 [n, hi/2, wi/2, cin/2]).  1x1 / stride 1 / pad 0 with one source runs
 * the dense-rows mode.  used_tensor_cores / wait_error as for
 * ppocr_selftest_gemm. */
/* Diagnostic (new): the measured FP32 CUDA-core throughput of `gpu` in
 * TFLOP/s (independent FMA chains, no memory traffic), with plain and packed
 * two-lane FMAs: the roofline denominator for the FP32 mode's SIMT kernels. */
int ppocr_measure_fp32_peak(ppocr_gpu* gpu, double* tflops_fma, double* tflops_fma2);

int ppocr_selftest_engine(ppocr_gpu* gpu, int planes, int n, int hi, int wi, int cin, int cout, int kh, int kw,
                          int stride, int pad, int second, const float* x, const float* x2, const float* w,
                          const float* bias, int act, float* out, int* used_tensor_cores, int* wait_error);

/* Diagnostic (new; the reference's wgpu path has no device-side waits):
 * failure detection of the tensor-core kernels.  Runs one small GEMM whose
 * first CTA never issues the loads of its first pipeline stage, so its waits
 * on that stage run out after wait_ms (1..2000) milliseconds, as a wait on an
 * arrive that never comes would in a forward.  kernel 0 = the BF16 tcgen05
 * GEMM, 1 = the engine with BF16 operands, 2 = the engine with FP32 operands
 * in three BF16 pieces, 3 = the split GEMM (FP32 activations split in shared
 * memory).  The kernel drains its copies and MMAs in flight,
 * frees its TMEM and returns; the call then fails with PPOCR_ERR_GPU and
 * *code holds the kernel's wait-expiry code (nonzero).  The device stays
 * usable.  In a model forward the same expiry fails the forward with
 * PPOCR_ERR_GPU (src/gpu/error.rs:8-45, Error::Gpu). */
int ppocr_selftest_wait_expiry(ppocr_gpu* gpu, int kernel, int wait_ms, int* code);

/* Recognizer only: the classifier's pre-softmax logits [n, t, classes]
 * (new; the reference fuses the softmax, src/cpu/backend.rs:1288-1290, so it
 * never exposes them). */
int ppocr_recognizer_forward_logits(ppocr_model* model, const float* input, size_t input_len,
                                    float* logits, size_t logits_capacity);

/* Device preprocessing alone (prepare_detector / prepare_recognizer,
 * src/preprocess.rs:37-76): quad resample of `image` into an NCHW F32
 * [1, 3, out_h, out_w] host array.  kind 0 = detector normalisation
 * (ImageNet mean/std), 1 = recognizer ((x/255 - 0.5)/0.5); columns at and
 * past `content_width` are zero. */
int ppocr_preprocess(ppocr_gpu* gpu, const ppocr_image* image, const float corners[8], size_t content_width,
                     size_t out_h, size_t out_w, int kind, float* output);

/* ppocr_preprocess without any device allocation.  This entry point has no
 * counterpart in the reference.  It is for callers that cannot call
 * cudaMalloc: code under a fixed device-memory budget or an allocator that
 * owns all device memory, and servers that forbid allocation calls (which
 * synchronise the device) while serving.  Same arguments and results as
 * ppocr_preprocess, but the output is staged in a fixed 4 MiB device array
 * built into the library (present on every GPU that loads it, until exit),
 * so 3 * out_h * out_w must not exceed 1048576 floats (InvalidInput beyond).
 * The first call on a device looks up that array's device address (once per
 * device); make that first call before any stream capture.  All calls on a
 * device share the array: calls whose GPU work overlaps race and must be
 * serialised by the caller.  A call that fails because the device did not
 * finish within the wait limit may leave the kernel and the copy still
 * writing the array and `output`; the gpu handle then refuses further calls
 * (see ppocr_model_synchronize). */
int ppocr_preprocess_noalloc(ppocr_gpu* gpu, const ppocr_image* image, const float corners[8], size_t content_width,
                             size_t out_h, size_t out_w, int kind, float* output);

/* Detector only: probability map plus the DB binarisation mask
 * (prob >= threshold, src/ocr.rs:745,1047) as bytes of n*h*w. Either output
 * may be NULL. */
int ppocr_detector_forward_mask(ppocr_model* model, const float* input, size_t input_len,
                                float threshold, float* probabilities, uint8_t* mask);

/* ------------------------------------------------------------------------
 * End-to-end pipeline (src/ocr.rs): the host steps around the two models
 * and an engine that runs them with device preprocessing / rectification.
 * ---------------------------------------------------------------------- */

/* Recognizer only: device rectification of `count` (== batch) crops of
 * `image` straight into the model input -- crop i is the quad corners[8 i ..
 * 8 i + 8] resampled to 48 x content_widths[i] on the model's canvas, as
 * ImagePreprocess::recognizer (src/gpu/runtime.rs:58-69) prepares one crop
 * and prepare_recognizer (src/preprocess.rs:49-76) stacks a batch -- then the
 * forward and the greedy-CTC statistics of ppocr_recognizer_forward_ctc,
 * each [count, t] (any output may be NULL). Only these statistics cross to
 * the host. */
int ppocr_recognizer_forward_crops(ppocr_model* model, const ppocr_image* image, size_t count, const float* corners,
                                   const size_t* content_widths, int32_t* indices, float* probabilities,
                                   float* margins);

/* ppocr_recognizer_forward_crops over crops of several images (crop i from
 * images[i]) filling the first `count` <= batch slots; unused slots are
 * zero-filled and the statistics are returned for the first `count` rows.
 * Each crop's result does not depend on the other slots. */
int ppocr_recognizer_forward_crops_ex(ppocr_model* model, const ppocr_image* const* images, size_t count,
                                      const float* corners, const size_t* content_widths, int32_t* indices,
                                      float* probabilities, float* margins);

/* Detector only: forward_image (full-image corners) of `count` == batch
 * images at once; probability maps [count, h, w]. */
int ppocr_detector_forward_images(ppocr_model* model, const ppocr_image* const* images, size_t count,
                                  float* probabilities);

/* DetectorPostprocessOptions (src/ocr.rs:231-271). */
typedef struct ppocr_postprocess_options {
    float binary_threshold; /* 0.2 */
    float box_threshold;    /* 0.4 */
    size_t min_area;        /* 3 */
    float unclip_ratio;     /* 1.4 */
    size_t max_boxes;       /* 1000 */
} ppocr_postprocess_options;
void ppocr_postprocess_options_default(ppocr_postprocess_options* options);

/* Detection (src/ocr.rs:225-229): quadrilateral x0 y0 .. x3 y3 in source pixels. */
typedef struct ppocr_detection {
    float polygon[8];
    float score;
} ppocr_detection;

/* extract_detections (src/ocr.rs:723-782), host only: components of the
 * [height, width] probability map's content area, boxes mapped to a source
 * image of source_w x source_h. Writes min(count, capacity) detections and
 * sets *count to the number found. */
int ppocr_db_postprocess(const float* probabilities, size_t height, size_t width, uint32_t source_w,
                         uint32_t source_h, uint32_t content_w, uint32_t content_h,
                         const ppocr_postprocess_options* options, ppocr_detection* detections, size_t capacity,
                         size_t* count);

/* Recognition dictionary (load_dictionary / parse_dictionary, src/ocr.rs:785-790, 892-965). */
typedef struct ppocr_dictionary ppocr_dictionary;
int ppocr_dictionary_parse(const char* contents, size_t length, ppocr_dictionary** out);
int ppocr_dictionary_load(const char* path, ppocr_dictionary** out);
int ppocr_dictionary_size(const ppocr_dictionary* dictionary, size_t* size);
/* UTF-8 entry `index`; *length = its byte length (copied when it fits `capacity`). */
int ppocr_dictionary_entry(const ppocr_dictionary* dictionary, size_t index, char* text, size_t capacity,
                           size_t* length);
void ppocr_dictionary_destroy(ppocr_dictionary* dictionary);

/* decode_ctc_greedy_for_input (src/ocr.rs:800-853), host only, from
 * probability rows [steps, classes]. The UTF-8 text is written to `text`
 * (NUL-terminated when it fits; *text_length = its byte length, InvalidInput
 * when capacity is too small). */
int ppocr_ctc_decode(const ppocr_dictionary* dictionary, const float* probabilities, size_t steps, size_t classes,
                     size_t content_width, size_t input_width, char* text, size_t text_capacity,
                     size_t* text_length, float* score);
/* The same from per-step arg-max classes and their probabilities, the
 * statistics ppocr_recognizer_forward_crops returns. */
int ppocr_ctc_decode_steps(const ppocr_dictionary* dictionary, const int32_t* indices, const float* probabilities,
                           size_t steps, size_t classes, size_t content_width, size_t input_width, char* text,
                           size_t text_capacity, size_t* text_length, float* score);

/* OcrEngine / OcrOptions (src/ocr.rs:276-326, 364-540) on this library's GPU
 * backend. detector_max_side 0 selects the released model's resize policy. */
typedef struct ppocr_engine ppocr_engine;
typedef struct ppocr_engine_options {
    int detector_size;            /* ppocr_model_size, PPOCR_TINY */
    int recognizer_size;          /* PPOCR_TINY */
    int precision;                /* ppocr_precision of both models, PPOCR_PRECISION_FP32 */
    uint32_t detector_max_side;   /* 736 */
    ppocr_postprocess_options postprocess;
    int recognizer_precision;     /* new: 0 = as `precision`; 1 + ppocr_precision for the recognizer alone */
    int reserved[7];
} ppocr_engine_options;
void ppocr_engine_options_default(ppocr_engine_options* options);
/* OcrEngine::load: the dictionary is parsed and checked against the
 * recognizer's classes; models are loaded per input shape on first use. */
int ppocr_engine_create(ppocr_gpu* gpu, const char* detector_model, const char* recognizer_model,
                        const char* dictionary, const ppocr_engine_options* options, ppocr_engine** out);
void ppocr_engine_destroy(ppocr_engine* engine);
/* OcrEngine::recognize on packed RGB8 pixels: format 0 writes the pretty JSON
 * of OcrResult (README.md:34-49), 1 its text() (non-empty lines joined by
 * newlines). *result is allocated by the library (free with
 * ppocr_string_free). */
int ppocr_engine_recognize(ppocr_engine* engine, const uint8_t* rgb, size_t rgb_length, uint32_t width,
                           uint32_t height, int format, char** result, size_t* result_length);
void ppocr_string_free(char* text);
/* OcrEngine::recognize over `count` pages at once (same results per page as
 * ppocr_engine_recognize): pages of one detector input size run through the
 * detector together, the DB postprocess runs on host threads, and crops of
 * all pages that share a canvas width are recognized in shared batches.
 * results[i] / result_lengths[i] as for ppocr_engine_recognize. */
int ppocr_engine_recognize_batch(ppocr_engine* engine, size_t count, const uint8_t* const* rgb,
                                 const size_t* rgb_lengths, const uint32_t* widths, const uint32_t* heights,
                                 int format, char** results, size_t* result_lengths);

/* New: wall time in ms of each stage of the last ppocr_engine_recognize_batch
 * call: [0] page uploads, [1] detector forwards, [2] DB postprocess, [3]
 * recognizer forwards with crop rectification (and any model loads), [4]
 * result assembly.  Writes min(count, 5) values. */
int ppocr_engine_stage_times(const ppocr_engine* engine, double* ms, size_t count);

/* New: several GPUs behind one OcrEngine call.  One ppocr_gpu + ppocr_engine
 * per listed device (the same models, dictionary and options on each), each
 * driven by its own host thread.  The reference drives one backend per
 * OcrEngine (src/ocr.rs:365-604); this is its recognize over a batch of pages
 * spread across devices, with no device-to-device traffic. */
typedef struct ppocr_engine_pool ppocr_engine_pool;
int ppocr_engine_pool_create(const int* devices, size_t count, const char* detector_model,
                             const char* recognizer_model, const char* dictionary,
                             const ppocr_engine_options* options, ppocr_engine_pool** out);
/* Waits for any worker still running a late shard, then frees every device. */
void ppocr_engine_pool_destroy(ppocr_engine_pool* pool);
int ppocr_engine_pool_size(const ppocr_engine_pool* pool, size_t* count);
/* ppocr_engine_recognize_batch over the pool: pages dealt round-robin to the
 * devices, results in page order.  A device whose shard is not done within
 * timeout_ms (<= 0: no limit) has its pages dealt again to the devices that
 * answered and gets no work until that shard has returned (its results are
 * dropped; it reads the caller's memory only before this call returns).  A
 * device failing with PPOCR_ERR_GPU is left out of the call and its pages
 * dealt again; PPOCR_ERR_GPU when no device is left.  devices_used[i] (may
 * be null) receives the CUDA ordinal that produced results[i]. */
int ppocr_engine_pool_recognize_batch(ppocr_engine_pool* pool, size_t count, const uint8_t* const* rgb,
                                      const size_t* rgb_lengths, const uint32_t* widths, const uint32_t* heights,
                                      int format, int timeout_ms, char** results, size_t* result_lengths,
                                      int* devices_used);
/* Diagnostic (new), host only: the pool's dispatcher over `workers` fake
 * devices (<= 32) and `items` items.  A worker whose bit is set in
 * stall_mask answers after stall_ms, one in fail_mask fails with
 * PPOCR_ERR_GPU, the others after 2 ms; every answer is item * 10.
 * owner[i] / values[i] receive the worker that produced item i and its value. */
int ppocr_selftest_dispatch(size_t workers, size_t items, uint32_t stall_mask, uint32_t fail_mask, int stall_ms,
                            int timeout_ms, int* owner, int* values);

#ifdef __cplusplus
}
#endif

#endif /* PPOCR_B200_H */
