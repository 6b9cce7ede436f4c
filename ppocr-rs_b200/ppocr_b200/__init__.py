"""Python face of the B200 PP-OCRv6 backend, shaped like ``ppocr_rs::gpu``.

ppocr-rs exposes ``Gpu``, ``GpuImage``, ``ImagePreprocess``, ``Detector``,
``Recognizer``, ``ModelOutput`` and ``ModelSize`` (src/gpu/mod.rs:1-13).  This
module mirrors them over the C ABI in include/ppocr_b200.h (ctypes, no
framework types): same constructors, argument meaning and error variants.
Every call goes to the compiled library; there is no fallback path, and a
missing library raises ``ImportError`` on first use.
"""

from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

__all__ = [
    "Error", "ReadFile", "Safetensors", "TensorNotFound", "UnsupportedDtype", "ShapeMismatch",
    "TensorSizeOverflow", "TensorByteLength", "InvalidTensorRange", "InvalidModel", "InvalidInput", "GpuError",
    "ModelSize", "Precision", "Gpu", "GpuImage", "ImagePreprocess", "ModelOutput", "Detector", "Recognizer",
    "library", "library_path", "gpu_count", "inspect_model", "Engine", "EnginePool", "selftest_dispatch",
]

_HERE = os.path.dirname(os.path.abspath(__file__))


def library_path() -> str:
    return os.environ.get("PPOCR_B200_LIB", os.path.join(_HERE, "libppocr_b200.so"))


# ---------------------------------------------------------------------------
# Errors: one class per gpu::Error variant (src/gpu/error.rs:8-45)
# ---------------------------------------------------------------------------


class Error(RuntimeError):
    code = -1


class ReadFile(Error):
    code = 1


class Safetensors(Error):
    code = 2


class TensorNotFound(Error):
    code = 3


class UnsupportedDtype(Error):
    code = 4


class ShapeMismatch(Error):
    code = 5


class TensorSizeOverflow(Error):
    code = 6


class TensorByteLength(Error):
    code = 7


class InvalidTensorRange(Error):
    code = 8


class InvalidModel(Error):
    code = 9


class InvalidInput(Error):
    code = 10


class GpuError(Error):
    code = 11


_ERRORS = {cls.code: cls for cls in (ReadFile, Safetensors, TensorNotFound, UnsupportedDtype, ShapeMismatch,
                                      TensorSizeOverflow, TensorByteLength, InvalidTensorRange, InvalidModel,
                                      InvalidInput, GpuError)}


class ModelSize:
    """ModelSize (src/models.rs:62-69)."""
    MEDIUM = 0
    SMALL = 1
    TINY = 2

    @staticmethod
    def parse(value) -> int:
        if isinstance(value, int):
            return value
        return {"medium": 0, "small": 1, "tiny": 2}[str(value).lower()]


class Precision:
    """FP32: CUDA-core FP32 (parity mode); BF16: BF16 storage + tcgen05 BF16 GEMMs;
    FP32_TC: FP32 storage; tcgen05 GEMMs / convs on three-way BF16-split operands
    (FP32-class products)."""
    FP32 = 0
    BF16 = 1
    FP32_TC = 2

    @staticmethod
    def parse(value) -> int:
        if isinstance(value, int):
            return value
        return {"fp32": 0, "bf16": 1, "fp32tc": 2}[str(value).lower()]


class _PostOptions(C.Structure):
    _fields_ = [("binary_threshold", C.c_float), ("box_threshold", C.c_float), ("min_area", C.c_size_t),
                ("unclip_ratio", C.c_float), ("max_boxes", C.c_size_t)]


class _Detection(C.Structure):
    _fields_ = [("polygon", C.c_float * 8), ("score", C.c_float)]


class _EngineOptions(C.Structure):
    _fields_ = [("detector_size", C.c_int), ("recognizer_size", C.c_int), ("precision", C.c_int),
                ("detector_max_side", C.c_uint32), ("postprocess", _PostOptions), ("recognizer_precision", C.c_int),
                ("reserved", C.c_int * 7)]


class _LoadOptions(C.Structure):
    _fields_ = [("precision", C.c_int), ("use_graph", C.c_int), ("simt_only", C.c_int), ("keep_tensors", C.c_int),
                ("reserved", C.c_int * 4)]


_SIZE4 = C.c_size_t * 4
_lib = None


def library() -> C.CDLL:
    """The loaded C-ABI library (loaded once; raises ImportError if it is not built)."""
    global _lib
    if _lib is not None:
        return _lib
    path = library_path()
    if not os.path.exists(path):
        raise ImportError(f"ppocr_b200 native library not found at {path}; build it with `make -C ppocr-rs_b200`")
    lib = C.CDLL(path)
    P, I, S = C.c_void_p, C.c_int, C.c_size_t
    FP = C.POINTER(C.c_float)
    sig = {
        "ppocr_last_error": (C.c_char_p, []),
        "ppocr_load_options_default": (None, [C.POINTER(_LoadOptions)]),
        "ppocr_gpu_count": (I, [C.POINTER(C.c_int)]),
        "ppocr_gpu_create": (I, [I, C.POINTER(P)]),
        "ppocr_gpu_destroy": (None, [P]),
        "ppocr_gpu_info": (I, [P, C.c_char_p, S]),
        "ppocr_upload_rgb": (I, [P, C.c_uint32, C.c_uint32, C.POINTER(C.c_uint8), S, C.POINTER(P)]),
        "ppocr_image_destroy": (None, [P]),
        "ppocr_detector_load": (I, [P, C.c_char_p, I, _SIZE4, C.POINTER(P)]),
        "ppocr_detector_load_ex": (I, [P, C.c_char_p, I, _SIZE4, C.POINTER(_LoadOptions), C.POINTER(P)]),
        "ppocr_recognizer_load": (I, [P, C.c_char_p, I, _SIZE4, C.POINTER(P)]),
        "ppocr_recognizer_load_ex": (I, [P, C.c_char_p, I, _SIZE4, C.POINTER(_LoadOptions), P, C.POINTER(P)]),
        "ppocr_model_destroy": (None, [P]),
        "ppocr_inspect_model": (I, [C.c_char_p, I, I, _SIZE4, I, C.POINTER(S), C.POINTER(S), C.POINTER(S), _SIZE4]),
        "ppocr_model_output_shape": (I, [P, _SIZE4, C.POINTER(S), C.POINTER(S)]),
        "ppocr_model_input_shape": (I, [P, _SIZE4]),
        "ppocr_model_forward": (I, [P, FP, S, FP, S]),
        "ppocr_model_forward_pipelined": (I, [P, FP, S, FP, S]),
        "ppocr_recognizer_forward_pipelined_ctc": (I, [P, FP, S, C.POINTER(C.c_int32), FP, S]),
        "ppocr_model_forward_image": (I, [P, P, FP, S, FP, S]),
        "ppocr_model_benchmark": (I, [P, FP, S, S, S, C.POINTER(C.c_double)]),
        "ppocr_model_forward_device": (I, [P, P, P, P]),
        "ppocr_model_device_buffers": (I, [P, C.POINTER(P), C.POINTER(P)]),
        "ppocr_model_run": (I, [P, P]),
        "ppocr_model_synchronize": (I, [P, I]),
        "ppocr_recognizer_forward_ctc": (I, [P, FP, S, C.POINTER(C.c_int32), FP, FP]),
        "ppocr_detector_forward_mask": (I, [P, FP, S, C.c_float, FP, C.POINTER(C.c_uint8)]),
        "ppocr_recognizer_forward_logits": (I, [P, FP, S, FP, S]),
        "ppocr_model_op_count": (I, [P, C.POINTER(S)]),
        "ppocr_model_op_info": (I, [P, S, C.c_char_p, S, C.c_char_p, S, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        "ppocr_model_profile": (I, [P, S, C.POINTER(C.c_double)]),
        "ppocr_selftest_gemm": (I, [P, I, I, I, FP, FP, FP, I, FP, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
        "ppocr_selftest_gemm_ex": (I, [P, I, I, I, FP, FP, FP, I, FP, I, I, I, FP, C.POINTER(C.c_int),
                                       C.POINTER(C.c_int)]),
        "ppocr_selftest_gemm_f32": (I, [P, I, I, I, FP, FP, FP, I, FP, I, FP, I, FP, C.POINTER(C.c_int)]),
        "ppocr_selftest_conv_split": (I, [P, I, I, I, I, I, I, I, I, I, FP, FP, FP, I, FP, FP]),
        "ppocr_measure_fp32_peak": (I, [P, C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        "ppocr_selftest_dwconv": (I, [P, I, I, I, I, I, I, I, I, I, I, I, I, FP, FP, FP, I, FP, I, I, FP,
                                      C.POINTER(C.c_int)]),
        "ppocr_selftest_pair_f32": (I, [P, I, I, I, FP, FP, FP, FP, FP, FP, I, I, FP]),
        "ppocr_preprocess_noalloc": (I, [P, P, FP, S, S, S, I, FP]),
        "ppocr_preprocess": (I, [P, P, FP, S, S, S, I, FP]),
        "ppocr_selftest_engine": (I, [P, I, I, I, I, I, I, I, I, I, I, I, FP, FP, FP, FP, I, FP, C.POINTER(C.c_int),
                                      C.POINTER(C.c_int)]),
        "ppocr_recognizer_forward_crops": (I, [P, P, S, FP, C.POINTER(S), C.POINTER(C.c_int32), FP, FP]),
        "ppocr_postprocess_options_default": (None, [C.POINTER(_PostOptions)]),
        "ppocr_db_postprocess": (I, [FP, S, S, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32,
                                     C.POINTER(_PostOptions), C.POINTER(_Detection), S, C.POINTER(S)]),
        "ppocr_dictionary_parse": (I, [C.c_char_p, S, C.POINTER(P)]),
        "ppocr_dictionary_load": (I, [C.c_char_p, C.POINTER(P)]),
        "ppocr_dictionary_size": (I, [P, C.POINTER(S)]),
        "ppocr_dictionary_entry": (I, [P, S, C.c_char_p, S, C.POINTER(S)]),
        "ppocr_dictionary_destroy": (None, [P]),
        "ppocr_ctc_decode": (I, [P, FP, S, S, S, S, C.c_char_p, S, C.POINTER(S), FP]),
        "ppocr_ctc_decode_steps": (I, [P, C.POINTER(C.c_int32), FP, S, S, S, S, C.c_char_p, S, C.POINTER(S), FP]),
        "ppocr_engine_options_default": (None, [C.POINTER(_EngineOptions)]),
        "ppocr_engine_create": (I, [P, C.c_char_p, C.c_char_p, C.c_char_p, C.POINTER(_EngineOptions), C.POINTER(P)]),
        "ppocr_engine_destroy": (None, [P]),
        "ppocr_engine_recognize": (I, [P, C.POINTER(C.c_uint8), S, C.c_uint32, C.c_uint32, I,
                                       C.POINTER(C.c_void_p), C.POINTER(S)]),
        "ppocr_string_free": (None, [C.c_void_p]),
        "ppocr_engine_stage_times": (I, [P, C.POINTER(C.c_double), S]),
        "ppocr_engine_recognize_batch": (I, [P, S, C.POINTER(C.c_void_p), C.POINTER(S), C.POINTER(C.c_uint32),
                                             C.POINTER(C.c_uint32), I, C.POINTER(C.c_void_p), C.POINTER(S)]),
        "ppocr_recognizer_forward_crops_ex": (I, [P, C.POINTER(C.c_void_p), S, FP, C.POINTER(S),
                                                  C.POINTER(C.c_int32), FP, FP]),
        "ppocr_detector_forward_images": (I, [P, C.POINTER(C.c_void_p), S, FP]),
        "ppocr_selftest_wait_expiry": (I, [P, I, I, C.POINTER(C.c_int)]),
        "ppocr_model_tensor_count": (I, [P, C.POINTER(S)]),
        "ppocr_model_tensor_info": (I, [P, S, C.c_char_p, S, _SIZE4, C.POINTER(C.c_int)]),
        "ppocr_model_read_tensor": (I, [P, S, FP, S]),
        "ppocr_write_seeded_weights": (I, [C.c_char_p, I, I, C.c_uint64]),
        "ppocr_engine_pool_create": (I, [C.POINTER(C.c_int), S, C.c_char_p, C.c_char_p, C.c_char_p,
                                         C.POINTER(_EngineOptions), C.POINTER(P)]),
        "ppocr_engine_pool_destroy": (None, [P]),
        "ppocr_engine_pool_size": (I, [P, C.POINTER(S)]),
        "ppocr_engine_pool_recognize_batch": (I, [P, S, C.POINTER(C.c_void_p), C.POINTER(S), C.POINTER(C.c_uint32),
                                                  C.POINTER(C.c_uint32), I, I, C.POINTER(C.c_void_p), C.POINTER(S),
                                                  C.POINTER(C.c_int)]),
        "ppocr_selftest_dispatch": (I, [S, S, C.c_uint32, C.c_uint32, I, I, C.POINTER(C.c_int),
                                        C.POINTER(C.c_int)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _check(status: int) -> None:
    if status != 0:
        msg = library().ppocr_last_error().decode("utf-8", "replace")
        raise _ERRORS.get(status, Error)(msg)


def _fptr(a: np.ndarray):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def gpu_count() -> int:
    n = C.c_int(0)
    _check(library().ppocr_gpu_count(C.byref(n)))
    return n.value


def write_seeded_weights(path: str, kind: str, size, seed: int = 0) -> str:
    """The C++ seeded checkpoint writer (ppocr-gpu-bench --seed-weights): the
    reference tensor layout with the benchmark configs' spec distributions."""
    _check(library().ppocr_write_seeded_weights(str(path).encode(), 0 if kind == "det" else 1, ModelSize.parse(size),
                                                int(seed)))
    return str(path)


def inspect_model(path: str, kind: str, size, input_shape: Sequence[int], precision="fp32") -> dict:
    """Device-free load check; returns ops, arena_bytes, weight_bytes, output_shape."""
    ops, arena, wbytes = C.c_size_t(), C.c_size_t(), C.c_size_t()
    out = _SIZE4()
    _check(library().ppocr_inspect_model(str(path).encode(), 0 if kind == "det" else 1, ModelSize.parse(size),
                                         _SIZE4(*input_shape), Precision.parse(precision), C.byref(ops), C.byref(arena),
                                         C.byref(wbytes), out))
    rank = 4 if kind == "det" else 3
    return {"ops": ops.value, "arena_bytes": arena.value, "weight_bytes": wbytes.value,
            "output_shape": [int(v) for v in list(out)[:rank]]}


# ---------------------------------------------------------------------------
# Gpu / images (src/gpu/runtime.rs:24-229)
# ---------------------------------------------------------------------------


class Gpu:
    """Gpu::new(): one CUDA device with its stream set and activation arena."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(library().ppocr_gpu_create(int(device), C.byref(h)))
        self._h = h
        self.device = int(device)

    def info(self) -> str:
        buf = C.create_string_buffer(256)
        _check(library().ppocr_gpu_info(self._h, buf, 256))
        return buf.value.decode()

    def upload_rgb(self, width: int, height: int, pixels) -> "GpuImage":
        arr = np.ascontiguousarray(np.asarray(pixels, dtype=np.uint8).reshape(-1))
        h = C.c_void_p()
        _check(library().ppocr_upload_rgb(self._h, int(width), int(height),
                                          arr.ctypes.data_as(C.POINTER(C.c_uint8)), arr.size, C.byref(h)))
        return GpuImage(h, self, int(width), int(height))

    def preprocess(self, image: "GpuImage", corners, content_width: int, out_h: int, out_w: int,
                   kind: str = "det") -> np.ndarray:
        """Device quad resample + normalisation into NCHW float32 [1, 3, out_h, out_w]."""
        c = np.asarray(corners, dtype=np.float32).reshape(8)
        out = np.empty((1, 3, int(out_h), int(out_w)), dtype=np.float32)
        _check(library().ppocr_preprocess(self._h, image._h, _fptr(c), int(content_width), int(out_h), int(out_w),
                                          0 if kind == "det" else 1, _fptr(out)))
        return out

    def preprocess_noalloc(self, image: "GpuImage", corners, content_width: int, out_h: int, out_w: int,
                           kind: str = "det") -> np.ndarray:
        """preprocess() for callers that cannot allocate device memory: the result is
        staged in a fixed 4 MiB device array inside the library (3 * out_h * out_w
        <= 1048576 floats); overlapping calls on one device must be serialised."""
        c = np.asarray(corners, dtype=np.float32).reshape(8)
        out = np.empty((1, 3, int(out_h), int(out_w)), dtype=np.float32)
        _check(library().ppocr_preprocess_noalloc(self._h, image._h, _fptr(c), int(content_width), int(out_h),
                                                  int(out_w), 0 if kind == "det" else 1, _fptr(out)))
        return out

    def selftest_gemm(self, a, w, bias=None, act: int = 0):
        """BF16 GEMM diagnostic: returns (C float32 [m, n], used_tensor_cores, wait_error)."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        m, k = a.shape
        n = w.shape[0]
        c = np.empty((m, n), dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        used, err = C.c_int(), C.c_int()
        _check(library().ppocr_selftest_gemm(self._h, m, n, k, _fptr(a), _fptr(w), None if b is None else _fptr(b),
                                             int(act), _fptr(c), C.byref(used), C.byref(err)))
        return c, bool(used.value), err.value

    def selftest_engine(self, planes, x, w, bias=None, act=0, stride=1, pad=0, second=0, x2=None):
        """Tensor-core engine conv diagnostic: x NHWC [n, h, w, cin], w OIHW; returns
        (out NHWC float32, used_tensor_cores, wait_error)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        n, hi, wi, cin = x.shape
        cout, _, kh, kw = w.shape
        ho, wo = (hi + 2 * pad - kh) // stride + 1, (wi + 2 * pad - kw) // stride + 1
        out = np.empty((n, ho, wo, cout), dtype=np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        x2a = None if x2 is None else np.ascontiguousarray(x2, dtype=np.float32)
        used, err = C.c_int(), C.c_int()
        _check(library().ppocr_selftest_engine(self._h, int(planes), n, hi, wi, cin, cout, kh, kw, int(stride), int(pad),
                                               int(second), _fptr(x), None if x2a is None else _fptr(x2a), _fptr(w),
                                               None if b is None else _fptr(b), int(act), _fptr(out), C.byref(used),
                                               C.byref(err)))
        return out, bool(used.value), err.value

    def selftest_wait_expiry(self, kernel: int, wait_ms: int = 20) -> int:
        """Makes one tensor-core pipeline wait run out (kernel 0: BF16 GEMM, 1 / 2:
        the engine with 1 / 3 operand planes); raises GpuError carrying the
        kernel's wait-expiry code as `.wait_code`."""
        code = C.c_int()
        status = library().ppocr_selftest_wait_expiry(self._h, int(kernel), int(wait_ms), C.byref(code))
        try:
            _check(status)
        except Error as e:
            e.wait_code = code.value
            raise
        return code.value

    def selftest_gemm_ex(self, a, w, c_init, coff: int, bias=None, act: int = 0, residual=None, out_bf16: bool = True):
        """GEMM diagnostic into columns [coff, coff + n) of c_init [m, ldc] (other columns must survive);
        returns (C float32 [m, ldc], used_tensor_cores, wait_error)."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        m, k = a.shape
        n = w.shape[0]
        c = np.array(c_init, dtype=np.float32, copy=True, order="C")
        ldc = c.shape[1]
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        used, err = C.c_int(), C.c_int()
        _check(library().ppocr_selftest_gemm_ex(self._h, m, n, k, _fptr(a), _fptr(w), None if b is None else _fptr(b),
                                                int(act), None if r is None else _fptr(r), int(bool(out_bf16)),
                                                int(ldc), int(coff), _fptr(c), C.byref(used), C.byref(err)))
        return c, bool(used.value), err.value

    def measure_fp32_peak(self):
        """Measured FP32 CUDA-core throughput (TFLOP/s) with plain and packed FMAs."""
        a, b = C.c_double(), C.c_double()
        _check(library().ppocr_measure_fp32_peak(self._h, C.byref(a), C.byref(b)))
        return a.value, b.value

    def selftest_pair_f32(self, a, w1, b1, w2, b2, gate=None, rows_per_image: int = 1, residual: bool = False):
        """Fused FP32 LCNet pair: a [m, c], w1 [2c, c], w2 [c', 2c]; returns out float32 [m, c']."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        w1 = np.ascontiguousarray(w1, dtype=np.float32)
        w2 = np.ascontiguousarray(w2, dtype=np.float32)
        b1 = np.ascontiguousarray(b1, dtype=np.float32)
        b2 = np.ascontiguousarray(b2, dtype=np.float32)
        m, c = a.shape
        co = w2.shape[0]
        out = np.zeros((m, co), np.float32)
        g = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32)
        _check(library().ppocr_selftest_pair_f32(self._h, m, c, co, _fptr(a), _fptr(w1), _fptr(b1), _fptr(w2), _fptr(b2),
                                                 None if g is None else _fptr(g), int(rows_per_image), int(bool(residual)),
                                                 _fptr(out)))
        return out

    def selftest_dwconv(self, x, w, bias=None, stride=(1, 1), pad=(0, 0, 0, 0), act: int = 0, residual=None,
                        bf16: bool = False, kernel: int = 0):
        """Depthwise conv diagnostic: x NHWC [n, hi, wi, c], w [c, kh, kw], pad (top, left, bottom, right);
        kernel 0 dispatch, 1 tiled, 2 rolling rows (3x3, 5x5).  Returns (out float32 NHWC, kernel that ran)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        n, hi, wi, c = x.shape
        kh, kw = w.shape[1], w.shape[2]
        sh, sw = stride
        pt, pl, pb, pr = pad
        ho, wo = (hi + pt + pb - kh) // sh + 1, (wi + pl + pr - kw) // sw + 1
        out = np.zeros((n, ho, wo, c), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        used = C.c_int()
        _check(library().ppocr_selftest_dwconv(self._h, n, hi, wi, c, kh, kw, sh, sw, pt, pl, pb, pr, _fptr(x), _fptr(w),
                                               None if b is None else _fptr(b), int(act),
                                               None if r is None else _fptr(r), int(bool(bf16)), int(kernel),
                                               _fptr(out), C.byref(used)))
        return out, used.value

    def selftest_gemm_f32(self, a, w, bias=None, act: int = 0, gate=None, rows_per_image: int = 1, residual=None,
                          kernel: int = 0):
        """FP32 GEMM diagnostic through one kernel (0 dispatch, 1 SIMT, 2 rows, 3 streaming,
        4 the tcgen05 split GEMM, 5 the split GEMM with A pre-split by its own kernel);
        returns (C float32 [m, n], kernel that ran)."""
        a = np.ascontiguousarray(a, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        m, k = a.shape
        n = w.shape[0]
        c = np.zeros((m, n), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        g = None if gate is None else np.ascontiguousarray(gate, dtype=np.float32)
        r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        used = C.c_int()
        _check(library().ppocr_selftest_gemm_f32(self._h, m, n, k, _fptr(a), _fptr(w), None if b is None else _fptr(b),
                                                 int(act), None if g is None else _fptr(g), int(rows_per_image),
                                                 None if r is None else _fptr(r), int(kernel), _fptr(c), C.byref(used)))
        return c, used.value

    def selftest_conv_split(self, x, w, bias=None, stride: int = 1, pad: int = 1, act: int = 0, residual=None):
        """The split GEMM's implicit conv (FP32 operands in three BF16 pieces on tcgen05):
        x NHWC float32 [n, hi, wi, cin] (cin 32, or above 32 in multiples of 4: each tap's channels
        read zero-padded to a multiple of 64), w OIHW [cout, cin, kh, kw], residual (optional) NHWC
        [n, ho, wo, cout] added after the activation;
        returns NHWC [n, ho, wo, cout]."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        w = np.ascontiguousarray(w, dtype=np.float32)
        n, hi, wi, cin = x.shape
        cout, _, kh, kw = w.shape
        ho, wo = (hi + 2 * pad - kh) // stride + 1, (wi + 2 * pad - kw) // stride + 1
        out = np.zeros((n, ho, wo, cout), np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float32)
        if r is not None and r.shape != out.shape:
            raise InvalidInput("residual must have the output's shape")
        _check(library().ppocr_selftest_conv_split(self._h, n, hi, wi, cin, cout, kh, kw, int(stride), int(pad), _fptr(x),
                                                   _fptr(w), None if b is None else _fptr(b), int(act),
                                                   None if r is None else _fptr(r), _fptr(out)))
        return out

    def close(self) -> None:
        if getattr(self, "_h", None):
            library().ppocr_gpu_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class GpuImage:
    def __init__(self, handle, gpu: Gpu, width: int, height: int):
        self._h, self.gpu, self.width, self.height = handle, gpu, width, height

    def __del__(self):
        try:
            if self._h:
                library().ppocr_image_destroy(self._h)
                self._h = None
        except Exception:
            pass


@dataclass
class ImagePreprocess:
    """ImagePreprocess::{detector, recognizer} (src/gpu/runtime.rs:50-69)."""
    corners: Sequence[Sequence[float]]
    content_width: Optional[int] = None

    @classmethod
    def detector(cls, corners) -> "ImagePreprocess":
        return cls(corners, None)

    @classmethod
    def recognizer(cls, corners, content_width: int) -> "ImagePreprocess":
        return cls(corners, int(content_width))


@dataclass
class ModelOutput:
    """ModelOutput {shape, values} (src/gpu/model.rs:38-42)."""
    shape: List[int]
    values: np.ndarray


class _Model:
    _kind = "det"

    def __init__(self, handle, gpu: Gpu, input_shape, owner_weights=None):
        self._h = handle
        self.gpu = gpu
        self.input_shape = [int(v) for v in input_shape]
        shape = _SIZE4()
        rank, elems = C.c_size_t(), C.c_size_t()
        _check(library().ppocr_model_output_shape(self._h, shape, C.byref(rank), C.byref(elems)))
        self.output_shape = [int(v) for v in list(shape)[: rank.value]]
        self.output_elements = elems.value
        self._owner = owner_weights

    def _input(self, values) -> np.ndarray:
        return np.ascontiguousarray(np.asarray(values, dtype=np.float32).reshape(-1))

    def forward(self, values) -> ModelOutput:
        x = self._input(values)
        out = np.empty(self.output_elements, dtype=np.float32)
        _check(library().ppocr_model_forward(self._h, _fptr(x), x.size, _fptr(out), out.size))
        return ModelOutput(list(self.output_shape), out)

    def forward_pipelined(self, values) -> np.ndarray:
        """Forward of any multiple of the model batch from host memory, chunk by chunk with
        the copies overlapped (ppocr_model_forward_pipelined); returns [images, ...] outputs
        as a flat float32 array of images x per-image output values."""
        x = np.ascontiguousarray(values, dtype=np.float32)
        per_in = int(np.prod(self.input_shape[1:]))
        if x.size % per_in:
            raise InvalidInput(f"invalid input: {x.size} values are not whole {self.input_shape[1:]} images")
        images = x.size // per_in
        per_out = self.output_elements // self.input_shape[0]
        out = np.empty(images * per_out, dtype=np.float32)
        _check(library().ppocr_model_forward_pipelined(self._h, _fptr(x), images, _fptr(out), out.size))
        return out

    def forward_image(self, image: GpuImage, preprocess: ImagePreprocess) -> ModelOutput:
        corners = np.asarray(preprocess.corners, dtype=np.float32).reshape(8)
        out = np.empty(self.output_elements, dtype=np.float32)
        cw = preprocess.content_width if preprocess.content_width is not None else self.input_shape[3]
        _check(library().ppocr_model_forward_image(self._h, image._h, _fptr(corners), int(cw), _fptr(out), out.size))
        return ModelOutput(list(self.output_shape), out)

    def benchmark(self, values, warmup: int, runs: int) -> List[float]:
        """Device time of each run in seconds (the reference returns Durations)."""
        x = self._input(values)
        samples = (C.c_double * max(int(runs), 1))()
        _check(library().ppocr_model_benchmark(self._h, _fptr(x), x.size, int(warmup), int(runs), samples))
        return [samples[i] / 1000.0 for i in range(int(runs))]

    # -- device-resident interface ------------------------------------------
    def device_buffers(self):
        i, o = C.c_void_p(), C.c_void_p()
        _check(library().ppocr_model_device_buffers(self._h, C.byref(i), C.byref(o)))
        return i.value, o.value

    def run(self, stream: int = 0) -> None:
        _check(library().ppocr_model_run(self._h, C.c_void_p(stream) if stream else None))

    def forward_device(self, device_input: int, device_output: int, stream: int = 0) -> None:
        _check(library().ppocr_model_forward_device(self._h, C.c_void_p(device_input), C.c_void_p(device_output),
                                                    C.c_void_p(stream) if stream else None))

    def ops(self) -> List[dict]:
        """Plan ops: name, kernel family, algorithmic bytes and FLOPs."""
        n = C.c_size_t()
        _check(library().ppocr_model_op_count(self._h, C.byref(n)))
        out = []
        for i in range(n.value):
            name, kind = C.create_string_buffer(256), C.create_string_buffer(64)
            b, f = C.c_double(), C.c_double()
            _check(library().ppocr_model_op_info(self._h, i, name, 256, kind, 64, C.byref(b), C.byref(f)))
            out.append({"name": name.value.decode(), "kind": kind.value.decode(), "bytes": b.value, "flops": f.value})
        return out

    def profile(self, runs: int = 3) -> List[float]:
        """Mean device milliseconds of every op, each bracketed by CUDA events."""
        n = C.c_size_t()
        _check(library().ppocr_model_op_count(self._h, C.byref(n)))
        ms = (C.c_double * n.value)()
        _check(library().ppocr_model_profile(self._h, int(runs), ms))
        return list(ms)

    def synchronize(self, timeout_ms: int = 0) -> None:
        _check(library().ppocr_model_synchronize(self._h, int(timeout_ms)))

    def tensors(self) -> List[dict]:
        """The plan's activation tensors: name, NHWC shape and storage type."""
        n = C.c_size_t()
        _check(library().ppocr_model_tensor_count(self._h, C.byref(n)))
        out = []
        for i in range(n.value):
            name = C.create_string_buffer(256)
            shape = _SIZE4()
            dt = C.c_int()
            _check(library().ppocr_model_tensor_info(self._h, i, name, 256, shape, C.byref(dt)))
            out.append({"index": i, "name": name.value.decode(), "shape": tuple(shape), "dtype": "bf16" if dt.value else "f32"})
        return out

    def read_tensor(self, name: str) -> np.ndarray:
        """Current contents of the named tensor as float32 NHWC (needs keep_tensors for intermediates)."""
        for t in self.tensors():
            if t["name"] == name:
                out = np.empty(t["shape"], dtype=np.float32)
                _check(library().ppocr_model_read_tensor(self._h, t["index"], _fptr(out), out.size))
                return out
        raise KeyError(name)

    def close(self) -> None:
        if getattr(self, "_h", None):
            library().ppocr_model_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _options(precision, use_graph: bool, simt_only: bool = False, keep_tensors: bool = False) -> _LoadOptions:
    o = _LoadOptions()
    library().ppocr_load_options_default(C.byref(o))
    o.precision = Precision.parse(precision)
    o.use_graph = 1 if use_graph else 0
    o.simt_only = 1 if simt_only else 0
    o.keep_tensors = 1 if keep_tensors else 0
    return o


class Detector(_Model):
    """gpu::Detector (src/gpu/model.rs:44-149)."""

    @classmethod
    def load(cls, gpu: Gpu, path: str, size, input_shape: Sequence[int], precision="fp32",
             use_graph: bool = True, simt_only: bool = False, keep_tensors: bool = False) -> "Detector":
        h = C.c_void_p()
        o = _options(precision, use_graph, simt_only, keep_tensors)
        _check(library().ppocr_detector_load_ex(gpu._h, str(path).encode(), ModelSize.parse(size),
                                                _SIZE4(*input_shape), C.byref(o), C.byref(h)))
        return cls(h, gpu, input_shape)

    def forward_mask(self, values, threshold: float = 0.2):
        """Probability map and DB binarisation mask (prob >= threshold), both [n, h, w]."""
        x = self._input(values)
        n, _, hh, ww = self.input_shape
        prob = np.empty((n, hh, ww), dtype=np.float32)
        mask = np.empty((n, hh, ww), dtype=np.uint8)
        _check(library().ppocr_detector_forward_mask(self._h, _fptr(x), x.size, float(threshold), _fptr(prob),
                                                     mask.ctypes.data_as(C.POINTER(C.c_uint8))))
        return prob, mask


class Recognizer(_Model):
    """gpu::Recognizer (src/gpu/model.rs:150-266)."""

    @classmethod
    def load(cls, gpu: Gpu, path: str, size, input_shape: Sequence[int], precision="fp32",
             use_graph: bool = True, shared_weights: Optional["Recognizer"] = None,
             simt_only: bool = False) -> "Recognizer":
        h = C.c_void_p()
        o = _options(precision, use_graph, simt_only)
        _check(library().ppocr_recognizer_load_ex(gpu._h, str(path).encode(), ModelSize.parse(size),
                                                  _SIZE4(*input_shape), C.byref(o),
                                                  shared_weights._h if shared_weights is not None else None,
                                                  C.byref(h)))
        return cls(h, gpu, input_shape, shared_weights)

    def forward_crops(self, image: "GpuImage", corners, content_widths):
        """Device rectification of each crop (corners [n, 4, 2], content widths [n]) into the
        input canvas, forward, and greedy-CTC statistics: (arg-max index, its probability,
        top-2 logit margin), each [n, t]."""
        n, t = self.output_shape[0], self.output_shape[1]
        c = np.ascontiguousarray(corners, dtype=np.float32).reshape(-1)
        cw = (C.c_size_t * n)(*[int(v) for v in content_widths])
        idx = np.empty((n, t), dtype=np.int32)
        prob = np.empty((n, t), dtype=np.float32)
        margin = np.empty((n, t), dtype=np.float32)
        _check(library().ppocr_recognizer_forward_crops(self._h, image._h, n, _fptr(c), cw,
                                                        idx.ctypes.data_as(C.POINTER(C.c_int32)), _fptr(prob),
                                                        _fptr(margin)))
        return idx, prob, margin

    def forward_logits(self, values) -> np.ndarray:
        """Pre-softmax classifier logits [n, t, classes]."""
        x = self._input(values)
        out = np.empty(self.output_shape, dtype=np.float32)
        _check(library().ppocr_recognizer_forward_logits(self._h, _fptr(x), x.size, _fptr(out), out.size))
        return out

    def forward_ctc(self, values):
        """Greedy-CTC statistics per step: (arg-max index, its probability, top-2 logit margin), each [n, t]."""
        x = self._input(values)
        n, t = self.output_shape[0], self.output_shape[1]
        idx = np.empty((n, t), dtype=np.int32)
        prob = np.empty((n, t), dtype=np.float32)
        margin = np.empty((n, t), dtype=np.float32)
        _check(library().ppocr_recognizer_forward_ctc(self._h, _fptr(x), x.size,
                                                      idx.ctypes.data_as(C.POINTER(C.c_int32)), _fptr(prob),
                                                      _fptr(margin)))
        return idx, prob, margin

    def forward_pipelined_ctc(self, values):
        """forward_pipelined over any multiple of the batch, returning only the greedy-CTC
        arg-max class and its probability per step, each [images, t]
        (ppocr_recognizer_forward_pipelined_ctc)."""
        x = np.ascontiguousarray(values, dtype=np.float32)
        per_in = int(np.prod(self.input_shape[1:]))
        if x.size % per_in:
            raise InvalidInput(f"invalid input: {x.size} values are not whole {self.input_shape[1:]} images")
        images, t = x.size // per_in, self.output_shape[1]
        idx = np.empty((images, t), dtype=np.int32)
        prob = np.empty((images, t), dtype=np.float32)
        _check(library().ppocr_recognizer_forward_pipelined_ctc(self._h, _fptr(x), images,
                                                                idx.ctypes.data_as(C.POINTER(C.c_int32)), _fptr(prob),
                                                                idx.size))
        return idx, prob


# ---------------------------------------------------------------------------
# End-to-end pipeline (src/ocr.rs): host postprocess, dictionary, CTC, engine
# ---------------------------------------------------------------------------


class PostprocessOptions:
    """DetectorPostprocessOptions (src/ocr.rs:231-271)."""

    def __init__(self, binary_threshold=0.2, box_threshold=0.4, min_area=3, unclip_ratio=1.4, max_boxes=1000):
        self.binary_threshold, self.box_threshold = binary_threshold, box_threshold
        self.min_area, self.unclip_ratio, self.max_boxes = min_area, unclip_ratio, max_boxes

    def _c(self) -> _PostOptions:
        return _PostOptions(float(self.binary_threshold), float(self.box_threshold), int(self.min_area),
                            float(self.unclip_ratio), int(self.max_boxes))


def db_postprocess(prob, source_size, content_size=None, options: PostprocessOptions = None):
    """extract_detections on a [h, w] probability map: [(polygon float32 [4, 2], score)]."""
    prob = np.ascontiguousarray(prob, dtype=np.float32)
    h, w = prob.shape[-2:]
    cw, ch = content_size if content_size is not None else (w, h)
    opts = (options or PostprocessOptions())._c()
    count = C.c_size_t()
    _check(library().ppocr_db_postprocess(_fptr(prob), h, w, int(source_size[0]), int(source_size[1]), int(cw), int(ch),
                                          C.byref(opts), None, 0, C.byref(count)))
    buf = (_Detection * max(count.value, 1))()
    _check(library().ppocr_db_postprocess(_fptr(prob), h, w, int(source_size[0]), int(source_size[1]), int(cw), int(ch),
                                          C.byref(opts), buf, count.value, C.byref(count)))
    return [(np.array(buf[i].polygon, dtype=np.float32).reshape(4, 2), np.float32(buf[i].score))
            for i in range(count.value)]


class Dictionary:
    """Recognition dictionary (parse_dictionary, src/ocr.rs:892-965)."""

    def __init__(self, handle):
        self._h = handle

    @classmethod
    def parse(cls, contents: str) -> "Dictionary":
        raw = contents.encode("utf-8")
        h = C.c_void_p()
        _check(library().ppocr_dictionary_parse(raw, len(raw), C.byref(h)))
        return cls(h)

    @classmethod
    def load(cls, path: str) -> "Dictionary":
        h = C.c_void_p()
        _check(library().ppocr_dictionary_load(str(path).encode(), C.byref(h)))
        return cls(h)

    def __len__(self) -> int:
        n = C.c_size_t()
        _check(library().ppocr_dictionary_size(self._h, C.byref(n)))
        return n.value

    def entries(self):
        out = []
        for i in range(len(self)):
            n = C.c_size_t()
            _check(library().ppocr_dictionary_entry(self._h, i, None, 0, C.byref(n)))
            buf = C.create_string_buffer(n.value + 1)
            _check(library().ppocr_dictionary_entry(self._h, i, buf, n.value + 1, C.byref(n)))
            out.append(buf.raw[:n.value].decode("utf-8", "replace"))
        return out

    def _text(self, fn, *args):
        n, score = C.c_size_t(), C.c_float()
        _check(fn(self._h, *args, None, 0, C.byref(n), C.byref(score)))
        buf = C.create_string_buffer(n.value + 1)
        _check(fn(self._h, *args, buf, n.value + 1, C.byref(n), C.byref(score)))
        return buf.raw[:n.value].decode("utf-8", "replace"), score.value

    def decode(self, probs, content_width: int, input_width: int):
        """decode_ctc_greedy_for_input on probability rows [t, classes] -> (text, score)."""
        probs = np.ascontiguousarray(probs, dtype=np.float32)
        t, c = probs.shape
        return self._text(library().ppocr_ctc_decode, _fptr(probs), t, c, int(content_width), int(input_width))

    def decode_steps(self, index, prob, classes: int, content_width: int, input_width: int):
        """The same from per-step arg-max classes and probabilities."""
        index = np.ascontiguousarray(index, dtype=np.int32)
        prob = np.ascontiguousarray(prob, dtype=np.float32)
        return self._text(library().ppocr_ctc_decode_steps, index.ctypes.data_as(C.POINTER(C.c_int32)), _fptr(prob),
                          index.size, int(classes), int(content_width), int(input_width))

    def close(self):
        if getattr(self, "_h", None):
            library().ppocr_dictionary_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _engine_options(detector_size, recognizer_size, precision, detector_max_side, postprocess, recognizer_precision):
    o = _EngineOptions()
    library().ppocr_engine_options_default(C.byref(o))
    o.detector_size = ModelSize.parse(detector_size)
    o.recognizer_size = ModelSize.parse(recognizer_size)
    o.precision = Precision.parse(precision)
    if recognizer_precision is not None:
        o.recognizer_precision = 1 + Precision.parse(recognizer_precision)
    o.detector_max_side = int(detector_max_side or 0)
    if postprocess is not None:
        o.postprocess = postprocess._c()
    return o


def _page_arrays(pages):
    pages = [np.ascontiguousarray(p, dtype=np.uint8) for p in pages]
    n = len(pages)
    ptrs = (C.c_void_p * n)(*[p.ctypes.data for p in pages])
    lens = (C.c_size_t * n)(*[p.size for p in pages])
    ws = (C.c_uint32 * n)(*[p.shape[1] for p in pages])
    hs = (C.c_uint32 * n)(*[p.shape[0] for p in pages])
    return pages, n, ptrs, lens, ws, hs


def _take_strings(outs, olens, n, fmt):
    import json

    res = []
    try:
        for i in range(n):
            text = C.string_at(outs[i], olens[i]).decode("utf-8")
            res.append(json.loads(text) if fmt == "json" else text)
    finally:
        for i in range(n):
            library().ppocr_string_free(outs[i])
    return res


class Engine:
    """OcrEngine (src/ocr.rs:364-540) on this library's GPU backend."""

    def __init__(self, gpu: Gpu, detector_model: str, recognizer_model: str, dictionary: str,
                 detector_size="tiny", recognizer_size="tiny", precision="fp32", detector_max_side: int = 736,
                 postprocess: PostprocessOptions = None, recognizer_precision=None):
        o = _engine_options(detector_size, recognizer_size, precision, detector_max_side, postprocess,
                            recognizer_precision)
        h = C.c_void_p()
        _check(library().ppocr_engine_create(gpu._h, str(detector_model).encode(), str(recognizer_model).encode(),
                                             str(dictionary).encode(), C.byref(o), C.byref(h)))
        self._h, self.gpu = h, gpu

    def recognize(self, rgb, fmt: str = "json"):
        """OcrEngine::recognize on an RGB8 [h, w, 3] array -> parsed JSON dict (fmt="json") or text."""
        import json

        rgb = np.ascontiguousarray(rgb, dtype=np.uint8)
        h, w = rgb.shape[:2]
        out, n = C.c_void_p(), C.c_size_t()
        _check(library().ppocr_engine_recognize(self._h, rgb.ctypes.data_as(C.POINTER(C.c_uint8)), rgb.size, w, h,
                                                0 if fmt == "json" else 1, C.byref(out), C.byref(n)))
        try:
            text = C.string_at(out, n.value).decode("utf-8")
        finally:
            library().ppocr_string_free(out)
        return json.loads(text) if fmt == "json" else text

    def stage_times(self) -> dict:
        """Wall ms of each stage of the last recognize_batch call."""
        ms = (C.c_double * 5)()
        _check(library().ppocr_engine_stage_times(self._h, ms, 5))
        return dict(zip(["upload", "detector", "postprocess", "recognizer", "assembly"], list(ms)))

    def recognize_batch(self, pages, fmt: str = "json"):
        """OcrEngine::recognize over several RGB8 pages at once (same per-page results)."""
        pages, n, ptrs, lens, ws, hs = _page_arrays(pages)
        outs = (C.c_void_p * n)()
        olens = (C.c_size_t * n)()
        _check(library().ppocr_engine_recognize_batch(self._h, n, ptrs, lens, ws, hs, 0 if fmt == "json" else 1,
                                                      outs, olens))
        return _take_strings(outs, olens, n, fmt)

    def close(self):
        if getattr(self, "_h", None):
            library().ppocr_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class EnginePool:
    """Several GPUs behind one OcrEngine call (new): one engine per device, each
    on its own host thread; pages are dealt round-robin and the results come
    back in page order.  A device whose shard misses `timeout_ms` has its pages
    dealt again to the others (the reference drives one backend per engine,
    src/ocr.rs:365-604)."""

    def __init__(self, devices, detector_model: str, recognizer_model: str, dictionary: str,
                 detector_size="tiny", recognizer_size="tiny", precision="fp32", detector_max_side: int = 736,
                 postprocess: PostprocessOptions = None, recognizer_precision=None):
        devices = [int(d) for d in devices]
        o = _engine_options(detector_size, recognizer_size, precision, detector_max_side, postprocess,
                            recognizer_precision)
        devs = (C.c_int * len(devices))(*devices)
        h = C.c_void_p()
        _check(library().ppocr_engine_pool_create(devs, len(devices), str(detector_model).encode(),
                                                  str(recognizer_model).encode(), str(dictionary).encode(),
                                                  C.byref(o), C.byref(h)))
        self._h, self.devices = h, devices
        self.last_devices = []

    def __len__(self):
        n = C.c_size_t()
        _check(library().ppocr_engine_pool_size(self._h, C.byref(n)))
        return n.value

    def recognize_batch(self, pages, fmt: str = "json", timeout_ms: int = 0):
        """Engine.recognize_batch spread over the pool's devices; `last_devices`
        then lists the CUDA ordinal that produced each page."""
        pages, n, ptrs, lens, ws, hs = _page_arrays(pages)
        outs = (C.c_void_p * n)()
        olens = (C.c_size_t * n)()
        used = (C.c_int * n)()
        _check(library().ppocr_engine_pool_recognize_batch(self._h, n, ptrs, lens, ws, hs, 0 if fmt == "json" else 1,
                                                           int(timeout_ms), outs, olens, used))
        self.last_devices = list(used)
        return _take_strings(outs, olens, n, fmt)

    def close(self):
        if getattr(self, "_h", None):
            library().ppocr_engine_pool_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def selftest_dispatch(workers: int, items: int, stall=(), fail=(), stall_ms: int = 300, timeout_ms: int = 100):
    """The engine pool's dispatcher over fake host workers (no GPU): workers in
    `stall` answer after stall_ms, those in `fail` raise a device error.
    Returns (owner per item, value per item); every value is item * 10."""
    owner = (C.c_int * max(items, 1))()
    values = (C.c_int * max(items, 1))()
    stall_mask = sum(1 << w for w in stall)
    fail_mask = sum(1 << w for w in fail)
    _check(library().ppocr_selftest_dispatch(workers, items, stall_mask, fail_mask, stall_ms, timeout_ms, owner,
                                             values))
    return list(owner)[:items], list(values)[:items]
