"""CPU oracle for device preprocessing and input planning.

TEST INFRASTRUCTURE ONLY (imported by tests/, smoke() and bench.py's CPU
baseline).  Restates, in float32 numpy:

* the scalar row kernel of ppocr-rs src/preprocess/kernels.rs:94-165 -- quad
  bilinear map sampled at pixel centres minus 0.5, edge-clamped, interpolated
  per channel and ROUNDED to an integer (half away from zero, Rust f32::round),
  BGR plane order, value * scale + bias with Normalization::new's
  scale = 1/(255 std), bias = -mean/std (kernels.rs:9-18), zero past
  content_width;
* DetectorInputPlan / recognition_input_plan geometry (src/ocr.rs:86-219).

The reference's AVX2/SSE2 bodies compute u as (x + 0.5) * (1/width) and round
via floor(v + 0.5); they agree with the scalar kernel except at exact
half-way points, and the reference's own test bounds the difference by 2e-6
(src/preprocess.rs:181-227).  The scalar form is the one restated here.
"""

from __future__ import annotations

import math
from typing import Sequence, Tuple

import numpy as np

f32 = np.float32

DETECTOR_MEAN_BGR = (0.485, 0.456, 0.406)
DETECTOR_STD_BGR = (0.229, 0.224, 0.225)
RECOGNIZER_MEAN_BGR = (0.5, 0.5, 0.5)
RECOGNIZER_STD_BGR = (0.5, 0.5, 0.5)


def normalization(mean, std) -> Tuple[np.ndarray, np.ndarray]:
    """Normalization::new (src/preprocess/kernels.rs:9-18), in f32."""
    scale = np.array([f32(1.0) / (f32(255.0) * f32(s)) for s in std], dtype=f32)
    bias = np.array([f32(-f32(m)) / f32(s) for m, s in zip(mean, std)], dtype=f32)
    return scale, bias


def _round_half_away(v: np.ndarray) -> np.ndarray:
    t = np.trunc(v)
    return (t + (np.abs(v - t) >= f32(0.5)) * np.sign(v)).astype(f32)


def normalized_bgr(rgb: np.ndarray, corners: Sequence[Sequence[float]], canvas_w: int, canvas_h: int,
                   content_w: int, mean, std) -> np.ndarray:
    """normalized_bgr (src/preprocess.rs:78-123) with the scalar row kernel; returns [1, 3, H, W] f32."""
    rgb = np.asarray(rgb, dtype=np.uint8)
    src_h, src_w = rgb.shape[:2]
    scale, bias = normalization(mean, std)
    c = np.asarray(corners, dtype=f32).reshape(4, 2)
    out = np.zeros((1, 3, canvas_h, canvas_w), dtype=f32)
    if content_w <= 0:
        return out
    xs = np.arange(content_w, dtype=f32)
    u = ((xs + f32(0.5)) / f32(content_w)).astype(f32)
    omu = (f32(1.0) - u).astype(f32)
    max_x, max_y = f32(src_w - 1), f32(src_h - 1)
    pix = rgb.astype(f32)
    for y in range(canvas_h):
        v = f32(f32(f32(y) + f32(0.5)) / f32(canvas_h))
        omv = f32(f32(1.0) - v)
        sx = ((c[0, 0] * omu + c[1, 0] * u) * omv + (c[3, 0] * omu + c[2, 0] * u) * v - f32(0.5)).astype(f32)
        sy = ((c[0, 1] * omu + c[1, 1] * u) * omv + (c[3, 1] * omu + c[2, 1] * u) * v - f32(0.5)).astype(f32)
        sx = np.clip(sx, f32(0.0), max_x).astype(f32)
        sy = np.clip(sy, f32(0.0), max_y).astype(f32)
        x0 = np.floor(sx).astype(np.int64)
        y0 = np.floor(sy).astype(np.int64)
        x1 = np.minimum(x0 + 1, src_w - 1)
        y1 = np.minimum(y0 + 1, src_h - 1)
        tx = (sx - x0.astype(f32)).astype(f32)
        ty = (sy - y0.astype(f32)).astype(f32)
        omtx = (f32(1.0) - tx).astype(f32)
        omty = (f32(1.0) - ty).astype(f32)
        vals = []
        for ch in range(3):
            tl = pix[y0, x0, ch]
            tr = pix[y0, x1, ch]
            bl = pix[y1, x0, ch]
            br = pix[y1, x1, ch]
            top = (tl * omtx + tr * tx).astype(f32)
            bottom = (bl * omtx + br * tx).astype(f32)
            val = (top * omty + bottom * ty).astype(f32)
            vals.append(np.clip(_round_half_away(val), f32(0.0), f32(255.0)))
        # plane 0 = blue (rgb[2]), 1 = green, 2 = red
        out[0, 0, y, :content_w] = (vals[2] * scale[0] + bias[0]).astype(f32)
        out[0, 1, y, :content_w] = (vals[1] * scale[1] + bias[1]).astype(f32)
        out[0, 2, y, :content_w] = (vals[0] * scale[2] + bias[2]).astype(f32)
    return out


def prepare_detector(rgb: np.ndarray, input_w: int, input_h: int) -> np.ndarray:
    """prepare_detector (src/preprocess.rs:37-47): full-image corners, ImageNet statistics."""
    h, w = rgb.shape[:2]
    corners = [(0.0, 0.0), (float(w), 0.0), (float(w), float(h)), (0.0, float(h))]
    return normalized_bgr(rgb, corners, input_w, input_h, input_w, DETECTOR_MEAN_BGR, DETECTOR_STD_BGR)


def prepare_recognizer_crop(rgb: np.ndarray, corners, canvas_w: int, content_w: int) -> np.ndarray:
    """One crop of prepare_recognizer (src/preprocess.rs:49-76): 48 rows, +-1 normalisation."""
    return normalized_bgr(rgb, corners, canvas_w, 48, content_w, RECOGNIZER_MEAN_BGR, RECOGNIZER_STD_BGR)


# ---------------------------------------------------------------------------
# Input planning (src/ocr.rs:86-219)
# ---------------------------------------------------------------------------

DETECTOR_LIMIT_SIDE = 736.0
DETECTOR_MAX_SIDE = 4000.0
RECOGNIZER_INPUT_WIDTH = 320
MAX_RECTIFIED_EDGE = 4096.0
MAX_RECTIFIED_PIXELS = 8_000_000.0


def aligned_dimension(value: float) -> int:
    """Round to the nearest multiple of 32, at least 32 (src/ocr.rs:186-195)."""
    if not math.isfinite(value) or value <= 0:
        raise ValueError(f"invalid resized image dimension {value}")
    units = max(_round_f64_half_away(value / 32.0), 1.0)
    return int(units) * 32


def _round_f64_half_away(v: float) -> float:
    return math.floor(v + 0.5) if v >= 0 else -math.floor(-v + 0.5)


def default_detector_ratio(width: int, height: int) -> float:
    min_side = float(min(width, height))
    ratio = DETECTOR_LIMIT_SIDE / min_side if min_side < DETECTOR_LIMIT_SIDE else 1.0
    if float(max(width, height)) * ratio > DETECTOR_MAX_SIDE:
        ratio = DETECTOR_MAX_SIDE / float(max(width, height))
    return ratio


def detector_input_size(width: int, height: int, max_side=None) -> Tuple[int, int]:
    """DetectorInputPlan::new (src/ocr.rs:86-101) -> (input_width, input_height)."""
    if max_side is not None:
        if max_side <= 0:
            raise ValueError("detector maximum side must be positive")
        ratio = min(float(max_side) / float(max(width, height)), 1.0)
    else:
        ratio = default_detector_ratio(width, height)
    return aligned_dimension(width * ratio), aligned_dimension(height * ratio)


def scaled_recognizer_width(width: int, height: int) -> int:
    """ceil(48 * w / h), at least 1 (src/ocr.rs:197-204)."""
    return max(-(-48 * width // height), 1)


def recognizer_batch_width(content_widths: Sequence[int]) -> int:
    """max(320, widest content) rounded up to a multiple of 4 (src/ocr.rs:206-219)."""
    m = max([RECOGNIZER_INPUT_WIDTH] + list(content_widths))
    return (m + 3) // 4 * 4
