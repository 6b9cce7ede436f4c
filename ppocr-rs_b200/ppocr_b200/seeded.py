"""Seeded random-init checkpoints and synthetic inputs for the benchmark configs.

The real PP-OCRv6 weights are downloaded from Hugging Face by the reference
(src/models.rs:200-222); with no network the benchmark runs on random-init
weights in the exact reference tensor layout.  Two weight profiles exist:

``spec``    the distributions the benchmark configs state:
            detector conv N(0, sqrt(2/fan_in)); recognizer conv/linear N(0, 0.02);
            batch norm gamma=1, beta=0, mean=0, var=1; layer norm weight 1,
            bias 0; every conv / linear bias 0.
``conditioned``
            variance-preserving conv / linear init N(0, sqrt(1/fan_in)) with
            non-trivial biases N(0, 0.05), batch-norm gamma U(0.5, 1),
            beta / mean N(0, 0.05), var U(0.8, 1.25) and layer-norm weight
            U(0.8, 1.2).  Activations stay O(1) through the network, like a
            trained model's; every fused term of a kernel (bias, folded scale,
            residual) is non-zero.  The ``spec`` detector is numerically
            chaotic (FP32 reassociation alone moves its probability map by
            ~6e-2), so reduced-precision modes are judged on this profile.

Each tensor draws from its own generator seeded by (seed, crc32(name)), so a
tensor's values do not depend on the order tensors are generated in.
"""

from __future__ import annotations

import math
import zlib
from typing import Dict

import numpy as np

from . import modelspec


def _rng(seed: int, name: str) -> np.random.Generator:
    return np.random.default_rng([int(seed) & 0xFFFFFFFF, zlib.crc32(name.encode())])


def _draw(kind: str, name: str, shape, role: str, fan_in: int, seed: int, profile: str) -> np.ndarray:
    rng = _rng(seed, name)
    cond = profile == "conditioned"
    if role == "conv":
        if cond:
            std = math.sqrt(1.0 / max(fan_in, 1))
        elif kind == "det":
            std = math.sqrt(2.0 / max(fan_in, 1))
        else:
            std = 0.02
        return rng.normal(0.0, std, size=shape).astype(np.float32)
    if role == "rank1":
        # Medium-detector neck 9x9 kernels: w[o, i] = p[o, i] * d[i] with |d[i]| = 1,
        # the only form the reference's rank-one factorisation accepts
        # (src/cpu/model.rs:221-369).
        out_c, in_c, kh, kw = shape
        d = rng.normal(0.0, 1.0, size=(in_c, kh * kw))
        d /= np.linalg.norm(d, axis=1, keepdims=True)
        std = math.sqrt((1.0 if cond else 2.0) / fan_in) * math.sqrt(kh * kw)
        p = rng.normal(0.0, std, size=(out_c, in_c))
        w = p[:, :, None] * d[None, :, :]
        return w.reshape(shape).astype(np.float32)
    if role == "bias":
        return (rng.normal(0.0, 0.05, size=shape) if cond else np.zeros(shape)).astype(np.float32)
    if role == "bn.gamma":
        return (rng.uniform(0.5, 1.0, size=shape) if cond else np.ones(shape)).astype(np.float32)
    if role == "bn.beta":
        return (rng.normal(0.0, 0.05, size=shape) if cond else np.zeros(shape)).astype(np.float32)
    if role == "bn.mean":
        return (rng.normal(0.0, 0.05, size=shape) if cond else np.zeros(shape)).astype(np.float32)
    if role == "bn.var":
        return (rng.uniform(0.8, 1.25, size=shape) if cond else np.ones(shape)).astype(np.float32)
    if role == "ln.weight":
        return (rng.uniform(0.8, 1.2, size=shape) if cond else np.ones(shape)).astype(np.float32)
    if role == "ln.bias":
        return (rng.normal(0.0, 0.05, size=shape) if cond else np.zeros(shape)).astype(np.float32)
    raise ValueError(f"unknown role {role}")


def make_weights(kind: str, size: str, seed: int = 0, profile: str = "spec") -> Dict[str, np.ndarray]:
    """Random-init tensors for one model in the reference's checkpoint layout."""
    if profile not in ("spec", "conditioned"):
        raise ValueError(f"unknown weight profile {profile!r}")
    inv = modelspec.inventory(kind, size)
    return {
        name: _draw(kind, name, shape, role, fan_in, seed, profile)
        for name, (shape, role, fan_in) in inv.items()
    }


def write_weights(path: str, kind: str, size: str, seed: int = 0, profile: str = "spec") -> str:
    from safetensors.numpy import save_file

    save_file(make_weights(kind, size, seed, profile), str(path))
    return str(path)


# ---------------------------------------------------------------------------
# Synthetic inputs (benchmark configs 1-5)
# ---------------------------------------------------------------------------

DET_MEAN_BGR = (0.485, 0.456, 0.406)
DET_STD_BGR = (0.229, 0.224, 0.225)


def uniform_rgb8(height: int, width: int, seed: int) -> np.ndarray:
    """Seeded uniform RGB8 pixels [H, W, 3]."""
    return np.random.default_rng(seed).integers(0, 256, size=(height, width, 3), dtype=np.uint8)


def text_page_rgb8(height: int, width: int, seed: int, blocks=(20, 60), block_h=(12, 48),
                   block_w=(40, 600), max_angle=30.0, background=None) -> np.ndarray:
    """Noise background with dark filled (optionally rotated) rectangles [H, W, 3].

    Configs 3 and 5 describe pages of dark text-like strokes on a noisy
    background; this draws them with an inside-rectangle test per pixel.
    """
    rng = np.random.default_rng(seed)
    if background is None:
        img = rng.integers(0, 256, size=(height, width, 3), dtype=np.int32)
    else:
        lo, hi = background
        img = rng.integers(lo, hi, size=(height, width, 3), dtype=np.int32)
    count = int(rng.integers(blocks[0], blocks[1] + 1))
    ys, xs = np.mgrid[0:height, 0:width].astype(np.float32)
    for _ in range(count):
        bh = float(rng.integers(block_h[0], block_h[1] + 1))
        bw = float(rng.integers(block_w[0], min(block_w[1], width - 1) + 1))
        cx = float(rng.uniform(0, width))
        cy = float(rng.uniform(0, height))
        angle = 0.0 if rng.random() < 0.5 else float(rng.uniform(-max_angle, max_angle))
        t = math.radians(angle)
        c, s = math.cos(t), math.sin(t)
        x0 = max(int(cx - bw), 0)
        x1 = min(int(cx + bw) + 1, width)
        y0 = max(int(cy - bw), 0)
        y1 = min(int(cy + bw) + 1, height)
        if x0 >= x1 or y0 >= y1:
            continue
        dx = xs[y0:y1, x0:x1] - cx
        dy = ys[y0:y1, x0:x1] - cy
        u = dx * c + dy * s
        v = -dx * s + dy * c
        mask = (np.abs(u) <= bw / 2) & (np.abs(v) <= bh / 2)
        shade = int(rng.integers(0, 60))
        region = img[y0:y1, x0:x1]
        region[mask] = shade
    return img.astype(np.uint8)


def det_input_from_rgb(rgb: np.ndarray) -> np.ndarray:
    """Same-size detector normalisation of RGB8 [H, W, 3] -> NCHW float32 [1, 3, H, W] in BGR order."""
    bgr = rgb[:, :, ::-1].astype(np.float32) / 255.0
    out = np.empty((3,) + rgb.shape[:2], dtype=np.float32)
    for ch in range(3):
        out[ch] = (bgr[:, :, ch] - DET_MEAN_BGR[ch]) / DET_STD_BGR[ch]
    return out[None]


def det_batch(batch: int, height: int, width: int, seed: int, text: bool = False) -> np.ndarray:
    """Config 1 (uniform pixels) or config 3 (text-like pages) as an NCHW float32 batch."""
    out = np.empty((batch, 3, height, width), dtype=np.float32)
    for i in range(batch):
        rgb = (text_page_rgb8(height, width, seed * 7919 + i) if text
               else uniform_rgb8(height, width, seed * 7919 + i))
        out[i] = det_input_from_rgb(rgb)[0]
    return out


def rec_crop(width: int, canvas_width: int, seed: int) -> np.ndarray:
    """Config 2/4 recognizer input: a 48 x width uniform crop, right zero-padded to canvas_width.

    Returns NCHW float32 [1, 3, 48, canvas_width] normalised as (x/255 - 0.5)/0.5 in BGR order.
    """
    rgb = uniform_rgb8(48, width, seed)
    bgr = rgb[:, :, ::-1].astype(np.float32) / 255.0
    out = np.zeros((1, 3, 48, canvas_width), dtype=np.float32)
    out[0, :, :, :width] = ((bgr - 0.5) / 0.5).transpose(2, 0, 1)
    return out


def rec_batch(batch: int, canvas_width: int, seed: int, min_width: int = 64) -> np.ndarray:
    rng = np.random.default_rng(seed)
    out = np.empty((batch, 3, 48, canvas_width), dtype=np.float32)
    for i in range(batch):
        w = int(rng.integers(min(min_width, canvas_width), canvas_width + 1))
        out[i] = rec_crop(w, canvas_width, seed * 104729 + i)[0]
    return out


def deterministic_input(length: int) -> np.ndarray:
    """The bench CLI's generated input: an LCG in [-1, 1) (src/bin/benchmark.rs:126-134)."""
    out = np.empty(length, dtype=np.float32)
    state = 0x243F6A88
    for i in range(length):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(np.float32(state >> 8) / np.float32(0x00FFFFFF)) * np.float32(2.0) - np.float32(1.0)
    return out


def synthetic_dictionary(size: str):
    """A dictionary whose length makes classes = entries + 1 (src/ocr.rs:806-813)."""
    classes = modelspec.RECOGNIZER_CLASSES[size]
    return [f"<{i}>" for i in range(classes - 1)]
