"""CPU oracle for the device-side DB binarisation and greedy CTC arg-max.

TEST INFRASTRUCTURE ONLY.  Restates ppocr-rs src/ocr.rs:
* DB binarisation: a pixel is text when prob >= binary_threshold (0.2 by
  default, src/ocr.rs:239-249, compared at 745 and 1047);
* greedy CTC (decode_ctc_greedy_for_input, src/ocr.rs:800-853): per step the
  arg-max class (the LAST index among equal maxima, Rust Iterator::max_by,
  src/ocr.rs:1171-1177), blank 0 and repeats skipped, only the first
  ceil(content_width * T / input_width) steps decoded, score the geometric
  mean of the emitted probabilities (row_probability, src/ocr.rs:1158-1169).
"""

from __future__ import annotations

import math
from typing import List, Sequence, Tuple

import numpy as np

PROBABILITY_EPSILON = 1e-8


def db_mask(prob: np.ndarray, threshold: float = 0.2) -> np.ndarray:
    return (np.asarray(prob, dtype=np.float32) >= np.float32(threshold)).astype(np.uint8)


def argmax_last(rows: np.ndarray) -> np.ndarray:
    """Arg-max per row with ties resolved to the highest index."""
    rows = np.asarray(rows)
    rev = rows[..., ::-1]
    return rows.shape[-1] - 1 - np.argmax(rev, axis=-1)


def top2_margin(logits: np.ndarray) -> np.ndarray:
    part = np.partition(np.asarray(logits, dtype=np.float64), -2, axis=-1)
    return (part[..., -1] - part[..., -2]).astype(np.float32)


def row_probability(row: np.ndarray, value: float) -> float:
    row = np.asarray(row, dtype=np.float32)
    s = np.float32(row.sum(dtype=np.float32))
    if np.all(row >= 0) and abs(s - 1.0) <= 0.01:
        return float(min(max(value, 0.0), 1.0))
    m = row.max()
    denom = np.exp(row - m).sum(dtype=np.float32)
    return float(min(max(np.exp(value - m) / denom, 0.0), 1.0))


def decode_ctc_greedy(probs: np.ndarray, dictionary: Sequence[str], content_width: int,
                      input_width: int) -> Tuple[str, float, List[int]]:
    """decode_ctc_greedy_for_input for one item: probs [T, classes] -> (text, score, emitted classes)."""
    probs = np.asarray(probs, dtype=np.float32)
    t, classes = probs.shape
    implicit_space = classes == len(dictionary) + 2
    if classes != len(dictionary) + 1 and not implicit_space:
        raise ValueError("recognizer output classes do not match the dictionary")
    if content_width == 0 or content_width > input_width:
        raise ValueError(f"recognizer content width {content_width} is outside 1..={input_width}")
    if not np.all(np.isfinite(probs)):
        raise ValueError("recognizer output contains non-finite values")
    valid = -(-content_width * t // input_width)
    valid = min(max(valid, 1), t)
    text, log_score, emitted, previous, cls_list = "", 0.0, 0, 0, []
    idx = argmax_last(probs[:valid])
    for step in range(valid):
        c = int(idx[step])
        if c != 0 and c != previous:
            text += " " if implicit_space and c == classes - 1 else dictionary[c - 1]
            log_score += math.log(max(row_probability(probs[step], float(probs[step, c])), PROBABILITY_EPSILON))
            emitted += 1
            cls_list.append(c)
        previous = c
    score = 0.0 if emitted == 0 else math.exp(log_score / emitted)
    return text, score, cls_list
