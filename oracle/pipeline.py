"""CPU oracle for the end-to-end pipeline's host steps -- TEST INFRASTRUCTURE ONLY.

Restates, in single precision where the reference computes in f32, the parts
of ppocr-rs src/ocr.rs that run around the two models:

* DB postprocess ``extract_detections`` (src/ocr.rs:723-782): raster scan of
  the content area, 8-connected breadth-first components of pixels with
  prob >= binary_threshold (``collect_component``, 993-1043), min_area and
  mean-score filters, ``fit_rotated_box`` (1045-1113: covariance angle,
  extent along the axis and its normal, unclip), mapping to source
  coordinates (DetectorTransform, 59-71), ``sort_detections`` (1115-1126)
  and the max_boxes cut;
* recognition planning: ``polygon_aspect_ratio``, ``bounded_crop_dimensions``
  (1134-1156), ``recognition_input_plan`` (154-172), ``recognizer_batch_width``
  (206-219) and the aspect-ratio order and chunks of six of ``recognize_with``
  (573-621);
* text assembly: ``parse_dictionary`` / ``parse_paddlex_character_dict`` /
  ``parse_yaml_scalar`` (892-965), ``append_with_overlap`` (1179-1196) and
  ``join_decoded_texts`` (702-721).

Every f32 operation is rounded to f32 in the reference's order (numpy float32
scalars, no fused multiply-add); sin, cos and atan2 are glibc's single
precision functions, which is what the reference's f32 methods call on Linux.
"""

from __future__ import annotations

import ctypes
import ctypes.util
import math
from collections import deque
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import preprocess as opre

F = np.float32
EPS = F(np.finfo(np.float32).eps)
RECOGNIZER_BATCH_SIZE = 6
MAX_RECTIFIED_EDGE = F(4096.0)
MAX_RECTIFIED_PIXELS = F(8_000_000.0)

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
for _name in ("cosf", "sinf"):
    getattr(_libm, _name).restype = ctypes.c_float
    getattr(_libm, _name).argtypes = [ctypes.c_float]
_libm.atan2f.restype = ctypes.c_float
_libm.atan2f.argtypes = [ctypes.c_float, ctypes.c_float]


def cosf(x) -> F:
    return F(_libm.cosf(float(x)))


def sinf(x) -> F:
    return F(_libm.sinf(float(x)))


def atan2f(y, x) -> F:
    return F(_libm.atan2f(float(y), float(x)))


@dataclass
class PostprocessOptions:
    """DetectorPostprocessOptions and its defaults (src/ocr.rs:231-271)."""

    binary_threshold: float = 0.2
    box_threshold: float = 0.4
    min_area: int = 3
    unclip_ratio: float = 1.4
    max_boxes: int = 1000

    def validate(self) -> None:
        for v, name in ((self.binary_threshold, "detector binary threshold"),
                        (self.box_threshold, "detector box threshold")):
            if not math.isfinite(v) or not 0.0 <= v <= 1.0:
                raise ValueError(f"{name} must be a finite value between zero and one")
        if self.min_area == 0:
            raise ValueError("detector minimum area must be at least one pixel")
        if self.max_boxes == 0:
            raise ValueError("detector maximum box count must be at least one")
        if not math.isfinite(self.unclip_ratio) or self.unclip_ratio <= 0:
            raise ValueError("detector unclip ratio must be a finite value greater than zero")


@dataclass
class Detection:
    polygon: List[Tuple[F, F]]
    score: F


def _total_key(v) -> int:
    """Integer key ordering f32 values like Rust's f32::total_cmp."""
    b = int(np.float32(v).view(np.int32))
    return b ^ 0x7FFFFFFF if b < 0 else b


def _sum_f32(values) -> F:
    s = F(-0.0)
    for v in values:
        s = F(s + v)
    return s


def polygon_center(poly) -> Tuple[F, F]:
    return (F(_sum_f32(p[0] for p in poly) / F(4.0)), F(_sum_f32(p[1] for p in poly) / F(4.0)))


def distance(a, b) -> F:
    dx = F(a[0] - b[0])
    dy = F(a[1] - b[1])
    return F(np.sqrt(F(F(dx * dx) + F(dy * dy))))


def collect_component(values: np.ndarray, out_w: int, cw: int, ch: int, sx: int, sy: int, thr: F,
                      visited: np.ndarray):
    """Breadth-first 8-connected component (src/ocr.rs:993-1043): points in pop order, f64 score sum."""
    neighbors = ((-1, -1), (0, -1), (1, -1), (-1, 0), (1, 0), (-1, 1), (0, 1), (1, 1))
    queue = deque([(sx, sy)])
    visited[sy * cw + sx] = True
    points, score_sum = [], 0.0
    while queue:
        x, y = queue.popleft()
        points.append((F(F(x) + F(0.5)), F(F(y) + F(0.5))))
        score_sum += float(values[y * out_w + x])
        for ox, oy in neighbors:
            nx, ny = x + ox, y + oy
            if nx < 0 or ny < 0 or nx >= cw or ny >= ch:
                continue
            ni = ny * cw + nx
            if not visited[ni] and values[ny * out_w + nx] >= thr:
                visited[ni] = True
                queue.append((nx, ny))
    return points, score_sum


def fit_rotated_box(points, unclip_ratio) -> List[Tuple[F, F]]:
    """src/ocr.rs:1045-1113 in f32."""
    count = F(len(points))
    cx = F(_sum_f32(p[0] for p in points) / count)
    cy = F(_sum_f32(p[1] for p in points) / count)
    cxx = cxy = cyy = F(0.0)
    for px, py in points:
        dx = F(px - cx)
        dy = F(py - cy)
        cxx = F(cxx + F(dx * dx))
        cxy = F(cxy + F(dx * dy))
        cyy = F(cyy + F(dy * dy))
    angle = F(F(0.5) * atan2f(F(F(2.0) * cxy), F(cxx - cyy)))
    ax, ay = cosf(angle), sinf(angle)
    if ax < 0 or (abs(ax) < EPS and ay < 0):
        ax, ay = F(-ax), F(-ay)
    nx, ny = F(-ay), ax
    min_a, max_a = F(np.inf), F(-np.inf)
    min_n, max_n = F(np.inf), F(-np.inf)
    for px, py in points:
        dx = F(px - cx)
        dy = F(py - cy)
        along_a = F(F(dx * ax) + F(dy * ay))
        along_n = F(F(dx * nx) + F(dy * ny))
        min_a, max_a = min(min_a, along_a), max(max_a, along_a)
        min_n, max_n = min(min_n, along_n), max(max_n, along_n)
    u = F(unclip_ratio)
    axis_center = F(F(min_a + max_a) * F(0.5))
    normal_center = F(F(min_n + max_n) * F(0.5))
    half_a = F(F(F(F(max_a - min_a) + F(1.0)) * u) * F(0.5))
    half_n = F(F(F(F(max_n - min_n) + F(1.0)) * u) * F(0.5))
    # center + (axis * axis_center + normal * normal_center)
    ox = F(F(ax * axis_center) + F(nx * normal_center))
    oy = F(F(ay * axis_center) + F(ny * normal_center))
    cx, cy = F(cx + ox), F(cy + oy)

    def corner(sa, sn):
        px = F(F(ax * F(sa * half_a)) + F(nx * F(sn * half_n)))
        py = F(F(ay * F(sa * half_a)) + F(ny * F(sn * half_n)))
        return (F(cx + px), F(cy + py))

    return [corner(-1, -1), corner(1, -1), corner(1, 1), corner(-1, 1)]


def _map(v, source: int, content: int) -> F:
    m = F(F(v * F(source)) / F(content))
    return F(min(max(m, F(0.0)), F(source)))


def _sort_detections(dets: List[Detection]) -> None:
    def key(d):
        c = polygon_center(d.polygon)
        return (_total_key(c[1]), _total_key(c[0]), _total_key(d.score))
    dets.sort(key=key)


def extract_detections(values: np.ndarray, height: int, width: int, source_size: Tuple[int, int],
                       content_size: Tuple[int, int], options: PostprocessOptions = PostprocessOptions()
                       ) -> List[Detection]:
    """extract_detections (src/ocr.rs:723-782) over a [height, width] probability map."""
    options.validate()
    values = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    if values.size != height * width:
        raise ValueError("detector output size does not match its shape")
    if not np.all(np.isfinite(values)):
        raise ValueError("detector output contains non-finite values")
    sw, sh = source_size
    cw = min(content_size[0], width)
    ch = min(content_size[1], height)
    thr = F(options.binary_threshold)
    visited = np.zeros(cw * ch, dtype=bool)
    dets: List[Detection] = []
    for y in range(ch):
        row = values[y * width:y * width + cw]
        for x in np.nonzero(row >= thr)[0]:
            x = int(x)
            if visited[y * cw + x]:
                continue
            points, score_sum = collect_component(values, width, cw, ch, x, y, thr, visited)
            if len(points) < options.min_area:
                continue
            score = F(score_sum / len(points))
            if score < F(options.box_threshold):
                continue
            poly = [(_map(px, sw, content_size[0]), _map(py, sh, content_size[1]))
                    for px, py in fit_rotated_box(points, options.unclip_ratio)]
            dets.append(Detection(poly, score))
    _sort_detections(dets)
    if len(dets) > options.max_boxes:
        def key(d):
            c = polygon_center(d.polygon)
            return (-_total_key(d.score), _total_key(c[1]), _total_key(c[0]))
        dets.sort(key=key)
        del dets[options.max_boxes:]
        _sort_detections(dets)
    return dets


# ---------------------------------------------------------------------------
# Recognition planning (src/ocr.rs:154-219, 573-621, 1128-1156)
# ---------------------------------------------------------------------------

def polygon_aspect_ratio(poly) -> F:
    w = max(distance(poly[0], poly[1]), distance(poly[3], poly[2]))
    h = max(distance(poly[0], poly[3]), distance(poly[1], poly[2]))
    return F(w / max(h, EPS))


def _round_half_away_f32(v: F) -> F:
    return F(math.floor(float(v) + 0.5)) if v >= 0 else F(-math.floor(-float(v) + 0.5))


def bounded_crop_dimensions(width: F, height: F) -> Tuple[int, int]:
    if not (math.isfinite(width) and math.isfinite(height)) or width <= 0 or height <= 0:
        raise ValueError(f"text polygon has an invalid crop size {width} by {height}")
    edge = min(F(MAX_RECTIFIED_EDGE / max(width, height)), F(1.0))
    pixel = min(F(np.sqrt(F(MAX_RECTIFIED_PIXELS / F(width * height)))), F(1.0))
    s = min(edge, pixel)
    w = min(max(_round_half_away_f32(F(width * s)), F(1.0)), MAX_RECTIFIED_EDGE)
    h = min(max(_round_half_away_f32(F(height * s)), F(1.0)), MAX_RECTIFIED_EDGE)
    return int(w), int(h)


def crop_content_width(poly) -> int:
    w = max(distance(poly[0], poly[1]), distance(poly[3], poly[2]))
    h = max(distance(poly[0], poly[3]), distance(poly[1], poly[2]))
    bw, bh = bounded_crop_dimensions(w, h)
    return opre.scaled_recognizer_width(bw, bh)


def batch_width(polys) -> int:
    return opre.recognizer_batch_width([crop_content_width(p) for p in polys])


def recognition_batches(dets: List[Detection]) -> List[Tuple[List[int], int, List[int]]]:
    """Aspect-ratio order in chunks of six: [(detection indices, canvas width, content widths)]."""
    order = sorted(range(len(dets)), key=lambda i: _total_key(polygon_aspect_ratio(dets[i].polygon)))
    out = []
    for s in range(0, len(order), RECOGNIZER_BATCH_SIZE):
        idx = order[s:s + RECOGNIZER_BATCH_SIZE]
        polys = [dets[i].polygon for i in idx]
        w = batch_width(polys)
        contents = [crop_content_width(p) for p in polys]
        if any(c > w for c in contents):
            raise ValueError("recognizer crop exceeds its batch canvas")
        out.append((idx, w, contents))
    return out


# ---------------------------------------------------------------------------
# Text assembly (src/ocr.rs:702-721, 892-965, 1179-1196)
# ---------------------------------------------------------------------------

def _parse_yaml_scalar(value: str, line: int) -> str:
    if value.startswith("'"):
        if len(value) < 2 or not value.endswith("'"):
            raise ValueError(f"unterminated single-quoted character on line {line}")
        return value[1:-1].replace("''", "'")
    if value.startswith('"'):
        if len(value) < 2 or not value.endswith('"'):
            raise ValueError(f"unterminated double-quoted character on line {line}")
        return value[1:-1]
    return value


def _rust_lines(contents: str) -> List[str]:
    """str::lines: split on \\n, strip one trailing \\r per line, no final empty line."""
    if contents == "":
        return []
    parts = contents.split("\n")
    if parts[-1] == "":
        parts.pop()
    return [p[:-1] if p.endswith("\r") else p for p in parts]


def _paddlex_dict(contents: str) -> Optional[List[str]]:
    lines = contents.split("\n")
    if lines and lines[-1] == "":
        lines.pop()
    for index, line in enumerate(lines):
        lt = line[:-1] if line.endswith("\r") else line
        if lt.strip() != "character_dict:":
            continue
        indentation = len(line) - len(line.lstrip())
        entries = []
        for offset, entry_line in enumerate(lines[index + 1:]):
            entry_line = entry_line[:-1] if entry_line.endswith("\r") else entry_line
            if entry_line.strip() == "":
                continue
            trimmed = entry_line.lstrip()
            if not trimmed.startswith("- "):
                if len(entry_line) - len(trimmed) <= indentation:
                    break
                raise ValueError(f"expected a character list entry on line {index + offset + 2}")
            entries.append(_parse_yaml_scalar(trimmed[2:], index + offset + 2))
        return entries
    return None


def parse_dictionary(contents: str) -> List[str]:
    entries = _paddlex_dict(contents)
    if entries is None:
        entries = _rust_lines(contents)
    if entries:
        entries[0] = entries[0].lstrip("\ufeff")
    if not entries:
        raise ValueError("recognition dictionary is empty")
    for i, e in enumerate(entries):
        if e == "":
            raise ValueError(f"recognition dictionary contains an empty entry on line {i + 1}")
    return entries


def append_with_overlap(target: str, nxt: str) -> Tuple[str, int]:
    if nxt == "":
        return target, 0
    if target == "":
        return nxt, len(nxt)
    maximum = min(len(target), len(nxt), 32)
    overlap = 0
    for size in range(maximum, 0, -1):
        if target[-size:] == nxt[:size]:
            overlap = size
            break
    return target + nxt[overlap:], len(nxt) - overlap


def join_decoded_texts(parts: Sequence[Tuple[str, float]]) -> Tuple[str, float]:
    text, score_sum, weight = "", 0.0, 0
    for t, s in parts:
        text, added = append_with_overlap(text, t)
        if added:
            score_sum += float(np.float32(s)) * added
            weight += added
    return text, float(F(score_sum / weight)) if weight else 0.0
