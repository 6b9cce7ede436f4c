"""The detector head's conv_down decomposition, checked in float64 on the CPU.

conv_down is a 3x3 conv (zero padding 1) over the concatenation of the four
neck outputs nearest-upsampled by 8, 4, 2 and 1 (DetectorHead,
src/cpu/model.rs:1479-1521).  The FP32 build runs the full 3x3 conv only over
the scale-1 source and, for each upsampled source, adds one precomputed vector
per output pixel: for a pixel whose row (column) is the first, an interior or
the last of its s x s block, the nine taps reach at most 2 x 2 source pixels,
so the source's contribution is a sum of at most four matrix-vector products
with tap weights summed per class, computed at the source's resolution.  This
restates that construction (the class offsets and weight sums of
`Builder::head_down`, the class index of `cls_index`) and requires it to equal
the direct conv.
"""

import numpy as np
import pytest


def _off(a, d):
    if a == 0:
        return -1 if d < 0 else 0
    if a == 2:
        return 1 if d > 0 else 0
    return 0


def _cls_row(r, s):
    return 0 if r == 0 else 2 if r == s - 1 else 1


def _cls_index(ry, rx, s):
    a, b = _cls_row(ry, s), _cls_row(rx, s)
    return (a >> 1) * 2 + (b >> 1) if s == 2 else a * 3 + b


def _direct(srcs, scales, w, b, h, wd):
    up = np.concatenate([np.repeat(np.repeat(f, s, 0), s, 1) for f, s in zip(srcs, scales)], axis=2)
    pad = np.zeros((h + 2, wd + 2, up.shape[2]))
    pad[1:-1, 1:-1] = up
    out = np.zeros((h, wd, w.shape[0])) + b
    for ky in range(3):
        for kx in range(3):
            out += pad[ky:ky + h, kx:kx + wd] @ w[:, :, ky, kx].T
    return out


def _decomposed(srcs, scales, w, b, h, wd):
    cs = srcs[0].shape[2]
    out = np.zeros((h, wd, w.shape[0])) + b
    f1 = srcs[-1]
    p1 = np.zeros((h + 2, wd + 2, cs))
    p1[1:-1, 1:-1] = f1
    w1 = w[:, (len(srcs) - 1) * cs:]
    for ky in range(3):
        for kx in range(3):
            out += p1[ky:ky + h, kx:kx + wd] @ w1[:, :, ky, kx].T
    for k, s in enumerate(scales[:-1]):
        f, wk = srcs[k], w[:, k * cs:(k + 1) * cs]
        hs, ws = h // s, wd // s
        ncls = 4 if s == 2 else 9
        r = np.zeros((hs, ws, ncls, w.shape[0]))
        for c in range(ncls):
            ra = (c // 2) * 2 if s == 2 else c // 3
            ca = (c % 2) * 2 if s == 2 else c % 3
            slots = 0
            for oi in (-1, 0, 1):
                for oj in (-1, 0, 1):
                    taps = [(dy, dx) for dy in (-1, 0, 1) for dx in (-1, 0, 1) if _off(ra, dy) == oi and _off(ca, dx) == oj]
                    if not taps:
                        continue
                    slots += 1
                    wc = sum(wk[:, :, dy + 1, dx + 1] for dy, dx in taps)
                    pad = np.zeros((hs + 2, ws + 2, cs))
                    pad[1:-1, 1:-1] = f
                    r[:, :, c] += pad[1 + oi:1 + oi + hs, 1 + oj:1 + oj + ws] @ wc.T
            assert 1 <= slots <= 4
        ys, xs = np.arange(h), np.arange(wd)
        cls = np.array([[_cls_index(y % s, x % s, s) for x in xs] for y in ys])
        out += r[ys[:, None] // s, xs[None, :] // s, cls]
    return out


@pytest.mark.parametrize("h,wd", [(16, 24), (32, 8), (8, 8)])
def test_class_decomposition_equals_direct_conv(h, wd):
    rng = np.random.default_rng(h * 100 + wd)
    scales = [8, 4, 2, 1]
    cs, co = 4, 3
    srcs = [rng.normal(size=(h // s, wd // s, cs)) for s in scales]
    w = rng.normal(size=(co, cs * 4, 3, 3))
    b = rng.normal(size=co)
    np.testing.assert_allclose(_decomposed(srcs, scales, w, b, h, wd), _direct(srcs, scales, w, b, h, wd), rtol=0, atol=1e-11)
