"""Depthwise conv kernels against each other and float64.

The rolling-row kernel (3x3, 5x5) and the tiled kernel sum each output's taps in
(ky, kx) order with the same packed FMAs and apply bias, activation and
residual in the same order, so on the same inputs they must agree bit for
bit.  Both must stay within a few FP32 ulps of the float64 result (scaled by
the sum of |products|); in the BF16 mode the inputs are the BF16-rounded
values and the output carries one BF16 rounding.
"""

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _act(x, act):
    if act == 1:
        return np.maximum(x, 0)
    if act == 2:
        return x / (1 + np.exp(-x))
    if act == 3:
        erf = np.vectorize(math.erf)
        return 0.5 * x * (1 + erf(x / math.sqrt(2)))
    if act == 4:
        return x * np.clip(x + 3, 0, 6) / 6
    if act == 5:
        return 1 / (1 + np.exp(-x))
    return x


def _bf16(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


def _reference(x, w, bias, stride, pad, act, residual):
    """float64 depthwise conv; also returns the sum of |products| per output."""
    n, hi, wi, c = x.shape
    kh, kw = w.shape[1:]
    sh, sw = stride
    pt, pl, pb, pr = pad
    ho, wo = (hi + pt + pb - kh) // sh + 1, (wi + pl + pr - kw) // sw + 1
    xp = np.zeros((n, hi + pt + pb, wi + pl + pr, c))
    xp[:, pt:pt + hi, pl:pl + wi] = x
    acc = np.zeros((n, ho, wo, c))
    mag = np.zeros((n, ho, wo, c))
    for ky in range(kh):
        for kx in range(kw):
            win = xp[:, ky:ky + sh * (ho - 1) + 1:sh, kx:kx + sw * (wo - 1) + 1:sw]
            acc += win * w[:, ky, kx]
            mag += np.abs(win * w[:, ky, kx])
    if bias is not None:
        acc += bias
        mag += np.abs(bias)
    out = _act(acc, act)
    if residual is not None:
        out = out + residual
        mag = mag + np.abs(residual)
    return out, mag


CASES = [
    # n, hi, wi, c, k, stride, pad, act, bias, residual
    (2, 12, 80, 64, 3, (1, 1), (1, 1, 1, 1), 0, True, False),     # recognizer token conv shape (one band)
    (1, 104, 184, 32, 3, (1, 1), (1, 1, 1, 1), 0, True, False),   # detector stage 1: two bands, row segments
    (3, 13, 23, 256, 3, (1, 1), (1, 1, 1, 1), 4, True, True),     # odd extents, several channel groups
    (2, 26, 46, 64, 3, (2, 2), (1, 1, 1, 1), 0, False, False),    # stride 2
    (2, 12, 80, 128, 3, (2, 1), (1, 1, 1, 1), 2, True, False),    # recognizer (2, 1) stride
    (1, 3, 80, 48, 3, (1, 1), (1, 1, 1, 1), 0, True, True),       # three-row map: the short ring
    (2, 9, 130, 16, 3, (1, 1), (1, 1, 1, 1), 1, True, False),     # 16 channels, 33 runs over two bands
    (1, 7, 9, 8, 3, (2, 2), (1, 1, 1, 1), 5, True, False),        # tiny map, one channel group of two quads
    (2, 20, 36, 4, 3, (1, 1), (1, 1, 1, 1), 3, True, True),       # one channel quad
    (1, 14, 30, 24, 5, (1, 1), (2, 2, 2, 2), 0, True, False),     # 5x5: RepLkFpn depthwise
    (2, 52, 92, 64, 5, (1, 1), (2, 2, 2, 2), 0, True, False),     # 5x5 detector neck shape, two bands, segments
    (1, 9, 40, 32, 5, (1, 1), (2, 2, 2, 2), 4, False, True),      # 5x5 with activation and residual
    (1, 12, 30, 16, 7, (1, 1), (3, 3, 3, 3), 0, True, False),     # 7x7 (tiled kernel only)
    (1, 3, 40, 32, (1, 7), (1, 1), (0, 3, 0, 3), 2, True, True),  # SVTR 1x7 + SiLU + residual (tiled)
]


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("n,hi,wi,c,k,stride,pad,act,has_bias,has_res", CASES)
def test_dwconv_kernels(gpu, n, hi, wi, c, k, stride, pad, act, has_bias, has_res, bf16):
    if bf16 and c % 8:
        pytest.skip("BF16 views need 8-channel alignment")
    kh, kw = (k, k) if isinstance(k, int) else k
    band = (kh, kw) in ((3, 3), (5, 5))
    rng = np.random.default_rng(n * 1000 + hi * 37 + wi * 11 + c + kh)
    x = rng.normal(0, 1, (n, hi, wi, c)).astype(np.float32)
    w = rng.normal(0, 1 / math.sqrt(kh * kw), (c, kh, kw)).astype(np.float32)
    b = rng.normal(0, 0.1, c).astype(np.float32) if has_bias else None
    ho = (hi + pad[0] + pad[2] - kh) // stride[0] + 1
    wo = (wi + pad[1] + pad[3] - kw) // stride[1] + 1
    r = rng.normal(0, 1, (n, ho, wo, c)).astype(np.float32) if has_res else None
    outs = {}
    for kernel in (1, 2):
        try:
            out, used = gpu.selftest_dwconv(x, w, b, stride, pad, act, r, bf16, kernel)
        except Exception as e:  # the rolling-row kernel covers 3x3 and 5x5
            assert "does not support" in str(e) and not band, e
            continue
        assert used == kernel
        outs[kernel] = out
    assert 1 in outs and (not band or 2 in outs)
    xs = _bf16(x) if bf16 else x
    rs = (_bf16(r) if bf16 else r) if r is not None else None
    ref, mag = _reference(xs.astype(np.float64), w.astype(np.float64), b, stride, pad, act, rs)
    tol = 4e-6 * mag + 1e-6
    if bf16:
        tol = tol + 2.0 ** -8 * np.abs(ref) + 1e-30
    for kernel, out in outs.items():
        err = np.abs(out - ref)
        assert np.all(err <= tol), f"kernel {kernel}: max err {err.max()} (bf16={bf16})"
    if 2 in outs:
        np.testing.assert_array_equal(outs[2], outs[1], err_msg="rolling-row kernel differs from the tiled kernel")
    _, used = gpu.selftest_dwconv(x, w, b, stride, pad, act, r, bf16, 0)
    assert used == (2 if (kh, kw) == (3, 3) else 1)
