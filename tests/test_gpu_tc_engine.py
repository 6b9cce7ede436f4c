"""tcgen05 engine (BF16 and three-way-split FP32 operands) against float64 references.

planes 1: operands are BF16 (the input and weights rounded to BF16 first) and
the output is rounded to BF16; planes 3: FP32 operands split into three BF16
pieces with the six leading products accumulated, which must be as accurate as
FP32 arithmetic (the bound is a few FP32 ulps of the sum of |products|).
"""

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bf16(x):
    x = np.asarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


def conv_ref(x, w, stride, pad):
    n, hi, wi, cin = x.shape
    cout, _, kh, kw = w.shape
    xp = np.zeros((n, hi + 2 * pad, wi + 2 * pad, cin), np.float64)
    xp[:, pad:pad + hi, pad:pad + wi] = x
    ho, wo = (hi + 2 * pad - kh) // stride + 1, (wi + 2 * pad - kw) // stride + 1
    out = np.zeros((n, ho, wo, cout), np.float64)
    for ky in range(kh):
        for kx in range(kw):
            patch = xp[:, ky:ky + stride * ho:stride, kx:kx + stride * wo:stride]
            out += patch @ w[:, :, ky, kx].astype(np.float64).T
    return out


def maxpool_su(x):
    # 2x2 stride-1 max pool whose bottom / right padding never wins.
    p = np.full((x.shape[0], x.shape[1] + 1, x.shape[2] + 1, x.shape[3]), -np.inf)
    p[:, :-1, :-1] = x
    return np.maximum(np.maximum(p[:, :-1, :-1], p[:, 1:, :-1]), np.maximum(p[:, :-1, 1:], p[:, 1:, 1:]))


def act_ref(v, act):
    if act == 1:
        return np.maximum(v, 0)
    if act == 3:
        return 0.5 * v * (1 + np.vectorize(math.erf)(v / math.sqrt(2)))
    return v


CASES = [
    # planes, n, hi, wi, cin, cout, k, stride, pad, second, act
    (3, 2, 20, 24, 16, 32, 3, 1, 1, 0, 0),
    (3, 1, 33, 41, 32, 64, 3, 2, 1, 0, 1),
    (3, 2, 17, 19, 64, 96, 1, 1, 0, 0, 3),      # dense rows, M not a multiple of 128
    (3, 1, 24, 32, 32, 16, 3, 1, 1, 1, 1),      # second source through the 2x2 max pool
    (3, 1, 16, 20, 32, 16, 3, 1, 1, 2, 0),      # second source through x2 upsampling
    (3, 1, 12, 16, 16, 200, 3, 1, 1, 0, 0),     # two N tiles
    (1, 2, 20, 24, 16, 32, 3, 1, 1, 0, 0),
    (1, 1, 33, 41, 32, 64, 3, 2, 1, 0, 1),
    (1, 2, 17, 19, 64, 96, 1, 1, 0, 0, 3),
    (1, 1, 24, 32, 32, 48, 3, 1, 1, 1, 1),
    (1, 1, 16, 20, 32, 16, 3, 1, 1, 2, 0),
    (1, 1, 12, 16, 16, 300, 3, 1, 1, 0, 0),
]


@pytest.mark.parametrize("planes,n,hi,wi,cin,cout,k,stride,pad,second,act", CASES)
def test_tc_engine_conv(gpu, planes, n, hi, wi, cin, cout, k, stride, pad, second, act):
    rng = np.random.default_rng(n * 100 + hi * 10 + cin + cout + planes)
    x = rng.normal(0, 1, (n, hi, wi, cin)).astype(np.float32)
    w = rng.normal(0, 1 / math.sqrt(cin * k * k), (cout, cin, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, cout).astype(np.float32)
    x2 = rng.normal(0, 1, (n, hi // 2, wi // 2, cin // 2)).astype(np.float32) if second == 2 else None
    if planes == 1:
        x, w = bf16(x), bf16(w)
        x2 = bf16(x2) if x2 is not None else None
    out, used, err = gpu.selftest_engine(planes, x, w, b, act, stride, pad, second, x2)
    assert used, "tensor-core path not taken"
    assert err == 0, f"wait expired (code {err})"
    xin = x.astype(np.float64)
    if second == 1:
        xin = np.concatenate([xin[..., :cin // 2], maxpool_su(xin[..., cin // 2:])], axis=-1)
    elif second == 2:
        up = np.repeat(np.repeat(x2.astype(np.float64), 2, axis=1), 2, axis=2)
        xin = np.concatenate([xin[..., :cin // 2], up], axis=-1)
    ref = act_ref(conv_ref(xin, w, stride, pad) + b, act)
    scale = conv_ref(np.abs(xin), np.abs(w), stride, pad) + np.abs(b)
    if planes == 3:
        tol = 4e-6 * scale + 1e-6
    else:
        tol = 1e-5 * scale + np.abs(ref) * 2.0 ** -8 + 1e-6
    bad = np.abs(out - ref) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} outside; max err {np.abs(out - ref).max():.3g}"
