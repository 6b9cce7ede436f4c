"""The FP32-class tcgen05 split GEMM (gemm_split.cu) against float64.

A and W are carried as three BF16 pieces each and the six leading products
are accumulated in FP32 in TMEM, so the result must stay within a few FP32
ulps of the sum of |products| of the float64 result (the same bound the
CUDA-core FP32 kernels meet), and close to the CUDA-core kernel's output.
Shapes cover the detector's pointwise layers (k 32..320, n 16..320), ragged
last tiles, several N tiles, the SE gate on A, the residual, and K up to
1,792 (the dominant sum split over up to six TMEM accumulators).  The
implicit-conv mode (32 input channels or a multiple of 64 per tap, stride 1 or 2, zero
padding through the TMA box) is checked the same way against a float64 conv.
"""

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _act(x, act):
    if act == 1:
        return np.maximum(x, 0)
    if act == 3:
        erf = np.vectorize(math.erf)
        return 0.5 * x * (1 + erf(x / math.sqrt(2)))
    return x


SHAPES = [
    # m, n, k, act, gated, residual, rows_per_image
    (1, 16, 16, 0, False, False, 1),
    (300, 16, 64, 0, False, False, 1),           # neck input_conv.pw: thin output
    (1000, 64, 32, 3, True, False, 250),         # stage-0 pw1, gate spanning images within a tile
    (2049, 32, 64, 0, False, True, 1),           # stage-0 pw2 with the residual, ragged last tile
    (777, 96, 48, 3, True, False, 259),          # stage-1 pw1: two N tiles
    (513, 48, 96, 0, False, True, 171),          # stage-1 pw2
    (640, 128, 64, 1, False, False, 1),
    (299, 320, 160, 3, False, False, 1),         # stage-3 pw1: five N tiles, three K blocks
    (299, 160, 320, 0, False, True, 1),          # stage-3 pw2: K = 320
    (4096, 64, 32, 0, False, False, 1),
    # K past 320: the dominant sum spread over several accumulators
    (700, 64, 576, 1, False, False, 1),          # two accumulators (5 + 4 K blocks)
    (300, 32, 1024, 3, True, False, 100),        # four
    (257, 16, 1792, 0, False, True, 1),          # six (the medium detector's longest K)
    (1000, 512, 1024, 0, True, True, 500),       # the medium detector's stage-2 pw2 shape: 16 N tiles, gated
]


@pytest.mark.parametrize("m,n,k,act,gated,res,rpi", SHAPES)
def test_split_gemm_fp32_class(gpu, m, n, k, act, gated, res, rpi):
    rng = np.random.default_rng(m * 5 + n * 3 + k)
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = rng.normal(0, 1 / np.sqrt(k), (n, k)).astype(np.float32)
    b = rng.normal(0, 0.1, n).astype(np.float32)
    g = rng.uniform(0, 1, (m // rpi, k)).astype(np.float32) if gated else None
    r = rng.normal(0, 1, (m, n)).astype(np.float32) if res else None
    c, used = gpu.selftest_gemm_f32(a, w, b, act, g, rpi, r, kernel=4)
    assert used == 4
    ag = a.astype(np.float64)
    if gated:
        ag = (a * np.repeat(g, rpi, axis=0)).astype(np.float64)   # the kernel gates in FP32
    pre = ag @ w.astype(np.float64).T + b
    ref = _act(pre, act)
    if res:
        ref = ref + r
    mag = np.abs(ag) @ np.abs(w.astype(np.float64)).T + np.abs(b)
    bound = 16 * 2.0 ** -24 * mag + (2.0 ** -24 * np.abs(r) if res else 0) + 1e-30
    err = np.abs(c - ref)
    assert np.all(err <= bound * 1.5 + 1e-6 * (act == 3)), f"worst {float((err / bound).max()):.2f}x the bound"
    # A pre-split into its pieces by its own kernel: the same products, bit for bit.
    c5, used5 = gpu.selftest_gemm_f32(a, w, b, act, g, rpi, r, kernel=5)
    assert used5 == 5
    np.testing.assert_array_equal(c5, c)
    # Close to the CUDA-core FP32 kernel on the same inputs.
    c2, _ = gpu.selftest_gemm_f32(a, w, b, act, g, rpi, r, kernel=1)
    assert np.abs(c - c2).max() <= 1e-4 * max(1.0, float(np.abs(c2).max()))



def _conv_ref(x, w, b, stride, pad):
    n, hi, wi, cin = x.shape
    cout, _, kh, kw = w.shape
    ho, wo = (hi + 2 * pad - kh) // stride + 1, (wi + 2 * pad - kw) // stride + 1
    xp = np.zeros((n, hi + 2 * pad, wi + 2 * pad, cin), np.float64)
    xp[:, pad:pad + hi, pad:pad + wi] = x
    out = np.zeros((n, ho, wo, cout), np.float64)
    mag = np.zeros_like(out)
    wd = w.astype(np.float64)
    for ky in range(kh):
        for kx in range(kw):
            patch = xp[:, ky:ky + stride * (ho - 1) + 1:stride, kx:kx + stride * (wo - 1) + 1:stride]
            out += patch @ wd[:, :, ky, kx].T
            mag += np.abs(patch) @ np.abs(wd[:, :, ky, kx]).T
    return out + b, mag + np.abs(b)


CONVS = [
    # n, hi, wi, cin, cout, k, stride, pad, act
    (2, 33, 70, 32, 16, 3, 2, 1, 1),     # stem3: 32 channels, stride 2, ragged tiles
    (2, 24, 40, 64, 16, 3, 1, 1, 1),     # head.conv_down: 64 channels, K = 576, two accumulators
    (1, 17, 35, 64, 48, 3, 1, 1, 0),
    (3, 9, 20, 32, 64, 3, 1, 1, 0),
    (2, 21, 38, 128, 64, 3, 2, 1, 1),    # the medium stem3: 128 channels (two K blocks per tap), K = 1,152
    (2, 27, 46, 48, 24, 3, 2, 1, 1),     # the small stem3: 48 channels, each tap zero-padded to 64
    (1, 12, 30, 96, 32, 3, 1, 1, 0),     # 96 channels: a tap's second K block half padding
    (1, 14, 22, 36, 16, 2, 1, 0, 1),     # 36 channels, 2 x 2 kernel
]


@pytest.mark.parametrize("n,hi,wi,cin,cout,k,stride,pad,act", CONVS)
def test_split_conv_fp32_class(gpu, n, hi, wi, cin, cout, k, stride, pad, act):
    rng = np.random.default_rng(hi * 7 + wi + cin + cout)
    x = rng.normal(0, 1, (n, hi, wi, cin)).astype(np.float32)
    w = rng.normal(0, 1 / np.sqrt(cin * k * k), (cout, cin, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, cout).astype(np.float32)
    got = gpu.selftest_conv_split(x, w, b, stride=stride, pad=pad, act=act)
    pre, mag = _conv_ref(x.astype(np.float64), w, b.astype(np.float64), stride, pad)
    ref = _act(pre, act)
    bound = 16 * 2.0 ** -24 * mag + 1e-30
    err = np.abs(got - ref)
    assert np.all(err <= bound * 1.5), f"worst {float((err / bound).max()):.2f}x the bound"


@pytest.mark.parametrize("n,hi,wi,cin,cout,stride,act", [
    (2, 26, 46, 64, 64, 2, 0),    # the medium neck's bottom-up 3x3 s2 conv + the projection residual
    (1, 19, 37, 48, 24, 1, 1),    # padded taps, ragged tiles, ReLU before the residual
])
def test_split_conv_residual(gpu, n, hi, wi, cin, cout, stride, act):
    rng = np.random.default_rng(hi + wi * 3 + cin + cout)
    x = rng.normal(0, 1, (n, hi, wi, cin)).astype(np.float32)
    w = rng.normal(0, 1 / np.sqrt(cin * 9), (cout, cin, 3, 3)).astype(np.float32)
    b = rng.normal(0, 0.1, cout).astype(np.float32)
    ho, wo = (hi + 2 - 3) // stride + 1, (wi + 2 - 3) // stride + 1
    r = rng.normal(0, 1, (n, ho, wo, cout)).astype(np.float32)
    got = gpu.selftest_conv_split(x, w, b, stride=stride, pad=1, act=act, residual=r)
    pre, mag = _conv_ref(x.astype(np.float64), w, b.astype(np.float64), stride, 1)
    ref = _act(pre, act) + r
    bound = 16 * 2.0 ** -24 * mag + 2.0 ** -24 * np.abs(ref) + 1e-30
    err = np.abs(got - ref)
    assert np.all(err <= bound * 1.5), f"worst {float((err / bound).max()):.2f}x the bound"
    # The residual is added after the activation, once: without it the output differs by r.
    plain = gpu.selftest_conv_split(x, w, b, stride=stride, pad=1, act=act)
    np.testing.assert_array_equal(got, (plain + r).astype(np.float32))


def test_split_conv_rejects_other_channel_counts(gpu):
    import ppocr_b200 as P

    for cin in (16, 34):   # below 32; not a multiple of 4
        x = np.zeros((1, 8, 8, cin), np.float32)
        w = np.zeros((16, cin, 3, 3), np.float32)
        with pytest.raises(P.InvalidInput):
            gpu.selftest_conv_split(x, w)
