"""FP32 pointwise GEMM kernels of the FP32 mode against each other and float64.

The three SIMT kernels (register-tiled, row-per-thread, streaming) sum each
output in k order with FMA and add bias, activation and residual in the same
order, so on the same inputs they must agree bit for bit; each must also stay
within a few FP32 ulps of the sum of |products| from the float64 result.
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


SHAPES = [
    # m, n, k, act, gated, residual, rows_per_image
    (1, 16, 16, 0, False, False, 1),
    (300, 16, 32, 4, False, False, 1),          # head-style thin output
    (1000, 32, 32, 3, True, True, 250),         # gate spanning several images per tile
    (2049, 64, 32, 0, False, True, 1),          # neck in_conv shape, ragged last tile
    (777, 48, 64, 2, True, False, 259),
    (4096, 96, 64, 3, False, False, 1),         # n between tile widths
    (513, 128, 64, 1, True, True, 171),
    (299, 128, 128, 0, False, False, 1),        # k at the streaming kernel's limit
    (640, 100, 20, 5, False, True, 1),          # n not a multiple of 4... of 8; k not of 16
]


@pytest.mark.parametrize("m,n,k,act,gated,res,rpi", SHAPES)
def test_fp32_gemm_kernels_agree_bitwise(gpu, m, n, k, act, gated, res, rpi):
    rng = np.random.default_rng(m * 13 + n * 7 + k)
    a = rng.normal(0, 1, (m, k)).astype(np.float32)
    w = rng.normal(0, 1 / np.sqrt(k), (n, k)).astype(np.float32)
    b = rng.normal(0, 0.1, n).astype(np.float32)
    g = rng.uniform(0, 1, (m // rpi, k)).astype(np.float32) if gated else None
    r = rng.normal(0, 1, (m, n)).astype(np.float32) if res else None
    outs = {}
    for kernel in (1, 2, 3):
        try:
            c, used = gpu.selftest_gemm_f32(a, w, b, act, g, rpi, r, kernel)
        except Exception as e:  # a kernel that does not cover the shape refuses it
            assert "does not support" in str(e), e
            continue
        assert used == kernel
        outs[kernel] = c
    assert 1 in outs and 3 in outs or k > 128, "streaming kernel should cover this shape"
    ref_a = a.astype(np.float64)
    if g is not None:
        ref_a = (a * np.repeat(g, rpi, axis=0)).astype(np.float32).astype(np.float64)
    pre = ref_a @ w.astype(np.float64).T + b
    ref = _act(pre, act)
    if r is not None:
        ref = ref + r
    scale = np.abs(ref_a) @ np.abs(w.astype(np.float64)).T + np.abs(b) + (np.abs(r) if r is not None else 0)
    for kernel, c in outs.items():
        assert np.all(np.abs(c - ref) <= 4e-6 * scale + 1e-6), f"kernel {kernel}: max err {np.abs(c - ref).max()}"
        np.testing.assert_array_equal(c, outs[1], err_msg=f"kernel {kernel} differs from the SIMT kernel")


def test_dispatch_choice(gpu):
    rng = np.random.default_rng(5)
    a = rng.normal(0, 1, (4096, 64)).astype(np.float32)
    w = rng.normal(0, 0.2, (32, 64)).astype(np.float32)
    _, used = gpu.selftest_gemm_f32(a, w, None, 0, None, 1, None, 0)
    assert used == 3   # thin output: the streaming kernel
    w = rng.normal(0, 0.2, (64, 64)).astype(np.float32)
    _, used = gpu.selftest_gemm_f32(a, w, None, 0, None, 1, None, 0)
    assert used == 1   # wider output: the register-tiled kernel
    a = rng.normal(0, 1, (64, 256)).astype(np.float32)
    w = rng.normal(0, 0.1, (16, 256)).astype(np.float32)
    _, used = gpu.selftest_gemm_f32(a, w, None, 0, None, 1, None, 0)
    assert used == 1   # k = 256 is past the streaming kernel's shared-memory tile


PAIRS = [
    # m, c, c', gated, residual, rows_per_image
    (1000, 32, 32, True, True, 250),     # detector stage-0 pair: gated, token residual
    (777, 32, 48, False, False, 1),      # stage transition pair (no residual)
    (513, 48, 48, True, True, 171),
    (300, 64, 64, False, True, 1),
    (129, 16, 16, True, False, 43),
]


@pytest.mark.parametrize("m,c,co,gated,res,rpi", PAIRS)
def test_fused_pair_matches_two_gemms(gpu, m, c, co, gated, res, rpi):
    """The fused pair kernel (used on maps of >= 98,304 rows, which the model tests
    never reach) equals the two-GEMM form bit for bit: the same k-ordered FMA chains."""
    rng = np.random.default_rng(m + 17 * c + co)
    a = rng.normal(0, 1, (m, c)).astype(np.float32)
    w1 = rng.normal(0, 1 / np.sqrt(c), (2 * c, c)).astype(np.float32)
    b1 = rng.normal(0, 0.1, 2 * c).astype(np.float32)
    w2 = rng.normal(0, 1 / np.sqrt(2 * c), (co, 2 * c)).astype(np.float32)
    b2 = rng.normal(0, 0.1, co).astype(np.float32)
    g = rng.uniform(0, 1, (m // rpi, c)).astype(np.float32) if gated else None
    fused = gpu.selftest_pair_f32(a, w1, b1, w2, b2, g, rpi, res)
    h, _ = gpu.selftest_gemm_f32(a, w1, b1, 3, g, rpi, None, 1)
    ga = (a * np.repeat(g, rpi, axis=0)).astype(np.float32) if gated else a
    two, _ = gpu.selftest_gemm_f32(h, w2, b2, 0, None, 1, ga if res else None, 1)
    np.testing.assert_array_equal(fused, two)
