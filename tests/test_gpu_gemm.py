"""tcgen05 BF16 GEMM against a float64 reference of the same BF16-rounded operands.

The kernel accumulates in FP32 (TMEM); the bound below is a few FP32 ulps of
the sum of |products|, far tighter than any BF16 operand error.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def bf16(x):
    x = np.asarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


def gelu(x):
    import math
    erf = np.vectorize(math.erf)
    return 0.5 * x * (1 + erf(x / math.sqrt(2)))


@pytest.mark.parametrize("m,n,k,act", [
    (1, 16, 16, 0), (40, 80, 160, 0), (128, 48, 24, 1), (300, 120, 80, 2), (257, 576, 192, 0),
    (1000, 1000, 768, 3), (64, 18710 // 10, 192, 0), (513, 256, 64, 0), (130, 208, 1536, 0),
])
def test_tc_gemm_matches_reference(gpu, m, n, k, act):
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a = bf16(rng.normal(0, 1, (m, k)))
    w = bf16(rng.normal(0, 1 / np.sqrt(k), (n, k)))
    b = rng.normal(0, 0.1, n).astype(np.float32)
    c, used_tc, err = gpu.selftest_gemm(a, w, b, act)
    assert used_tc, "tensor-core path not taken"
    assert err == 0, f"wait expired (code {err})"
    ref = a.astype(np.float64) @ w.astype(np.float64).T + b
    if act == 1:
        ref = np.maximum(ref, 0)
    elif act == 2:
        ref = ref / (1 + np.exp(-ref))
    elif act == 3:
        ref = gelu(ref)
    scale = np.abs(a).astype(np.float64) @ np.abs(w).astype(np.float64).T + np.abs(b)
    tol = 1e-5 * scale + 1e-6
    assert np.all(np.abs(c - ref) <= tol), f"max err {np.abs(c - ref).max()}"
