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


def _act(ref, act):
    if act == 1:
        return np.maximum(ref, 0)
    if act == 2:
        return ref / (1 + np.exp(-ref))
    if act == 3:
        return gelu(ref)
    if act == 4:
        return ref * np.clip(ref + 3, 0, 6) / 6
    if act == 5:
        return 1 / (1 + np.exp(-ref))
    return ref


SENTINEL = 1232.0   # exact in BF16


@pytest.mark.parametrize("m,n,k,act,coff,ldc,out_bf16,res", [
    (300, 64, 96, 3, 32, 160, True, True),      # staged TMA store into a channel slice, residual
    (257, 96, 64, 0, 8, 200, True, False),      # tile wider than n: the store box is clipped at n
    (130, 48, 32, 4, 16, 72, True, True),
    (513, 256, 192, 3, 0, 256, True, False),
    (64, 200, 128, 5, 0, 200, False, True),     # FP32 output through the staged store
    (100, 50, 64, 0, 3, 57, False, False),      # unaligned FP32 slice: direct-store epilogue
    (77, 120, 64, 2, 4, 130, True, True),       # unaligned BF16 pitch: direct-store epilogue
])
def test_tc_gemm_slice_residual_and_neighbours(gpu, m, n, k, act, coff, ldc, out_bf16, res):
    rng = np.random.default_rng(m + 11 * n + 5 * k)
    a = bf16(rng.normal(0, 1, (m, k)))
    w = bf16(rng.normal(0, 1 / np.sqrt(k), (n, k)))
    b = rng.normal(0, 0.1, n).astype(np.float32)
    r = bf16(rng.normal(0, 1, (m, n))) if res else None
    c0 = np.full((m, ldc), SENTINEL, np.float32)
    c, used_tc, err = gpu.selftest_gemm_ex(a, w, c0, coff, b, act, r, out_bf16)
    assert used_tc, "tensor-core path not taken"
    assert err == 0, f"wait expired (code {err})"
    ref = _act(a.astype(np.float64) @ w.astype(np.float64).T + b, act)
    if r is not None:
        ref = ref + r
    scale = np.abs(a).astype(np.float64) @ np.abs(w).astype(np.float64).T + np.abs(b) + (0 if r is None else np.abs(r))
    tol = 1e-5 * scale + 1e-6 + (np.abs(ref) * 2.0 ** -8 if out_bf16 else 0)
    got = c[:, coff:coff + n]
    assert np.all(np.abs(got - ref) <= tol), f"max err {np.abs(got - ref).max()}"
    outside = np.ones(ldc, bool)
    outside[coff:coff + n] = False
    assert np.all(c[:, outside] == SENTINEL), "columns outside the slice were written"
