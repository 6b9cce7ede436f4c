"""Failure detection of the tensor-core kernels, made without faulting the GPU.

Every pipeline wait in the tcgen05 GEMM and engine kernels is bounded by the
GPU's global timer.  ppocr_selftest_wait_expiry runs a GEMM whose first CTA
never issues its first stage's loads (an arrive that never comes), with a
20 ms bound: the kernel must drain what it has in flight, free its TMEM,
return, and the call must fail with Error::Gpu carrying the kernel's code.
The device must then still compute correctly.
"""

import numpy as np
import pytest

import ppocr_b200 as P

pytestmark = pytest.mark.gpu


def bf16(x):
    x = np.asarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return (u.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.parametrize("kernel", [0, 1, 2, 3])
def test_wait_expiry_fails_cleanly(gpu, kernel):
    with pytest.raises(P.GpuError) as info:
        gpu.selftest_wait_expiry(kernel, 20)
    assert info.value.wait_code != 0
    assert "wait ran out" in str(info.value)
    # The context survives: a normal tensor-core GEMM on the same device.
    rng = np.random.default_rng(kernel)
    a = bf16(rng.normal(0, 1, (256, 128)))
    w = bf16(rng.normal(0, 0.1, (64, 128)))
    c, used_tc, err = gpu.selftest_gemm(a, w)
    assert used_tc and err == 0
    ref = a.astype(np.float64) @ w.astype(np.float64).T
    assert np.abs(c - ref).max() <= 1e-3


def test_model_forward_still_clean_after_expiry(gpu, weights_file):
    """A model forward after an expiry reports no stale wait error (the flag is per model)."""
    from ppocr_b200 import seeded

    with pytest.raises(P.GpuError):
        gpu.selftest_wait_expiry(0, 20)
    path = weights_file("rec", "tiny", "conditioned")
    rec = P.Recognizer.load(gpu, path, "tiny", (2, 3, 48, 64), precision="bf16")
    out = rec.forward(seeded.rec_batch(2, 64, seed=1))
    assert np.isfinite(out.values).all()
