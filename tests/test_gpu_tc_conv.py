"""FP32 tensor-core conv / GEMM (3xTF32 on tcgen05) against float64.

The bound is FP32-class: a few units of 2^-22 of the sum of |products|,
which a BF16 or single-TF32 product would exceed by orders of magnitude.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,h,w,cin,cout,k,stride,pad,act", [
    (1, 7, 9, 16, 32, 1, 1, 0, 0),        # dense GEMM mode
    (2, 13, 11, 32, 64, 1, 1, 0, 1),
    (3, 50, 37, 160, 320, 1, 1, 0, 3),     # K tail (160 = 5 x 32), two N tiles
    (1, 9, 10, 48, 40, 1, 1, 0, 2),        # N not a multiple of 16
    (2, 17, 23, 32, 16, 3, 1, 1, 1),       # gather mode: 3x3, pad 1
    (1, 26, 30, 64, 64, 3, 2, 1, 0),       # 3x3 stride 2
    (2, 15, 14, 32, 32, 7, 1, 3, 0),       # 7x7 (intraclass)
    (1, 40, 36, 8, 16, 2, 1, 0, 1),        # 2x2
])
def test_tc_conv_matches_float64(gpu, n, h, w, cin, cout, k, stride, pad, act):
    rng = np.random.default_rng(n + h * 3 + w * 5 + cin + cout + k)
    x = rng.normal(0, 1, (n, h, w, cin)).astype(np.float32)
    wt = rng.normal(0, 1 / np.sqrt(cin * k * k), (cout, cin, k, k)).astype(np.float32)
    b = rng.normal(0, 0.1, cout).astype(np.float32)
    out, err = gpu.selftest_conv(x, wt, b, stride=stride, pad=pad, act=act)
    assert err == 0, f"wait expired (code {err})"
    xt = torch.from_numpy(x).double().permute(0, 3, 1, 2)
    ref = F.conv2d(xt, torch.from_numpy(wt).double(), torch.from_numpy(b).double(), stride=stride, padding=pad)
    mag = F.conv2d(xt.abs(), torch.from_numpy(wt).double().abs(), torch.from_numpy(b).double().abs(), stride=stride,
                   padding=pad)
    if act == 1:
        ref = ref.clamp(min=0)
    elif act == 2:
        ref = ref / (1 + torch.exp(-ref))
    elif act == 3:
        ref = 0.5 * ref * (1 + torch.erf(ref / np.sqrt(2)))
    ref = ref.permute(0, 2, 3, 1).numpy()
    mag = mag.permute(0, 2, 3, 1).numpy()
    tol = 8 * 2.0 ** -22 * mag + 1e-6
    d = np.abs(out - ref)
    assert np.all(d <= tol), f"max err {d.max()}, worst ratio {(d / tol).max()}"
