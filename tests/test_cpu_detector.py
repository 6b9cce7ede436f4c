"""The C++ CPU restatement of the detector (oracle/cpu_detector.cpp, the timed
CPU baseline) against the torch port of the reference (oracle/model.py).
Both are FP32 with different summation orders, so they are compared on the
conditioned weight profile (activations O(1)) at FP32-rounding tolerance."""

import numpy as np
import pytest

from ppocr_b200 import seeded
from oracle import model as om
from oracle.cpu_detector import CpuDetector


@pytest.mark.parametrize("size,shape", [("tiny", (2, 3, 64, 96)), ("small", (1, 3, 96, 64))])
def test_cpu_restatement_matches_torch_port(weights_file, size, shape):
    path = weights_file("det", size, "conditioned")
    x = seeded.det_batch(shape[0], shape[2], shape[3], seed=4, text=True)
    got = CpuDetector(path, size).forward(x, threads=2)
    want = om.Detector(om.Weights.load(path), size).forward(x)
    assert got.shape == want.shape
    assert np.abs(got - want).max() <= 1e-4
