"""ppocr_preprocess_noalloc: device preprocessing with no allocation call.

It is for callers that cannot call cudaMalloc (a fixed device-memory budget,
an allocator that owns all device memory, or a server that forbids the
device-synchronising allocation calls while serving).  It stages its output
in a fixed 4 MiB device array inside the library instead of a per-call
allocation, so its results must equal ppocr_preprocess's exactly, call after
call: the second call below also checks that nothing from the first call's
larger output leaks into a smaller one.  This file sorts last so that a
`pytest -x` run has executed every other test before it.
"""

import numpy as np
import pytest

import ppocr_b200 as P

pytestmark = pytest.mark.gpu


def test_noalloc_preprocess_matches_allocating_entry_point(gpu):
    rng = np.random.default_rng(21)
    rgb = rng.integers(0, 256, size=(270, 480, 3), dtype=np.uint8)
    img = gpu.upload_rgb(480, 270, rgb)
    calls = [
        # (corners, content_width, out_h, out_w, kind): a full detector frame, then a
        # smaller rotated recognizer crop with zero padding past its content.
        ([(0, 0), (480, 0), (480, 270), (0, 270)], 736, 416, 736, "det"),
        ([(30.5, 40.0), (300.0, 60.25), (296.0, 110.0), (26.0, 90.5)], 100, 48, 160, "rec"),
    ]
    for corners, content, h, w, kind in calls:
        want = gpu.preprocess(img, corners, content, h, w, kind)
        got = gpu.preprocess_noalloc(img, corners, content, h, w, kind)
        assert got.shape == want.shape
        np.testing.assert_array_equal(got, want)
        assert np.all(got[..., content:] == 0)


def test_noalloc_preprocess_rejects_outputs_beyond_its_limit(gpu):
    img = gpu.upload_rgb(4, 4, np.zeros(48, np.uint8))
    with pytest.raises(P.InvalidInput, match="limit"):
        gpu.preprocess_noalloc(img, [(0, 0), (4, 0), (4, 4), (0, 4)], 600, 600, 600, "det")
