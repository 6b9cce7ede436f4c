"""ppocr_model_forward_pipelined: chunked host-buffer forward with overlapped copies.

Each chunk is one forward of the model's batch, so the result must equal the
plain forward of the same chunk bit for bit; and since every kernel is
batch-invariant, it must also equal a model loaded at the full batch.
"""

import numpy as np
import pytest

import ppocr_b200 as P
from ppocr_b200 import seeded

pytestmark = pytest.mark.gpu


def _chunks(model, x, per):
    outs = [np.asarray(model.forward(x[i:i + per]).values, np.float32) for i in range(0, x.shape[0], per)]
    return np.concatenate(outs)


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_detector_pipelined_matches_forward(gpu, weights_file, precision):
    path = weights_file("det", "tiny", "spec")
    x = seeded.det_batch(6, 160, 224, seed=3)
    m2 = P.Detector.load(gpu, path, "tiny", (2, 3, 160, 224), precision=precision)
    got = m2.forward_pipelined(x)
    np.testing.assert_array_equal(got, _chunks(m2, x, 2))
    got_again = m2.forward_pipelined(x)            # staging buffers and events reused
    np.testing.assert_array_equal(got_again, got)
    m6 = P.Detector.load(gpu, path, "tiny", (6, 3, 160, 224), precision=precision)
    np.testing.assert_array_equal(got, np.asarray(m6.forward(x).values, np.float32))


def test_recognizer_pipelined_matches_forward(gpu, weights_file):
    path = weights_file("rec", "tiny", "spec")
    x = seeded.rec_batch(12, 160, seed=4)
    m4 = P.Recognizer.load(gpu, path, "tiny", (4, 3, 48, 160))
    got = m4.forward_pipelined(x)
    np.testing.assert_array_equal(got, _chunks(m4, x, 4))


def test_pipelined_rejects_bad_inputs(gpu, weights_file):
    path = weights_file("det", "tiny", "spec")
    m2 = P.Detector.load(gpu, path, "tiny", (2, 3, 128, 128))
    x = seeded.det_batch(3, 128, 128, seed=5)
    with pytest.raises(P.InvalidInput):
        m2.forward_pipelined(x)                    # 3 images: not a multiple of the batch
    x = seeded.det_batch(4, 128, 128, seed=5).copy()
    x[3, 1, 5, 7] = np.nan
    with pytest.raises(P.InvalidInput):
        m2.forward_pipelined(x)                    # non-finite input in the second chunk
    ok = m2.forward_pipelined(seeded.det_batch(4, 128, 128, seed=6))   # usable after an error
    assert np.isfinite(ok).all()


@pytest.mark.parametrize("precision", ["fp32", "bf16"])
def test_recognizer_pipelined_ctc_matches_forward_ctc(gpu, weights_file, precision):
    # Only the arg-max class and its probability cross to the host; both must
    # equal ppocr_recognizer_forward_ctc of the same chunk bit for bit.
    path = weights_file("rec", "tiny", "spec")
    x = seeded.rec_batch(12, 320, seed=7)
    m4 = P.Recognizer.load(gpu, path, "tiny", (4, 3, 48, 320), precision=precision)
    idx, prob = m4.forward_pipelined_ctc(x)
    ref = [m4.forward_ctc(x[i:i + 4]) for i in range(0, 12, 4)]
    np.testing.assert_array_equal(idx, np.concatenate([r[0] for r in ref]))
    np.testing.assert_array_equal(prob, np.concatenate([r[1] for r in ref]))
    # The same statistics as the full probabilities of ppocr_model_forward_pipelined.
    full = m4.forward_pipelined(x).reshape(12, idx.shape[1], -1)
    np.testing.assert_array_equal(prob, full.max(axis=2))
    idx2, prob2 = m4.forward_pipelined_ctc(x)      # reuses the staging
    np.testing.assert_array_equal(idx2, idx)
    np.testing.assert_array_equal(prob2, prob)
    with pytest.raises(P.InvalidInput):
        m4.forward_pipelined_ctc(x[:6])            # not a multiple of the batch


def test_pipelined_ctc_needs_a_recognizer(gpu, weights_file):
    path = weights_file("det", "tiny", "spec")
    m = P.Detector.load(gpu, path, "tiny", (1, 3, 128, 128))
    with pytest.raises(P.InvalidInput):
        P._check(P.library().ppocr_recognizer_forward_pipelined_ctc(m._h, None, 1, None, None, 0))
