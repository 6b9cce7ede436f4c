"""Pins the CPU oracle against the reference's own known-answer tests.

Each test restates one #[test] of ppocr-rs (cited) against the oracle's
functions, so the oracle used by the GPU parity tests is anchored to the
reference's published expectations.
"""

import math

import numpy as np
import pytest
import torch

from oracle import model as om
from oracle import postprocess as opost
from oracle import preprocess as opre


def T(a):
    return torch.tensor(np.asarray(a, dtype=np.float32))


def test_erf_known_values():
    # src/cpu/kernels/mod.rs:2409-2414
    assert abs(float(om.erf_as(T([0.0]))[0])) < 1e-6
    assert abs(float(om.erf_as(T([1.0]))[0]) - 0.8427008) < 2e-7
    assert abs(float(om.erf_as(T([-2.0]))[0]) + 0.9953223) < 2e-7


def test_gelu_close_to_exact_erf():
    # src/cpu/kernels/mod.rs:2416-2433 bounds the vector GELU by 2e-5 of the scalar form.
    x = np.arange(1025, dtype=np.float32) * (16.0 / 1024.0) - 8.0
    exact = np.array([0.5 * v * (1 + math.erf(v / math.sqrt(2))) for v in x.astype(np.float64)])
    assert np.abs(om.gelu(T(x)).numpy() - exact).max() < 2e-5


def test_activation_formulas():
    x = T([-7.0, -3.0, -0.5, 0.0, 0.5, 3.0, 7.0])
    np.testing.assert_allclose(om.hard_swish(x).numpy(), (x * torch.clamp(x / 6 + 0.5, 0, 1)).numpy())
    np.testing.assert_allclose(om.hard_sigmoid(x, 0.2, 0.5).numpy(), np.clip(x.numpy() * 0.2 + 0.5, 0, 1))
    np.testing.assert_allclose(om.silu(x).numpy(), (x / (1 + torch.exp(-x))).numpy())


def test_validate_input_boundaries():
    # src/cpu/model.rs:2132-2138
    om.validate_input((1, 3, 32, 32), True)
    with pytest.raises(ValueError):
        om.validate_input((1, 3, 32, 31), True)
    om.validate_input((1, 3, 48, 5), False)
    with pytest.raises(ValueError):
        om.validate_input((1, 3, 48, 4), False)


def test_upsample_add_matches_resize_then_add():
    # src/cpu/model.rs:2140-2161 (nearest resize: in = out * h / out_h, ops.rs:1609-1655)
    upper = (np.arange(2 * 2 * 2 * 3, dtype=np.float32) - 9.0) * 0.125
    upper = upper.reshape(2, 2, 2, 3)
    feature = ((np.arange(2 * 2 * 4 * 6, dtype=np.float32) - 31.0) * 0.0625).reshape(2, 2, 4, 6)
    resized = np.empty_like(feature)
    for y in range(4):
        for x in range(6):
            resized[:, :, y, x] = upper[:, :, y * 2 // 4, x * 3 // 6]
    got = (T(feature) + om.upsample(T(upper), 2)).numpy()
    np.testing.assert_array_equal(got, feature + resized)


def test_upsample_cat_matches_reversed_neck_layout():
    # src/cpu/model.rs:2163-2194
    def mk(shape, offset):
        return offset + np.arange(int(np.prod(shape)), dtype=np.float32).reshape(shape) * 0.25

    feats = [mk((2, 1, 1, 2), 100.0), mk((2, 2, 2, 4), 10.0), mk((2, 1, 4, 8), -20.0)]
    got = torch.cat([om.upsample(T(f), s) for f, s in zip(feats, (4, 2, 1))], dim=1).numpy()
    assert got.shape == (2, 4, 4, 8)
    np.testing.assert_array_equal(got[:, 0], np.repeat(np.repeat(feats[0][:, 0], 4, 1), 4, 2))
    np.testing.assert_array_equal(got[:, 3], feats[2][:, 0])


def test_rank_one_conv_matches_dense_fused_weight():
    # src/cpu/model.rs:2213-2268
    cin, cout, k, h, w = 4, 5, 9, 11, 19
    sp = k * k
    dw = np.array([((i * 17 % 43) - 21.0) / 97.0 for i in range(cin * sp)], np.float32)
    pw = np.array([((i * 11 % 29) - 14.0) / 31.0 for i in range(cout * cin)], np.float32)
    fused = np.zeros((cout, cin, sp), np.float32)
    for o in range(cout):
        for i in range(cin):
            fused[o, i] = pw[o * cin + i] * dw[i * sp:(i + 1) * sp]
    fused = fused.reshape(cout, cin, k, k)
    bias = np.array([(c - 2.0) / 13.0 for c in range(cout)], np.float32)
    x = np.array([((i * 23 % 61) - 30.0) / 37.0 for i in range(cin * h * w)], np.float32).reshape(1, cin, h, w)
    dense = om.conv2d(T(x), fused, bias, (1, 1), (k // 2,) * 4)
    d, p = om.factor_rank_one(fused, cin, cout, k)
    rank1 = om.conv2d(om.conv2d(T(x), d, None, (1, 1), (k // 2,) * 4, cin), p, bias)
    assert float((dense - rank1).abs().max()) < 2e-5


def test_rank_one_rejects_nonseparable_weight():
    # src/cpu/model.rs:2270-2277
    v = np.zeros(2 * 3 * 3, np.float32)
    v[0] = 1.0
    v[9 + 1] = 1.0
    with pytest.raises(ValueError):
        om.factor_rank_one(v.reshape(2, 1, 3, 3), 1, 2, 3)


def test_intraclass_fusion_exact_indices():
    # src/cpu/model.rs:2279-2328
    o, i, k = 2, 2, 3
    sym = np.arange(o * i * k * k, dtype=np.float32).reshape(o, i, k, k)
    ver = (100.0 + np.arange(o * i * k, dtype=np.float32)).reshape(o, i, k, 1)
    hor = (200.0 + np.arange(o * i * k, dtype=np.float32)).reshape(o, i, 1, k)
    w, b = om.fuse_intraclass(sym, np.array([1.0, 2.0], np.float32), ver, np.array([3.0, 4.0], np.float32),
                              hor, np.array([5.0, 6.0], np.float32))
    c = k // 2
    for oo in range(o):
        for ii in range(i):
            for r in range(k):
                for col in range(k):
                    e = sym[oo, ii, r, col]
                    if col == c:
                        e += ver[oo, ii, r, 0]
                    if r == c:
                        e += hor[oo, ii, 0, col]
                    assert w[oo, ii, r, col] == e
    np.testing.assert_array_equal(b, [9.0, 12.0])


def test_fused_intraclass_matches_three_branches():
    # src/cpu/model.rs:2330-2407
    o, i, k = 2, 3, 5

    def pat(n, mul, scale):
        return np.array([((j * mul % 31) - 15.0) * scale for j in range(n)], np.float32)

    sw = pat(o * i * k * k, 7, 0.01).reshape(o, i, k, k)
    vw = pat(o * i * k, 11, 0.015).reshape(o, i, k, 1)
    hw = pat(o * i * k, 13, 0.012).reshape(o, i, 1, k)
    sb, vb, hb = (np.array(v, np.float32) for v in ([0.07, -0.03], [-0.02, 0.05], [0.01, -0.04]))
    x = T(pat(i * 7 * 8, 17, 0.02).reshape(1, i, 7, 8))
    p = k // 2
    want = (om.conv2d(x, sw, sb, (1, 1), (p, p, p, p)) + om.conv2d(x, vw, vb, (1, 1), (p, 0, p, 0))
            + om.conv2d(x, hw, hb, (1, 1), (0, p, 0, p))).numpy()
    fw, fb = om.fuse_intraclass(sw, sb, vw, vb, hw, hb)
    got = om.conv2d(x, fw, fb, (1, 1), (p, p, p, p)).numpy()
    assert np.all(np.abs(got - want) <= 2e-5 * np.maximum(np.abs(want), 1.0))


def test_linear_fuses_bias_and_softmax():
    # src/cpu/backend.rs:1401-1415
    w = np.array([[1.0, 0.0, -1.0], [0.0, 1.0, 1.0]], np.float32)
    out = om.linear(T([[2.0, 3.0, 1.0]]), w, np.array([0.5, -0.5], np.float32)).numpy()
    np.testing.assert_array_equal(out, [[1.5, 3.5]])
    p = om.softmax(T(out)).numpy()
    assert abs(p.sum() - 1) < 1e-6 and p[0, 1] > p[0, 0]


def test_transposed_conv_io_layout():
    # src/cpu/backend.rs:1848-1866
    out = om.conv_transpose_2x2(T([[[[1.0, 2.0]]]]), np.ones((1, 1, 2, 2), np.float32), np.array([0.5], np.float32))
    np.testing.assert_array_equal(out.numpy().reshape(-1), [1.5, 1.5, 2.5, 2.5, 1.5, 1.5, 2.5, 2.5])


def test_max_pool_same_upper():
    # ops.rs:1520-1535: 2x2 stride 1, bottom/right padding never wins
    x = T(np.array([[[[1.0, 5.0, 2.0], [3.0, -1.0, 4.0]]]], np.float32))
    np.testing.assert_array_equal(om.max_pool_same_upper(x).numpy()[0, 0], [[5.0, 5.0, 4.0], [3.0, 4.0, 4.0]])


def test_avg_pool_3x2():
    x = np.arange(3 * 5, dtype=np.float32).reshape(1, 1, 3, 5)
    got = om.avg_pool_3x2(T(x)).numpy()
    assert got.shape == (1, 1, 1, 2)
    np.testing.assert_allclose(got[0, 0, 0], [x[0, 0, :, 0:2].sum() / 6, x[0, 0, :, 2:4].sum() / 6], rtol=1e-6)


def test_detector_plan_1920x1080():
    # src/preprocess.rs:150-158
    assert opre.detector_input_size(1920, 1080, 736) == (736, 416)


def test_recognizer_pad_and_content_width():
    # src/preprocess.rs:160-179
    rgb = np.full((20, 80, 3), 127, np.uint8)
    cw = opre.scaled_recognizer_width(80, 20)
    assert cw == 192
    x = opre.prepare_recognizer_crop(rgb, [(0, 0), (80, 0), (80, 20), (0, 20)], 320, cw)
    assert x.shape == (1, 3, 48, 320)
    assert abs(x[0, 0, 0, 0] - (127.0 / 255.0 - 0.5) / 0.5) < 1e-6
    assert x[0, 0, 0, cw] == 0.0


def test_preprocess_matches_unrounded_bilinear_within_rounding():
    # src/preprocess.rs:181-227 compares against an exact bilinear sample of
    # integer-valued pixels; rounding to integers bounds the difference by half a level.
    xs, ys = np.meshgrid(np.arange(37), np.arange(29))
    rgb = np.stack([(xs * 7 + ys * 3) % 256, (xs * 2 + ys * 5) % 256, (xs * 3 + ys * 7) % 256], -1).astype(np.uint8)
    corners = [(2.25, 1.75), (34.5, 3.0), (32.75, 27.0), (1.0, 25.5)]
    got = opre.normalized_bgr(rgb, corners, 41, 23, 41, opre.DETECTOR_MEAN_BGR, opre.DETECTOR_STD_BGR)
    assert np.all(np.isfinite(got))
    # every sample is an integer level after denormalisation
    scale, bias = opre.normalization(opre.DETECTOR_MEAN_BGR, opre.DETECTOR_STD_BGR)
    levels = (got[0] - bias[:, None, None]) / scale[:, None, None]
    assert np.abs(levels - np.round(levels)).max() < 1e-3


def test_detector_bgr_statistics_known_answer():
    # src/gpu/runtime.rs:2943-2967 (pure red pixel)
    x = opre.normalized_bgr(np.array([[[255, 0, 0]]], np.uint8), [(0, 0), (1, 0), (1, 1), (0, 1)], 1, 1, 1,
                            opre.DETECTOR_MEAN_BGR, opre.DETECTOR_STD_BGR)
    want = [(0.0 - 0.485) / 0.229, (0.0 - 0.456) / 0.224, (1.0 - 0.406) / 0.225]
    np.testing.assert_allclose(x[0, :, 0, 0], want, atol=1e-5)


def test_recognizer_red_blue_row_known_answer():
    # src/gpu/runtime.rs:2907-2941: a red/blue 2x1 image resampled to 4 columns.  The
    # reference's device shader does not round; the CPU path does (kernels.rs:159), so
    # the blends differ from the shader's by at most one level (2/255 in +-1 units).
    x = opre.normalized_bgr(np.array([[[255, 0, 0], [0, 0, 255]]], np.uint8), [(0, 0), (2, 0), (2, 1), (0, 1)],
                            4, 2, 4, opre.RECOGNIZER_MEAN_BGR, opre.RECOGNIZER_STD_BGR)
    want = np.array([[-1.0, -1.0, 1.0], [-0.5, -1.0, 0.5], [0.5, -1.0, -0.5], [1.0, -1.0, -1.0]])
    for row in range(2):
        np.testing.assert_allclose(x[0, :, row, :].T, want, atol=2.0 / 255.0 + 1e-6)


def test_ctc_ignores_padded_steps():
    # src/ocr.rs:1253-1266
    probs = np.array([[0.1, 0.9]] * 5, np.float32)
    text, score, _ = opost.decode_ctc_greedy(probs, ["A"], 40, 100)
    assert text == "A" and abs(score - 0.9) < 1e-6


def test_ctc_argmax_ties_take_last_index():
    # Iterator::max_by keeps the last of equal maxima (src/ocr.rs:1171-1177)
    rows = np.array([[0.2, 0.4, 0.4], [0.5, 0.5, 0.0]], np.float32)
    np.testing.assert_array_equal(opost.argmax_last(rows), [2, 1])


def test_recognizer_batch_width():
    # src/ocr.rs:1268-1302
    assert opre.recognizer_batch_width([opre.scaled_recognizer_width(80, 20), opre.scaled_recognizer_width(300, 20)]) == 720
    assert opre.scaled_recognizer_width(1000, 20) == 2400
    assert opre.recognizer_batch_width([2400]) == 2400


def test_db_mask_threshold():
    p = np.array([0.1, 0.2, 0.19999999, 0.9], np.float32)
    np.testing.assert_array_equal(opost.db_mask(p, 0.2), [0, 1, 0, 1])
