"""The oracle's end-to-end host steps against the reference's own tests (src/ocr.rs:1220-1302)."""

import numpy as np
import pytest

from oracle import pipeline as opl


def test_detector_postprocess_maps_components_to_source_coordinates():
    # src/ocr.rs:1225-1250
    values = np.zeros(416 * 736, np.float32)
    for y in range(20, 22):
        values[y * 736 + 10:y * 736 + 14] = 0.9
    dets = opl.extract_detections(values, 416, 736, (736, 416), (736, 416),
                                  opl.PostprocessOptions(min_area=4, unclip_ratio=1.0))
    assert len(dets) == 1
    assert abs(dets[0].score - 0.9) < 1e-6
    assert abs(dets[0].polygon[0][0] - 10.0) < 1e-4


def test_recognition_plan_preserves_the_entire_crop():
    # src/ocr.rs:1268-1283
    poly = [(0.0, 0.0), (1000.0, 0.0), (1000.0, 20.0), (0.0, 20.0)]
    assert opl.batch_width([poly]) == 2400
    assert opl.crop_content_width(poly) == 2400


def test_recognizer_batch_uses_the_largest_aspect_ratio():
    # src/ocr.rs:1285-1302
    narrow = [(0.0, 0.0), (80.0, 0.0), (80.0, 20.0), (0.0, 20.0)]
    wide = [(0.0, 0.0), (300.0, 0.0), (300.0, 20.0), (0.0, 20.0)]
    assert opl.batch_width([narrow, wide]) == 720


def test_rotated_component_box_is_tight_and_sorted():
    # A rotated bar: the fitted box must contain every component pixel centre and
    # detections must come back in reading order (centre y, then x).
    h, w = 96, 160
    values = np.zeros((h, w), np.float32)
    ys, xs = np.mgrid[0:h, 0:w]
    t = np.deg2rad(20.0)
    u = (xs - 60) * np.cos(t) + (ys - 50) * np.sin(t)
    v = -(xs - 60) * np.sin(t) + (ys - 50) * np.cos(t)
    values[(np.abs(u) < 30) & (np.abs(v) < 5)] = 0.8
    values[5:9, 100:140] = 0.7
    dets = opl.extract_detections(values, h, w, (w, h), (w, h), opl.PostprocessOptions(unclip_ratio=1.0))
    assert len(dets) == 2
    assert opl.polygon_center(dets[0].polygon)[1] < opl.polygon_center(dets[1].polygon)[1]
    poly = np.array(dets[1].polygon, np.float64)
    ax = poly[1] - poly[0]
    ang = np.degrees(np.arctan2(ax[1], ax[0]))
    assert abs(ang - 20.0) < 3.0


def test_max_boxes_keeps_the_highest_scores():
    values = np.zeros((32, 64), np.float32)
    for i, s in enumerate([0.5, 0.9, 0.7]):
        values[4 + 8 * i:7 + 8 * i, 4:20] = s
    dets = opl.extract_detections(values, 32, 64, (64, 32), (64, 32), opl.PostprocessOptions(max_boxes=2))
    assert [round(float(d.score), 3) for d in dets] == [0.9, 0.7]


def test_postprocess_options_validate():
    with pytest.raises(ValueError):
        opl.PostprocessOptions(min_area=0).validate()
    with pytest.raises(ValueError):
        opl.PostprocessOptions(binary_threshold=1.5).validate()
    with pytest.raises(ValueError):
        opl.PostprocessOptions(unclip_ratio=0.0).validate()


def test_parse_dictionary_forms():
    assert opl.parse_dictionary("﻿a\nb\r\nc") == ["a", "b", "c"]
    yml = "Global:\n  x: 1\nPostProcess:\n  character_dict:\n    - a\n    - ' '\n    - \"q\"\n    - 'it''s'\n  other: 2\n"
    assert opl.parse_dictionary(yml) == ["a", " ", "q", "it's"]
    with pytest.raises(ValueError):
        opl.parse_dictionary("a\n\nb")
    with pytest.raises(ValueError):
        opl.parse_dictionary("")
    with pytest.raises(ValueError):
        opl.parse_dictionary("character_dict:\n  - 'x\n")


def test_join_decoded_texts_overlap():
    assert opl.append_with_overlap("hello wor", "world") == ("hello world", 2)
    text, score = opl.join_decoded_texts([("abc", 0.5), ("bcd", 1.0), ("", 0.1)])
    assert text == "abcd"
    assert abs(score - (0.5 * 3 + 1.0 * 1) / 4) < 1e-7
