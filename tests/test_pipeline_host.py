"""Host steps of the end-to-end pipeline (C ABI, no GPU) against the oracle restatement.

DB postprocess boxes and scores, dictionary parsing and CTC text assembly must
be bit-identical to the oracle's (src/ocr.rs restated in oracle/pipeline.py).
"""

import numpy as np
import pytest

import ppocr_b200 as P
from oracle import pipeline as opl
from oracle import postprocess as opost


def _rotated_bars(h, w, seed, count=12):
    rng = np.random.default_rng(seed)
    values = (rng.random((h, w)) * 0.15).astype(np.float32)
    ys, xs = np.mgrid[0:h, 0:w].astype(np.float32)
    for _ in range(count):
        cx, cy = rng.uniform(0, w), rng.uniform(0, h)
        bw, bh = rng.uniform(4, w / 3), rng.uniform(2, 12)
        t = np.deg2rad(rng.uniform(-30, 30))
        u = (xs - cx) * np.cos(t) + (ys - cy) * np.sin(t)
        v = -(xs - cx) * np.sin(t) + (ys - cy) * np.cos(t)
        m = (np.abs(u) < bw / 2) & (np.abs(v) < bh / 2)
        values[m] = rng.uniform(0.2, 1.0, size=int(m.sum())).astype(np.float32)
    return values


def _compare(values, source, content, options_kwargs=None):
    kw = options_kwargs or {}
    h, w = values.shape
    want = opl.extract_detections(values, h, w, source, content, opl.PostprocessOptions(**kw))
    got = P.db_postprocess(values, source, content, P.PostprocessOptions(**kw))
    assert len(got) == len(want)
    for (poly, score), d in zip(got, want):
        np.testing.assert_array_equal(poly, np.array(d.polygon, dtype=np.float32))
        assert score == d.score
    return len(want)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_db_postprocess_matches_oracle(seed):
    values = _rotated_bars(96, 160, seed)
    assert _compare(values, (160, 96), (160, 96)) > 0


def test_db_postprocess_maps_content_to_source():
    values = _rotated_bars(128, 224, 7, count=20)
    assert _compare(values, (1920, 1080), (192, 108)) > 0   # content smaller than the map, upscaled source


def test_db_postprocess_options_and_max_boxes():
    values = _rotated_bars(96, 160, 3, count=25)
    n = _compare(values, (160, 96), (160, 96), dict(binary_threshold=0.3, box_threshold=0.5, min_area=5,
                                                    unclip_ratio=2.0, max_boxes=4))
    assert n == 4


def test_db_postprocess_reference_known_answer():
    # src/ocr.rs:1225-1250
    values = np.zeros((416, 736), np.float32)
    values[20:22, 10:14] = 0.9
    got = P.db_postprocess(values, (736, 416), (736, 416), P.PostprocessOptions(min_area=4, unclip_ratio=1.0))
    assert len(got) == 1
    assert abs(got[0][1] - 0.9) < 1e-6
    assert abs(got[0][0][0, 0] - 10.0) < 1e-4


def test_db_postprocess_rejects_bad_input():
    values = np.zeros((32, 32), np.float32)
    values[3, 3] = np.nan
    with pytest.raises(P.InvalidInput):
        P.db_postprocess(values, (32, 32))
    with pytest.raises(P.InvalidInput):
        P.db_postprocess(np.zeros((32, 32), np.float32), (32, 32), options=P.PostprocessOptions(min_area=0))


DICTS = [
    "﻿a\nb\r\nc",
    "Global:\n  x: 1\nPostProcess:\n  character_dict:\n    - a\n    - ' '\n    - \"q\"\n    - 'it''s'\n  other: 2\n",
    "x\ny\nz\n",
    "漢\n字\né\n",
]


@pytest.mark.parametrize("contents", DICTS)
def test_dictionary_parse_matches_oracle(contents):
    assert P.Dictionary.parse(contents).entries() == opl.parse_dictionary(contents)


@pytest.mark.parametrize("contents", ["", "a\n\nb", "character_dict:\n  - 'x\n", "character_dict:\n  oops\n"])
def test_dictionary_errors(contents):
    with pytest.raises(ValueError):
        opl.parse_dictionary(contents)
    with pytest.raises(P.InvalidInput):
        P.Dictionary.parse(contents)


def _softmax(x):
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


@pytest.mark.parametrize("seed,implicit_space,content", [(0, False, 320), (1, True, 200), (2, False, 37)])
def test_ctc_decode_matches_oracle(seed, implicit_space, content):
    rng = np.random.default_rng(seed)
    dictionary = [f"<{i}>" for i in range(30)] + ["漢"]
    classes = len(dictionary) + (2 if implicit_space else 1)
    logits = rng.normal(0, 3, size=(40, classes)).astype(np.float32)
    logits[::3, 0] += 6   # some blanks
    logits[5:9, 7] += 9   # a repeat run
    probs = _softmax(logits)
    d = P.Dictionary.parse("\n".join(dictionary))
    text, score = d.decode(probs, content, 320)
    want_text, want_score, _ = opost.decode_ctc_greedy(probs, dictionary, content, 320)
    assert text == want_text
    assert abs(score - want_score) <= 1e-6 * max(1.0, abs(want_score))
    idx = opost.argmax_last(probs).astype(np.int32)
    text2, score2 = d.decode_steps(idx, probs[np.arange(40), idx], classes, content, 320)
    assert text2 == want_text and abs(score2 - want_score) <= 1e-6


def test_ctc_decode_non_probability_rows_and_errors():
    # Rows that are not a probability distribution go through the softmax
    # branch of row_probability (src/ocr.rs:1158-1169).
    rng = np.random.default_rng(5)
    rows = rng.normal(0, 2, size=(12, 6)).astype(np.float32)
    d = P.Dictionary.parse("a\nb\nc\nd\ne")
    text, score = d.decode(rows, 100, 100)
    want_text, want_score, _ = opost.decode_ctc_greedy(rows, ["a", "b", "c", "d", "e"], 100, 100)
    assert text == want_text and abs(score - want_score) <= 1e-6
    with pytest.raises(P.InvalidInput):
        d.decode(rows[:, :4], 100, 100)          # classes != entries + 1
    with pytest.raises(P.InvalidInput):
        d.decode(rows, 0, 100)                   # content width outside 1..=input
