"""End-to-end engine (detector -> DB postprocess -> device rectification ->
recognizer -> CTC text) on a synthetic page, checked stage by stage.

* The engine's boxes and detection scores equal the oracle's DB postprocess
  (src/ocr.rs:723-782) applied to the same device probability map, bit for bit.
* Each recognition chunk (aspect-ratio order, six per chunk, canvas width of the
  chunk) matches the oracle's planning; the device rectification + forward
  gives the same greedy-CTC classes as the host-preprocessed forward, and the
  oracle recognizer agrees wherever its top-2 logit margin is at least 1e-2.
* The engine's text is the CTC assembly of those classes.
"""

import json
import os
import struct
import subprocess
import zlib

import numpy as np
import pytest

import ppocr_b200 as P
from oracle import model as om
from oracle import pipeline as opl
from oracle import postprocess as opost
from oracle import preprocess as opre
from ppocr_b200 import seeded

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CTC_MARGIN = 1e-2


@pytest.fixture(scope="module")
def setup(weights_file, tmp_path_factory):
    det = weights_file("det", "tiny", "spec")
    rec = weights_file("rec", "tiny", "spec")
    d = tmp_path_factory.mktemp("dict") / "dict.txt"
    entries = seeded.synthetic_dictionary("tiny")
    d.write_text("\n".join(entries) + "\n", encoding="utf-8")
    rgb = seeded.text_page_rgb8(180, 320, seed=21, blocks=(6, 10), block_h=(12, 28), block_w=(40, 200),
                                max_angle=15.0, background=(170, 250))
    return det, rec, str(d), entries, rgb


def test_engine_matches_oracle_stage_by_stage(gpu, setup):
    det_path, rec_path, dict_path, entries, rgb = setup
    h, w = rgb.shape[:2]
    eng = P.Engine(gpu, det_path, rec_path, dict_path)
    result = eng.recognize(rgb)
    assert result["source_size"] == [w, h]
    iw, ih = opre.detector_input_size(w, h, 736)
    assert result["detector_input_size"] == [iw, ih]

    # Detector stage: the same device probability map through the oracle's postprocess.
    detm = P.Detector.load(gpu, det_path, "tiny", (1, 3, ih, iw))
    img = gpu.upload_rgb(w, h, rgb)
    prob = detm.forward_image(img, P.ImagePreprocess.detector([(0, 0), (w, 0), (w, h), (0, h)])).values
    prob = np.asarray(prob, np.float32).reshape(ih, iw)
    dets = opl.extract_detections(prob, ih, iw, (w, h), (iw, ih))
    assert len(dets) == len(result["lines"]) and len(dets) > 0
    for d, line in zip(dets, result["lines"]):
        np.testing.assert_array_equal(np.array(line["polygon"], np.float32), np.array(d.polygon, np.float32))
        assert np.float32(line["detection_score"]) == d.score

    # Recognizer stage, chunk by chunk.
    orec = om.load_recognizer(rec_path, "tiny")
    checked = 0
    for idx, width, contents in opl.recognition_batches(dets):
        n = len(idx)
        recm = P.Recognizer.load(gpu, rec_path, "tiny", (n, 3, 48, width))
        corners = np.array([dets[i].polygon for i in idx], np.float32)
        dev_idx, dev_prob, _ = recm.forward_crops(img, corners, contents)
        x = np.concatenate([opre.prepare_recognizer_crop(rgb, dets[i].polygon, width, c)
                            for i, c in zip(idx, contents)])
        host_idx, host_prob, _ = recm.forward_ctc(x)
        np.testing.assert_array_equal(dev_idx, host_idx)
        np.testing.assert_array_equal(dev_prob, host_prob)
        logits = orec.logits(x)
        want = opost.argmax_last(logits)
        decided = opost.top2_margin(logits) >= CTC_MARGIN
        np.testing.assert_array_equal(dev_idx[decided], want[decided])
        for k, i in enumerate(idx):
            text, score = P.Dictionary.parse("\n".join(entries)).decode_steps(
                dev_idx[k], dev_prob[k], len(entries) + 1, contents[k], width)
            assert result["lines"][i]["text"] == text
            assert abs(result["lines"][i]["recognition_score"] - score) <= 1e-6
            checked += 1
    assert checked == len(dets)
    assert eng.recognize(rgb, fmt="text") == "\n".join(l["text"] for l in result["lines"] if l["text"])


def _png(rgb: np.ndarray) -> bytes:
    h, w = rgb.shape[:2]
    raw = b"".join(b"\x00" + rgb[y].tobytes() for y in range(h))

    def chunk(t, body):
        return struct.pack(">I", len(body)) + t + body + struct.pack(">I", zlib.crc32(t + body) & 0xFFFFFFFF)

    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, 2, 0, 0, 0)) +
            chunk(b"IDAT", zlib.compress(raw)) + chunk(b"IEND", b""))


def test_ppocr_cli_matches_engine(gpu, setup, tmp_path):
    det_path, rec_path, dict_path, entries, rgb = setup
    png = tmp_path / "page.png"
    png.write_bytes(_png(rgb))
    cli = os.path.join(HERE, "..", "ppocr-rs_b200", "ppocr_b200", "ppocr")
    out = subprocess.run([cli, str(png), "--detector-model", det_path, "--recognizer-model", rec_path,
                          "--dictionary", dict_path], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    got = json.loads(out.stdout)
    want = P.Engine(gpu, det_path, rec_path, dict_path).recognize(rgb)
    assert got == want


def test_engine_rejects_mismatched_dictionary(gpu, setup, tmp_path):
    det_path, rec_path, _, _, _ = setup
    d = tmp_path / "short.txt"
    d.write_text("a\nb\n")
    with pytest.raises(P.InvalidInput):
        P.Engine(gpu, det_path, rec_path, str(d))


def test_engine_batch_matches_single_pages(gpu, setup):
    # Pages of two sizes; every page's result from the batched call must equal
    # its own single-page result exactly (crops of all pages share batches).
    det_path, rec_path, dict_path, _, rgb = setup
    pages = [rgb,
             seeded.text_page_rgb8(180, 320, seed=33, blocks=(6, 10), block_h=(12, 28), block_w=(40, 200),
                                   max_angle=15.0, background=(170, 250)),
             seeded.text_page_rgb8(240, 200, seed=34, blocks=(4, 8), block_h=(12, 28), block_w=(40, 150),
                                   max_angle=15.0, background=(170, 250))]
    eng = P.Engine(gpu, det_path, rec_path, dict_path)
    batch = eng.recognize_batch(pages)
    single = [P.Engine(gpu, det_path, rec_path, dict_path).recognize(p) for p in pages]
    assert batch == single
    assert sum(len(r["lines"]) for r in batch) > 0


def test_engine_pool_matches_single_engine(gpu, setup):
    # Two engines on device 0 (two handles, two streams, two host threads)
    # plus, on a multi-GPU box, one per device: pages dealt round-robin must
    # give exactly the single-engine batch results, in page order.
    det_path, rec_path, dict_path, _, rgb = setup
    pages = [rgb] + [seeded.text_page_rgb8(180, 320, seed=40 + i, blocks=(6, 10), block_h=(12, 28),
                                           block_w=(40, 200), max_angle=15.0, background=(170, 250))
                     for i in range(4)]
    expect = P.Engine(gpu, det_path, rec_path, dict_path).recognize_batch(pages)
    devices = [0, 0] + list(range(1, P.gpu_count()))
    pool = P.EnginePool(devices, det_path, rec_path, dict_path)
    assert len(pool) == len(devices)
    assert pool.recognize_batch(pages, timeout_ms=120000) == expect
    assert pool.last_devices == [devices[i % len(devices)] for i in range(len(pages))]
    # A second call reuses every engine's page staging and model cache.
    assert pool.recognize_batch(pages[::-1], fmt="text") == \
        P.Engine(gpu, det_path, rec_path, dict_path).recognize_batch(pages[::-1], fmt="text")
    pool.close()
