"""Generate tests/golden/golden.npz: committed oracle outputs for small seeded cases.

    python tests/golden/make_golden.py

The Rust reference cannot run in this environment (no Rust toolchain, and its
GPU path needs Vulkan), so these fixtures are produced by the CPU restatement
under oracle/ from seeded inputs and seeded random-init weights in the
reference checkpoint layout.  They freeze the oracle's answers so that

* the CPU suite detects any drift of the oracle, the weight generator or the
  input generators (tests/test_golden.py), and
* the GPU suite compares the CUDA path against fixed numbers that do not
  depend on the checker running beside it (tests/test_gpu_golden.py).

Every model case records the weight checksum (sha256 over the sorted tensor
names and raw bytes of seeded.make_weights), so a fixture can never be
compared against a checkpoint other than the one that produced it.
"""

from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (os.path.join(ROOT, "ppocr-rs_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

from ppocr_b200 import seeded  # noqa: E402

OUT = os.path.join(HERE, "golden.npz")

# (name, kind, size, profile, seed, input builder, float64?)
DET_CASES = [
    ("det_tiny_conditioned", "tiny", "conditioned", (1, 64, 96, 11, True), False),
    ("det_small_conditioned", "small", "conditioned", (1, 64, 96, 12, True), False),
    ("det_medium_conditioned", "medium", "conditioned", (1, 64, 96, 13, True), False),
    # The spec-weight tiny detector is chaotic in FP32; its reference answer is
    # the float64 evaluation of the same graph.
    ("det_tiny_spec_f64", "tiny", "spec", (1, 64, 96, 14, False), True),
]
REC_CASES = [
    ("rec_tiny_conditioned", "tiny", "conditioned", (1, 64, 21)),
    ("rec_medium_conditioned", "medium", "conditioned", (1, 64, 22)),
]
# Every REC_STRIDE-th class of the medium recognizer's 18,710 logits is kept
# (plus the per-step arg-max and margin) to keep the fixture small.
REC_STRIDE = {"tiny": 1, "medium": 16}

PRE_IMAGE = (57, 83, 5)   # height, width, seed
PRE_CASES = [
    ("pre_det_full", [(0, 0), (83, 0), (83, 57), (0, 57)], 96, 64, 96, "det"),
    ("pre_rec_quad", [(3.5, 2.25), (70.0, 6.0), (66.5, 50.0), (1.0, 44.0)], 48, 80, 120, "rec"),
    ("pre_rec_steep", [(10, 40), (80, 20), (82, 30), (12, 50)], 48, 100, 160, "rec"),
]


def weights_checksum(kind: str, size: str, profile: str, seed: int = 0) -> str:
    h = hashlib.sha256()
    tensors = seeded.make_weights(kind, size, seed, profile)
    for name in sorted(tensors):
        h.update(name.encode())
        h.update(np.ascontiguousarray(tensors[name]).tobytes())
    return h.hexdigest()


def det_input(batch, h, w, seed, text):
    return seeded.det_batch(batch, h, w, seed, text=text)


def rec_input(batch, w, seed):
    return seeded.rec_batch(batch, w, seed, min_width=32)


def pre_image():
    h, w, seed = PRE_IMAGE
    return np.random.default_rng(seed).integers(0, 256, size=(h, w, 3), dtype=np.uint8)


def generate() -> dict:
    import torch

    from oracle import model as om
    from oracle import postprocess as opost
    from oracle import preprocess as opre

    torch.manual_seed(0)
    out = {}
    for name, size, profile, (b, h, w, seed, text), f64 in DET_CASES:
        weights = om.Weights(seeded.make_weights("det", size, 0, profile))
        x = det_input(b, h, w, seed, text)
        if f64:
            with om.compute_dtype(torch.float64):
                prob = om.Detector(weights, size).forward(x)
            # FP32 rounding noise of the network itself: the oracle's own float32
            # evaluation against the float64 one.
            f32_prob = om.Detector(weights, size).forward(x)
            out[f"{name}.oracle_f32_err"] = np.array(np.abs(f32_prob - prob).max(), dtype=np.float32)
        else:
            prob = om.Detector(weights, size).forward(x)
        out[f"{name}.input"] = x
        out[f"{name}.prob"] = prob.astype(np.float32)
        # The conditioned maps sit near 0.5, so their mask threshold is the map's
        # median (3 decimals) to give a mask with both values; spec maps use 0.2.
        thr = 0.2 if f64 else round(float(np.median(prob)), 3)
        out[f"{name}.threshold"] = np.array(thr, dtype=np.float32)
        out[f"{name}.mask"] = opost.db_mask(prob, thr)
        out[f"{name}.weights_sha256"] = np.array(weights_checksum("det", size, profile))
    for name, size, profile, (b, w, seed) in REC_CASES:
        weights = om.Weights(seeded.make_weights("rec", size, 0, profile))
        x = rec_input(b, w, seed)
        logits = om.Recognizer(weights, size).logits(x)
        out[f"{name}.input"] = x
        out[f"{name}.logits_strided"] = logits[..., ::REC_STRIDE[size]].astype(np.float32)
        out[f"{name}.argmax"] = opost.argmax_last(logits).astype(np.int32)
        out[f"{name}.margin"] = opost.top2_margin(logits)
        out[f"{name}.max_logit"] = logits.max(axis=-1).astype(np.float32)
        out[f"{name}.weights_sha256"] = np.array(weights_checksum("rec", size, profile))
        probs = om.softmax(om.t(logits)).numpy()
        text, score, classes = opost.decode_ctc_greedy(probs[0], seeded.synthetic_dictionary(size), w, w)
        out[f"{name}.ctc_classes"] = np.array(classes, dtype=np.int32)
        out[f"{name}.ctc_score"] = np.array(score, dtype=np.float64)
    rgb = pre_image()
    out["pre.rgb"] = rgb
    for name, corners, h, content, w, kind in PRE_CASES:
        mean, std = ((opre.DETECTOR_MEAN_BGR, opre.DETECTOR_STD_BGR) if kind == "det"
                     else (opre.RECOGNIZER_MEAN_BGR, opre.RECOGNIZER_STD_BGR))
        out[f"{name}.out"] = opre.normalized_bgr(rgb, corners, w, h, content, mean, std)
    return out


def main() -> None:
    data = generate()
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT}: {len(data)} arrays, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
