"""ppocr-gpu-bench: the reference's benchmark CLI contract
(src/bin/benchmark.rs:13-57 flags, 194-227 report keys, 229-285 --reference
metrics), run as a subprocess on seeded weights (--seed-weights)."""

import os
import subprocess

import numpy as np
import pytest

import ppocr_b200 as P
from ppocr_b200 import seeded

pytestmark = pytest.mark.gpu

CLI = os.path.join(os.path.dirname(P.__file__), "ppocr-gpu-bench")
REPORT_KEYS = ["backend", "kind", "model", "input_shape", "output_shape", "output_min", "output_max", "output_sum",
               "warmup", "runs", "average_ms", "p50_ms", "p90_ms", "p95_ms", "throughput"]


def run(args, tmp_path):
    r = subprocess.run([CLI] + args, capture_output=True, text=True, timeout=600, env=dict(os.environ, TMPDIR=str(tmp_path)))
    assert r.returncode == 0, r.stderr
    rep = {}
    for line in r.stdout.splitlines():
        k, _, v = line.partition(": ")
        rep[k] = v
    return rep


@pytest.mark.parametrize("kind,size,h,w", [("det", "tiny", 64, 96), ("rec", "tiny", 48, 160)])
def test_cli_report_and_reference(tmp_path, gpu, kind, size, h, w):
    dump = str(tmp_path / "out.f32")
    base = ["--kind", kind, "--model-size", size, "--seed-weights", "7", "--height", str(h), "--width", str(w),
            "--warmup", "1", "--runs", "3"]
    rep = run(base + ["--dump", dump], tmp_path)
    keys = list(rep)
    assert keys[: len(REPORT_KEYS)] == REPORT_KEYS
    assert rep["kind"] == kind and rep["runs"] == "3" and rep["warmup"] == "1"
    assert rep["input_shape"] == f"[1, 3, {h}, {w}]"
    assert float(rep["average_ms"]) > 0 and float(rep["throughput"]) > 0
    # The dump equals this library's forward on the same seeded checkpoint and
    # the generated input (benchmark.rs:126-134).
    weights = os.path.join(str(tmp_path), f"ppocr-seeded-{kind}-{size}-7.safetensors")
    assert rep["model"] == weights
    x = seeded.deterministic_input(3 * h * w).reshape(1, 3, h, w)
    M = P.Detector if kind == "det" else P.Recognizer
    want = M.load(gpu, weights, size, (1, 3, h, w)).forward(x).values
    got = np.fromfile(dump, dtype=np.float32)
    np.testing.assert_array_equal(got, want)
    # --reference against its own dump: zero difference, zero mismatches.
    rep2 = run(base + ["--reference", dump], tmp_path)
    assert float(rep2["reference_max_abs"]) == 0.0 and float(rep2["reference_mean_abs"]) == 0.0
    key = "reference_threshold_0.5_mismatches" if kind == "det" else "reference_argmax_mismatches"
    assert rep2[key] == "0"


def test_cli_gpus_flag(tmp_path, gpu):
    n = P.gpu_count()
    gpus = 2 if n >= 2 else 1
    rep = run(["--kind", "det", "--model-size", "tiny", "--seed-weights", "1", "--height", "64", "--width", "64",
               "--warmup", "1", "--runs", "2", "--batch", "2", "--gpus", str(gpus)], tmp_path)
    assert float(rep["images_per_s"]) > 0
    if gpus > 1:
        assert rep["gpus"] == str(gpus)
        assert float(rep["aggregate_images_per_s"]) > float(rep["images_per_s"])


def test_cli_rejects_model_and_seed(tmp_path):
    r = subprocess.run([CLI, "--kind", "det", "--model", "x.safetensors", "--seed-weights", "1"], capture_output=True,
                       text=True, timeout=60)
    assert r.returncode != 0 and "mutually exclusive" in r.stderr
