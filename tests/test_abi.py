"""C-ABI library: exports and host-side loader behaviour (no GPU needed).

The loader checks mirror gpu::Weights / gpu::Detector::load /
gpu::Recognizer::load (src/gpu/weights.rs:28-155, src/gpu/model.rs:50-93,
156-220, 268-286); ppocr_inspect_model runs them without a device.
"""

import json
import os
import re
import struct

import numpy as np
import pytest

import ppocr_b200 as P
from ppocr_b200 import modelspec, seeded

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "ppocr_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ppocr_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_function():
    lib = P.library()
    names = header_functions()
    assert len(names) >= 30
    for name in names:
        assert hasattr(lib, name), f"{name} declared in include/ppocr_b200.h but not exported"


def test_gpu_count_and_create_without_device():
    n = P.gpu_count()
    assert n >= 0
    if n == 0:
        with pytest.raises(P.GpuError):
            P.Gpu(0)
    assert P.library().ppocr_last_error() is not None


def write_safetensors(path, tensors, dtype_override=None, offset_skew=None, byte_trim=None):
    """Minimal safetensors writer that can emit malformed files for the error tests."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr)
        data = a.tobytes()
        dtype = {np.float32: "F32", np.float16: "F16"}[a.dtype.type]
        if dtype_override and name in dtype_override:
            dtype = dtype_override[name]
        end = off + len(data)
        if byte_trim and name in byte_trim:
            end -= byte_trim[name]
            data = data[: len(data) - byte_trim[name]]
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, end]}
        blobs.append(data)
        off = end
    if offset_skew:
        name, extra = offset_skew
        header[name]["data_offsets"][1] += extra
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


@pytest.mark.parametrize("kind,size,shape,out", [
    ("det", "tiny", (2, 3, 416, 736), [2, 1, 416, 736]),
    ("det", "small", (1, 3, 64, 96), [1, 1, 64, 96]),
    ("det", "medium", (1, 3, 128, 160), [1, 1, 128, 160]),
    ("rec", "tiny", (3, 3, 48, 320), [3, 40, 6906]),
    ("rec", "small", (1, 3, 48, 160), [1, 20, 18710]),
    ("rec", "medium", (2, 3, 48, 480), [2, 60, 18710]),
])
def test_inspect_builds_every_tier(weights_file, kind, size, shape, out):
    for precision in ("fp32", "bf16"):
        info = P.inspect_model(weights_file(kind, size), kind, size, shape, precision)
        assert info["output_shape"] == out
        assert info["ops"] > 20 and info["arena_bytes"] > 0 and info["weight_bytes"] > 0


def test_missing_file_is_read_file_error(tmp_path):
    with pytest.raises(P.ReadFile):
        P.inspect_model(str(tmp_path / "nope.safetensors"), "det", "tiny", (1, 3, 32, 32))


def test_garbage_is_safetensors_error(tmp_path):
    p = tmp_path / "bad.safetensors"
    p.write_bytes(b"\x05\x00\x00\x00\x00\x00\x00\x00{oops")
    with pytest.raises(P.Safetensors):
        P.inspect_model(str(p), "det", "tiny", (1, 3, 32, 32))
    p.write_bytes(b"\x01\x02")
    with pytest.raises(P.Safetensors):
        P.inspect_model(str(p), "det", "tiny", (1, 3, 32, 32))


def _tiny_det():
    return seeded.make_weights("det", "tiny", 0, "spec")


def test_tensor_count_is_invalid_model(tmp_path):
    w = _tiny_det()
    w.pop(next(iter(w)))
    p = tmp_path / "short.safetensors"
    write_safetensors(p, w)
    with pytest.raises(P.InvalidModel, match="271"):
        P.inspect_model(str(p), "det", "tiny", (1, 3, 32, 32))


def test_renamed_tensor_is_not_found(tmp_path):
    w = _tiny_det()
    name = "head.conv_final.bias"
    w["head.conv_final.renamed"] = w.pop(name)
    p = tmp_path / "renamed.safetensors"
    write_safetensors(p, w)
    with pytest.raises(P.TensorNotFound, match="conv_final"):
        P.inspect_model(str(p), "det", "tiny", (1, 3, 32, 32))


def test_half_tensor_is_unsupported_dtype(tmp_path):
    w = _tiny_det()
    w["head.conv_final.bias"] = w["head.conv_final.bias"].astype(np.float16)
    p = tmp_path / "half.safetensors"
    write_safetensors(p, w)
    with pytest.raises(P.UnsupportedDtype):
        P.inspect_model(str(p), "det", "tiny", (1, 3, 32, 32))


def test_wrong_shape_is_shape_mismatch(tmp_path):
    w = _tiny_det()
    w["head.conv_final.bias"] = np.zeros(2, np.float32)
    p = tmp_path / "shape.safetensors"
    write_safetensors(p, w)
    with pytest.raises(P.ShapeMismatch):
        P.inspect_model(str(p), "det", "tiny", (1, 3, 32, 32))


def test_byte_length_and_range_errors(tmp_path):
    w = _tiny_det()
    p = tmp_path / "trim.safetensors"
    write_safetensors(p, w, byte_trim={"head.conv_final.bias": 2})
    with pytest.raises(P.TensorByteLength):
        P.inspect_model(str(p), "det", "tiny", (1, 3, 32, 32))
    names = list(w)
    q = tmp_path / "range.safetensors"
    write_safetensors(q, w, offset_skew=(names[-1], 1 << 20))
    with pytest.raises(P.InvalidTensorRange):
        P.inspect_model(str(q), "det", "tiny", (1, 3, 32, 32))


def test_nonseparable_medium_neck_is_invalid_model(tmp_path):
    w = seeded.make_weights("det", "medium", 0, "spec")
    name = "model.neck.input_feature_projection_convolution.2.weight"
    w[name] = w[name] + np.random.default_rng(0).normal(0, 0.1, w[name].shape).astype(np.float32)
    p = tmp_path / "dense9.safetensors"
    write_safetensors(p, w)
    with pytest.raises(P.InvalidModel, match="rank-one"):
        P.inspect_model(str(p), "det", "medium", (1, 3, 64, 64))


@pytest.mark.parametrize("kind,shape", [
    ("det", (0, 3, 64, 64)), ("det", (1, 1, 64, 64)), ("det", (1, 3, 63, 64)), ("det", (1, 3, 64, 16)),
    ("rec", (1, 3, 32, 320)), ("rec", (1, 3, 48, 30)), ("rec", (1, 3, 48, 322)), ("rec", (0, 3, 48, 320)),
])
def test_input_shape_rules(weights_file, kind, shape):
    size = "tiny"
    with pytest.raises(P.InvalidInput):
        P.inspect_model(weights_file(kind, size), kind, size, shape)


def test_seeded_inventory_matches_reference_counts():
    # tensor counts of src/gpu/model.rs:11-16, parameter totals of models.json byte sizes
    totals = {("det", "tiny"): 437517, ("det", "small"): 2475373, ("det", "medium"): 21993025,
              ("rec", "tiny"): 1113470, ("rec", "medium"): 19176118}
    for kind in ("det", "rec"):
        for size in ("tiny", "small", "medium"):
            inv = modelspec.inventory(kind, size)
            assert len(inv) == modelspec.expected_tensor_count(kind, size)
            if (kind, size) in totals:
                assert sum(int(np.prod(s)) for s, _, _ in inv.values()) == totals[(kind, size)]


def test_seeded_weights_are_deterministic():
    a = seeded.make_weights("rec", "tiny", 7, "conditioned")
    b = seeded.make_weights("rec", "tiny", 7, "conditioned")
    assert all(np.array_equal(a[k], b[k]) for k in a)
    c = seeded.make_weights("rec", "tiny", 8, "conditioned")
    assert not np.array_equal(a["head.fc2.weight"], c["head.fc2.weight"])


def test_deterministic_input_matches_lcg():
    # src/bin/benchmark.rs:126-134
    v = seeded.deterministic_input(4)
    state, want = 0x243F6A88, []
    for _ in range(4):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        want.append(np.float32(np.float32(state >> 8) / np.float32(0xFFFFFF)) * np.float32(2) - np.float32(1))
    np.testing.assert_array_equal(v, np.array(want, np.float32))
    assert np.all(v >= -1) and np.all(v < 1)
