"""The C++ seeded checkpoint writer (ppocr_write_seeded_weights, behind
ppocr-gpu-bench --seed-weights) against the Python inventory of the
reference's tensor layout (ppocr_b200.modelspec): same names, same shapes,
and the benchmark configs' spec distributions.  Needs no GPU."""

import math

import numpy as np
import pytest

import ppocr_b200 as P
from ppocr_b200 import modelspec


@pytest.mark.parametrize("kind,size", [("det", "tiny"), ("det", "small"), ("det", "medium"),
                                       ("rec", "tiny"), ("rec", "small"), ("rec", "medium")])
def test_seeded_checkpoint_layout_and_distributions(tmp_path, kind, size):
    from safetensors.numpy import load_file

    path = P.write_seeded_weights(str(tmp_path / "w.safetensors"), kind, size, seed=3)
    got = load_file(path)
    inv = modelspec.inventory(kind, size)
    assert set(got) == set(inv)
    assert len(got) == modelspec.expected_tensor_count(kind, size)
    for name, (shape, role, fan_in) in inv.items():
        v = got[name]
        assert v.shape == tuple(shape), name
        assert v.dtype == np.float32
        if role in ("bn.gamma", "bn.var", "ln.weight"):
            assert np.all(v == 1), name
        elif role in ("bias", "bn.beta", "bn.mean", "ln.bias"):
            assert np.all(v == 0), name
        elif v.size >= 256:
            # rank1 kernels p[o, i] d[i, :] with |d[i]| = 1 keep the same element std.
            want = math.sqrt(2.0 / fan_in) if kind == "det" else 0.02
            assert abs(float(v.std()) - want) <= 0.15 * want, (name, float(v.std()), want)
            assert abs(float(v.mean())) <= 0.2 * want, name
    # Deterministic in (kind, size, seed).
    again = load_file(P.write_seeded_weights(str(tmp_path / "w2.safetensors"), kind, size, seed=3))
    assert all(np.array_equal(got[k], again[k]) for k in got)


def test_seeded_checkpoint_loads(tmp_path):
    """The written file passes the loader's checks (tensor counts, shapes, rank-one form)."""
    for kind, size, shape in (("det", "medium", (1, 3, 64, 64)), ("rec", "tiny", (1, 3, 48, 64))):
        path = P.write_seeded_weights(str(tmp_path / f"{kind}.safetensors"), kind, size, seed=1)
        info = P.inspect_model(path, kind, size, shape)
        assert info["ops"] > 0
