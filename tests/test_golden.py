"""The committed golden fixtures (tests/golden/golden.npz) against the oracle and generators.

The fixtures freeze the oracle's answers on small seeded cases; this CPU test
fails when the oracle, the seeded weight generator or the input generators
drift from what produced them.
"""

import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import make_golden as mg  # noqa: E402

GOLDEN = os.path.join(HERE, "golden", "golden.npz")


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="module")
def regenerated():
    return mg.generate()


def test_fixture_keys_complete(golden):
    names = [c[0] for c in mg.DET_CASES] + [c[0] for c in mg.REC_CASES]
    for n in names:
        assert f"{n}.input" in golden and f"{n}.weights_sha256" in golden
    for c in mg.PRE_CASES:
        assert f"{c[0]}.out" in golden


def test_inputs_and_weights_are_reproducible(golden):
    for name, size, profile, (b, h, w, seed, text), _ in mg.DET_CASES:
        np.testing.assert_array_equal(golden[f"{name}.input"], mg.det_input(b, h, w, seed, text))
        assert str(golden[f"{name}.weights_sha256"]) == mg.weights_checksum("det", size, profile)
    for name, size, profile, (b, w, seed) in mg.REC_CASES:
        np.testing.assert_array_equal(golden[f"{name}.input"], mg.rec_input(b, w, seed))
        assert str(golden[f"{name}.weights_sha256"]) == mg.weights_checksum("rec", size, profile)
    np.testing.assert_array_equal(golden["pre.rgb"], mg.pre_image())


def test_oracle_reproduces_golden(golden, regenerated):
    for name, *_ in mg.DET_CASES:
        np.testing.assert_allclose(regenerated[f"{name}.prob"], golden[f"{name}.prob"], rtol=0, atol=1e-5)
    for name, *_ in mg.REC_CASES:
        np.testing.assert_allclose(regenerated[f"{name}.logits_strided"], golden[f"{name}.logits_strided"],
                                   rtol=0, atol=1e-5)
        np.testing.assert_array_equal(regenerated[f"{name}.argmax"], golden[f"{name}.argmax"])
        np.testing.assert_array_equal(regenerated[f"{name}.ctc_classes"], golden[f"{name}.ctc_classes"])
    for c in mg.PRE_CASES:
        np.testing.assert_array_equal(regenerated[f"{c[0]}.out"], golden[f"{c[0]}.out"])


def test_golden_cases_exercise_the_decoder(golden):
    # The CTC fixture must contain emitted classes, and the masks must contain both values,
    # otherwise the comparisons built on them are vacuous.
    for name, *_ in mg.REC_CASES:
        assert golden[f"{name}.ctc_classes"].size > 0
    for name, *_ in mg.DET_CASES:
        m = golden[f"{name}.mask"]
        assert 0 < m.sum() < m.size, name
