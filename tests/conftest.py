import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "ppocr-rs_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device")


_CACHE = {}


@pytest.fixture(scope="session")
def weights_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("weights")


@pytest.fixture(scope="session")
def weights_file(weights_dir):
    """weights_file(kind, size, profile='spec', seed=0) -> path of a seeded checkpoint."""
    from ppocr_b200 import seeded

    def make(kind, size, profile="spec", seed=0):
        key = (kind, size, profile, seed)
        if key not in _CACHE:
            path = weights_dir / f"{kind}_{size}_{profile}_{seed}.safetensors"
            seeded.write_weights(str(path), kind, size, seed, profile)
            _CACHE[key] = str(path)
        return _CACHE[key]

    return make


@pytest.fixture(scope="session")
def gpu():
    import ppocr_b200 as P

    g = P.Gpu(0)
    yield g
    g.close()
