"""ctypes binding of the C++ CPU restatement of the detector (cpu_detector.cpp).

TEST INFRASTRUCTURE ONLY: bench.py's CPU baseline times it beside the torch
port (oracle/model.py); tests/test_cpu_detector.py holds it to the torch port.
Built by `make -C oracle` (g++ -O3 -march=native -fopenmp) into oracle/_build/.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_lib = None


def _host_key() -> str:
    """-march=native code is tied to the host CPU: one build per CPU model."""
    import hashlib

    try:
        with open("/proc/cpuinfo") as f:
            info = [l for l in f if l.startswith(("model name", "flags"))][:2]
    except OSError:
        info = []
    return hashlib.sha1("".join(info).encode()).hexdigest()[:12]


def lib_path() -> str:
    return os.path.join(HERE, "_build", _host_key(), "libcpu_detector.so")


def build() -> str:
    out = lib_path()
    subprocess.run(["make", "-s", "-C", HERE, f"OUT={out}"], check=True)
    return out


def library() -> C.CDLL:
    global _lib
    if _lib is None:
        lib = C.CDLL(build())
        lib.cpu_det_load.argtypes = [C.c_char_p, C.c_int, C.POINTER(C.c_void_p)]
        lib.cpu_det_load.restype = C.c_int
        lib.cpu_det_forward.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_int, C.c_int, C.c_int,
                                        C.POINTER(C.c_float), C.c_int]
        lib.cpu_det_forward.restype = C.c_int
        lib.cpu_det_free.argtypes = [C.c_void_p]
        lib.cpu_det_error.restype = C.c_char_p
        _lib = lib
    return _lib


class CpuDetector:
    """Tiny or small detector on the host cores (images spread over `threads` threads)."""

    SIZES = {"tiny": 0, "small": 1}

    def __init__(self, path: str, size: str):
        if size not in self.SIZES:
            raise ValueError("the C++ restatement covers the tiny and small detectors")
        self._h = C.c_void_p()
        if library().cpu_det_load(str(path).encode(), self.SIZES[size], C.byref(self._h)):
            raise RuntimeError(library().cpu_det_error().decode())

    def forward(self, x: np.ndarray, threads: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        n, c, h, w = x.shape
        out = np.empty((n, 1, h, w), dtype=np.float32)
        fp = C.POINTER(C.c_float)
        if library().cpu_det_forward(self._h, x.ctypes.data_as(fp), n, h, w, out.ctypes.data_as(fp), int(threads)):
            raise RuntimeError(library().cpu_det_error().decode())
        return out

    def __del__(self):
        if getattr(self, "_h", None) and self._h.value:
            library().cpu_det_free(self._h)
            self._h = C.c_void_p()
