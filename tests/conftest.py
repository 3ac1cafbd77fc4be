"""Shared fixtures.  `gpu`-marked tests need a B200 and run through
libhexcuda's C ABI; everything else runs on the CPU."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs through libhexcuda)")
    config.addinivalue_line("markers", "slow: full-size benchmark-shape checks")


def golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o
    o.lib()
    return o


@pytest.fixture(scope="session")
def hx():
    """libhexcuda on device 0 (built in-tree if missing: no fallback)."""
    lib_path = REPO / "hexkernels_b200" / "libhexcuda.so"
    if not lib_path.exists():
        subprocess.run(["make", "-s", "-C", str(REPO / "hexkernels_b200" / "csrc")], check=True)
    from hexkernels_b200 import _lib, ops
    lib = _lib.load()
    n = ops.init(1)
    assert n == 1, "libhexcuda could not initialise device 0"
    return ops


def rel_close(got, exp, rtol, atol):
    """|got - exp| <= atol + rtol * |exp|, elementwise; returns (ok, worst index info)."""
    g = np.asarray(got, np.float64)
    e = np.asarray(exp, np.float64)
    d = np.abs(g - e)
    lim = atol + rtol * np.abs(e)
    bad = d > lim
    return (not bad.any()), int(bad.sum()), float((d / np.maximum(np.abs(e), 1e-30)).max())
