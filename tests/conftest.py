"""Shared test configuration.

Markers: `gpu` tests need a B200 and call the CUDA library through its C ABI; everything else
runs on the CPU (oracle pins, golden fixtures, ABI symbol table, host-side sharding logic).
"""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

# The parity bar: fp16 storage, fp32 accumulation, element passes when
# |x - r| <= ATOL + RTOL * |r| (max-abs 2e-3 / max-rel 1e-2).
ATOL = 2e-3
RTOL = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def assert_close(x, r, atol=ATOL, rtol=RTOL, what=""):
    x = np.asarray(x, np.float64)
    r = np.asarray(r, np.float64)
    assert x.shape == r.shape, (x.shape, r.shape)
    assert np.isfinite(x).all(), f"{what}: non-finite output"
    err = np.abs(x - r)
    bad = err > atol + rtol * np.abs(r)
    big = np.abs(r) > 1e-3
    max_rel = float((err[big] / np.abs(r[big])).max()) if big.any() else 0.0
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} elements out of tolerance; "
                           f"max-abs {err.max():.3e} max-rel {max_rel:.3e}")
    return float(err.max()), max_rel


@pytest.fixture(scope="session")
def oracle():
    from oracle import pyoracle
    pyoracle.lib()
    return pyoracle


@pytest.fixture(scope="session")
def golden_dir():
    return ROOT / "tests" / "golden"
