"""Shared test setup.

Markers: ``gpu`` -- needs a B200 (run with ``-m gpu``); everything else runs on
CPU.  The CPU checker (oracle/) and the library are built on first use if
missing (both build without a GPU).
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

# Parity bar from the task's north star: routing bit-exact; outputs within
# max-abs 2e-2 and relative 1e-2 of the fp32 reference.
ATOL = 2e-2
RTOL = 1e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a)")


def _ensure_oracle():
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True,
                       capture_output=True)


def _ensure_lib():
    if not os.path.exists(os.path.join(ROOT, "overhang_b200", "libomc.so")):
        from overhang_b200 import build
        build.build()


@pytest.fixture(scope="session")
def oracle():
    _ensure_oracle()
    import pyoracle
    return pyoracle


@pytest.fixture(scope="session")
def omc_lib():
    _ensure_lib()
    import overhang_b200
    return overhang_b200


@pytest.fixture(scope="session")
def gpu(omc_lib):
    """Initialised library on cuda:0 (GPU tests only).  Every test uploads its
    own layers and the slab only grows (it is a bump allocator), so the
    session's budget covers the whole suite: 120 GiB of the B200's 180."""
    omc_lib.init(0, 120 << 30)
    yield omc_lib


# The bounded router (the default for T >= 16 on OLMoE- and Qwen-family
# layers) keeps the indices bit-exact; its routing weights differ from the
# reference's by a few ulps (the softmax sum includes approximated logits of
# experts that cannot be selected).  This is the bar for them.
WREL = 2e-5


def assert_weights(w, rw, exact, what="routing weights"):
    """exact: bit-equal; else max |w - rw| / |rw| <= WREL."""
    import numpy as np
    if exact:
        assert np.array_equal(w.view(np.uint32), rw.view(np.uint32)), f"{what} differ"
        return
    d = np.abs(w.astype(np.float64) - rw.astype(np.float64)) / np.maximum(np.abs(rw.astype(np.float64)), 1e-30)
    mx = float(d.max()) if d.size else 0.0
    assert mx <= WREL, f"{what}: max relative difference {mx:.3e} (<= {WREL})"


def assert_close(got, want, atol=ATOL, rtol=RTOL, what="output"):
    """max|got-want| <= atol and max|got-want| / max|want| <= rtol."""
    import numpy as np
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    mx = float(d.max()) if d.size else 0.0
    scale = float(np.abs(want).max()) if want.size else 1.0
    rel = mx / max(scale, 1e-30)
    assert np.all(np.isfinite(got)), f"{what}: non-finite values"
    assert mx <= atol and rel <= rtol, f"{what}: max-abs {mx:.3e} (<= {atol}), rel {rel:.3e} (<= {rtol})"
    return mx, rel
