"""Shared pytest setup.

Markers: ``gpu`` -- needs a CUDA device and the built ``libnova_b200.so``
(run with ``-m gpu`` on a B200); everything else runs on the CPU.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built CUDA library")


def golden(name: str) -> dict:
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


def fp16_ulp(want: np.ndarray) -> np.ndarray:
    """Spacing of fp16 at each element of ``want`` (tests/test_kvattn.py:74-78)."""
    w = np.asarray(want, np.float16)
    up = np.abs(np.nextafter(w, np.float16(np.inf)).astype(np.float32) - w.astype(np.float32))
    return np.maximum(up, np.float32(2.0 ** -24))


def assert_ulp_or_abs(got, want, max_ulp: float, abs_tol: float, tag: str = "") -> dict:
    """The reference's attention criterion: each element within ``max_ulp`` fp16
    ULP of ``want`` or within ``abs_tol`` absolute (tests/test_kvattn.py:83-94)."""
    got = np.asarray(got, np.float32)
    want32 = np.asarray(want, np.float32)
    diff = np.abs(got - want32)
    ulp = diff / fp16_ulp(want)
    bad = (ulp > max_ulp) & (diff > abs_tol)
    assert not bad.any(), (f"{tag}: {int(bad.sum())} elements beyond {max_ulp} ULP and {abs_tol:g} abs "
                           f"(max {ulp.max():.2f} ULP, max abs {diff.max():.3e})")
    return {"max_ulp": float(ulp.max()), "max_abs": float(diff.max()), "exact": float((diff == 0).mean())}


@pytest.fixture(scope="session")
def cuda_lib():
    """Loads the CUDA library and skips when no GPU is present.  Used only by
    ``gpu``-marked tests; on a GPU machine a missing library is an error."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nova_b200 import _lib

    return _lib.lib()
