import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

PKG = "gemma-4-webgpu-kernels-multimodal_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def g4m():
    return importlib.import_module(PKG)


@pytest.fixture(scope="session")
def syn():
    return importlib.import_module(PKG + ".synthetic")


@pytest.fixture(scope="session")
def native():
    return importlib.import_module(PKG + "._native")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    return O


@pytest.fixture(scope="session")
def ctx(native):
    """A context on cuda:0.  GPU tests use it; it raises if the CUDA library
    or the GPU is missing (no CPU fallback)."""
    c = native.Context()
    yield c
    c.close()


def row_metrics(ref: np.ndarray, got: np.ndarray):
    """(min per-row cosine, max |got - ref| / RMS(ref))."""
    ref = np.asarray(ref, np.float64).reshape(ref.shape[0], -1)
    got = np.asarray(got, np.float64).reshape(ref.shape)
    num = (ref * got).sum(1)
    den = np.linalg.norm(ref, axis=1) * np.linalg.norm(got, axis=1)
    cos = np.where(den > 0, num / np.maximum(den, 1e-300), 1.0)
    rms = np.sqrt((ref ** 2).mean())
    return float(cos.min()), float(np.abs(got - ref).max() / max(rms, 1e-300))


# per-row cosine >= 0.999 and max-abs <= 1e-2 * RMS
COS_MIN = 0.999
MAXABS_RMS = 1e-2


def assert_parity(ref, got, cos_min=COS_MIN, maxabs=MAXABS_RMS, what=""):
    cos, ma = row_metrics(ref, got)
    assert np.isfinite(np.asarray(got)).all(), f"{what}: non-finite output"
    assert cos >= cos_min and ma <= maxabs, f"{what}: min row cos {cos:.6f} (>= {cos_min}), max-abs/RMS {ma:.3e} (<= {maxabs})"
    return cos, ma
