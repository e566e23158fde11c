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


def row_metrics_all(ref: np.ndarray, got: np.ndarray):
    """Per-row cosine and per-row max |got - ref| / RMS(ref) (arrays)."""
    ref = np.asarray(ref, np.float64).reshape(ref.shape[0], -1)
    got = np.asarray(got, np.float64).reshape(ref.shape)
    num = (ref * got).sum(1)
    den = np.linalg.norm(ref, axis=1) * np.linalg.norm(got, axis=1)
    cos = np.where(den > 0, num / np.maximum(den, 1e-300), 1.0)
    rms = max(np.sqrt((ref ** 2).mean()), 1e-300)
    return cos, np.abs(got - ref).max(1) / rms


def assert_parity_quantised(ref, got, what="", frac=0.99, cos_floor=0.99):
    """Parity under static input quantisation.  srqScalar rounds x / s to an
    integer code; the device and the oracle sum in different orders (their
    pre-quantisation values agree to ~1e-6 relative), so an element within
    that distance of a half-step rounds the other way and moves by one code
    step (1/127 of the calibration absmax), perturbing the rows that use it.
    Every row keeps cosine >= cos_floor and at least `frac` of the rows meet
    the north-star bound (cosine >= 0.999, max-abs <= 1e-2 * RMS)."""
    assert np.isfinite(np.asarray(got)).all(), f"{what}: non-finite output"
    cos, ma = row_metrics_all(ref, got)
    ok = (cos >= COS_MIN) & (ma <= MAXABS_RMS)
    msg = (f"{what}: {ok.mean() * 100:.2f}% of {ok.size} rows within the north-star bound (>= {frac * 100:.0f}%), "
           f"min row cos {cos.min():.6f} (>= {cos_floor}), max-abs/RMS {ma.max():.3e}")
    print(msg)
    assert ok.mean() >= frac and cos.min() >= cos_floor, msg
    return ok.mean(), cos.min(), ma.max()


def perturbed(x, eps, seed):
    """x * (1 + eps * N(0,1)), float32: a rounding-level input perturbation."""
    x = np.asarray(x, np.float32)
    return (x * (1 + eps * np.random.default_rng(seed).standard_normal(x.shape))).astype(np.float32)


def assert_within_envelope(ref, got, envelope, what="", factor=1.5):
    """Parity for hypersensitive configurations (static input quantisation,
    where a code that rounds the other way moves an input by 1/127 of the
    calibration absmax): the device result must be no farther from the oracle
    than `factor` x the oracle's own distance to itself under input
    perturbations (`envelope`: oracle outputs on perturbed inputs), in the
    fraction of rows meeting the north-star bound, the minimum row cosine and
    the median row max-abs."""
    assert np.isfinite(np.asarray(got)).all(), f"{what}: non-finite output"

    def stats(x):
        cos, ma = row_metrics_all(ref, x)
        return ((cos >= COS_MIN) & (ma <= MAXABS_RMS)).mean(), cos.min(), float(np.median(ma))

    g_ok, g_cos, g_med = stats(got)
    env = [stats(e) for e in envelope]
    e_ok = min(e[0] for e in env)
    e_cos = min(e[1] for e in env)
    e_med = max(e[2] for e in env)
    msg = (f"{what}: device rows ok {g_ok * 100:.1f}% / min cos {g_cos:.6f} / median max-abs {g_med:.2e}; "
           f"oracle envelope {e_ok * 100:.1f}% / {e_cos:.6f} / {e_med:.2e}")
    print(msg)
    assert g_ok >= e_ok / factor or g_ok >= 0.99, msg
    assert (1 - g_cos) <= factor * (1 - e_cos) + 1e-4, msg
    assert g_med <= factor * e_med + 1e-5, msg
    return g_ok, g_cos, g_med


def report(name, **kv):
    print(f"{name}: " + ", ".join(f"{k} {v:.3e}" if isinstance(v, float) else f"{k} {v}" for k, v in kv.items()))


def assert_float64_envelope(oracle_out, device_out, f64_out, what):
    """North-star bound against the oracle, or the device no farther from the
    float64 evaluation than twice the oracle is."""
    assert np.isfinite(device_out).all(), f"{what}: non-finite output"
    cos, ma = row_metrics(oracle_out, device_out)
    d_cos, d_ma = row_metrics(f64_out, device_out)
    o_cos, o_ma = row_metrics(f64_out, oracle_out)
    report(what, dev_vs_oracle_cos=cos, dev_vs_oracle_maxabs=ma, dev_vs_f64_cos=d_cos, dev_vs_f64_maxabs=d_ma,
            oracle_vs_f64_cos=o_cos, oracle_vs_f64_maxabs=o_ma)
    if cos >= COS_MIN and ma <= MAXABS_RMS:
        return cos, ma, d_ma, o_ma
    assert d_ma <= 2 * o_ma and (1 - d_cos) <= 2 * (1 - o_cos) + 1e-9, (
        f"{what}: device vs oracle cos {cos:.6f} max-abs/RMS {ma:.3e} misses the bound, and the device is farther "
        f"from float64 (cos {d_cos:.7f}, max-abs/RMS {d_ma:.3e}) than 2x the oracle (cos {o_cos:.7f}, {o_ma:.3e})")
    return cos, ma, d_ma, o_ma
