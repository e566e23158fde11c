"""The oracle against its committed seeded vectors (tests/golden/make_golden.py):
the seeded generators must reproduce the same inputs (byte checksums) and the
oracle the same outputs (to f32 rounding; libm may differ between hosts)."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(HERE, "golden", "oracle_small.npz"))


@pytest.fixture(scope="module")
def mk():
    import make_golden
    return make_golden


def test_seeded_inputs_unchanged(gold, mk):
    assert int(mk.input_checksum(*mk.qat_inputs())) == int(gold["qat_i8/input_checksum"])
    assert int(mk.input_checksum(*mk.packed4_inputs())) == int(gold["packed4/input_checksum"])


def test_oracle_reproduces_golden(gold, mk):
    c = mk.cases()
    for k in ("qat_i8/y", "packed4/y", "vision48/embedding", "audio_tone/embeddings", "logmel/features"):
        ref = gold[k].astype(np.float64)
        got = c[k].astype(np.float64)
        assert got.shape == ref.shape, k
        scale = max(np.abs(ref).max(), 1e-30)
        assert np.abs(got - ref).max() <= 1e-5 * scale, k
    assert gold["vision48/embedding"].shape == (1, 1536)  # 48 x 48, maxSoftTokens 1 -> one token
    assert gold["audio_tone/embeddings"].shape == (2, 1536)  # 0.08 s -> 2 rows
