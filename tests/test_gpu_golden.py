"""Device path against the committed oracle vectors (tests/golden/
oracle_small.npz): no oracle run needed, north-star tolerance."""
import os
import sys

import numpy as np
import pytest

from conftest import assert_parity

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))


@pytest.fixture(scope="module")
def gold():
    return np.load(os.path.join(HERE, "golden", "oracle_small.npz"))


def test_golden_qat_linears(gold, ctx):
    import make_golden
    x, w, s, b = make_golden.qat_inputs()
    y = ctx.qat_linear(x, w, s, bits=0, bias=b)
    assert_parity(gold["qat_i8/y"], y, what="golden int8 QAT linear")
    xp, wp, sp = make_golden.packed4_inputs()
    yp = ctx.qat_linear(xp, wp, sp, bits=4)
    assert_parity(gold["packed4/y"], yp, what="golden 4-bit packed QAT linear")


def test_golden_towers(gold, native, syn, tmp_path):
    W = dict(syn.vision_weights(0, layers=1))
    W.update(syn.audio_weights(0, layers=1))
    path = str(tmp_path / "golden.safetensors")
    syn.write_safetensors(path, W)
    c = native.Context()
    try:
        c.load_weights(path)
        outs, rows = c.vision_embed([gold["vision48/pixels"]], 1, 1)
        assert rows[0] == 1
        assert_parity(gold["vision48/embedding"], outs[0], what="golden 48x48 image, 1 layer")
        outs, rows = c.audio_embed([gold["audio_tone/samples"]], 16000, 1)
        assert rows[0] == 2
        assert_parity(gold["audio_tone/embeddings"], outs[0], what="golden 0.08 s tone, 1 layer")
    finally:
        c.close()
