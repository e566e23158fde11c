"""Failure detection without a GPU fault: a device wait that runs out (a
barrier nothing arrives on, short budget) comes back as G4M_E_TIMEOUT and the
context keeps working; cancellation between layers (the reference's
AbortSignal checks, src/vision/encoder.ts:179) comes back as G4M_E_CANCELLED."""
import numpy as np
import pytest

from conftest import assert_parity

pytestmark = pytest.mark.gpu


def test_bounded_wait_timeout_then_recovery(ctx, native, syn, oracle):
    L = native.lib()
    rc = L.g4m_selftest_wait_timeout(ctx.h, 0, 2_000_000)  # ~1 ms of SM clock
    assert rc == 5 and "kernel error code 1" in native.last_error()
    x, w, s, b = syn.qat_linear_case(0, rows=64)
    y = ctx.qat_linear(x, w, s, bias=b)  # the error word was cleared: the context still works
    assert_parity(oracle.add_bias_rows(oracle.qat_i8_linear(x, w, s), b), y, what="linear after a timeout")
    assert L.g4m_selftest_wait_timeout(ctx.h, 0, 0) == 1  # budget must be positive


def test_cancel_between_layers(native, syn, tmp_path):
    W = syn.vision_weights(0, layers=2)
    path = str(tmp_path / "v2.safetensors")
    syn.write_safetensors(path, W)
    c = native.Context()
    try:
        c.load_weights(path)
        pix = syn.image_pixels(0, 96, 96)
        c.cancel()
        with pytest.raises(native.G4MError) as e:
            c.vision_embed([pix], 4, 2)
        assert e.value.status == 6
        c.clear_cancel()
        outs, rows = c.vision_embed([pix], 4, 2)
        assert rows[0] == 4 and np.isfinite(outs[0]).all()
    finally:
        c.close()
