"""GPU parity of the QAT linear boundary (g4m_qat_linear / g4m_linear_*)
against the oracle's runQatI8LinearCpu / runPackedQatLinearCpu restatements."""
import numpy as np
import pytest

from conftest import assert_parity, row_metrics

pytestmark = pytest.mark.gpu


def test_qat_linear_cfg0(ctx, oracle, syn):
    """256 x 768 -> 768 int8 QAT linear with bias, seed 0 (the int8-linear
    benchmark configuration)."""
    x, w, s, b = syn.qat_linear_case(0)
    ref = oracle.add_bias_rows(oracle.qat_i8_linear(x, w, s), b)
    got = ctx.qat_linear(x, w, s, bias=b)
    cos, ma = assert_parity(ref, got, what="cfg0")
    # split-fp16 operands give fp32-grade results: far inside the budget
    assert ma < 1e-4, ma


def test_qat_linear_simt_shapes_exact(ctx, oracle):
    """Shapes outside the tensor-core tiling run the exact-order SIMT kernel:
    bit-identical to the oracle for s_in = s_out = 0."""
    rng = np.random.default_rng(5)
    for rows, inp, out in [(1, 100, 37), (13, 64, 100), (7, 200, 256)]:
        x = rng.standard_normal((rows, inp)).astype(np.float32)
        w = rng.integers(-127, 128, (out, inp)).astype(np.int8)
        s = rng.uniform(0.002, 0.02, out).astype(np.float32)
        got = ctx.qat_linear(x, w, s)
        assert np.array_equal(got, oracle.qat_i8_linear(x, w, s)), (rows, inp, out)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_packed_qat_linear(ctx, oracle, syn, bits):
    rng = np.random.default_rng(bits)
    inp, out, rows = 1024, 512, 250
    codes = rng.integers(0, 2 ** bits, size=(out, inp))
    w = syn.pack_codes(codes, bits) if bits != 8 else codes.astype(np.uint8)
    x = rng.standard_normal((rows, inp)).astype(np.float32)
    s = rng.uniform(0.002, 0.02, out).astype(np.float32)
    ref = oracle.packed_qat_linear(x, w, s, inp, out, bits)
    got = ctx.qat_linear(x, w, s, bits=bits)
    assert_parity(ref, got, what=f"packed {bits}-bit")


def test_packed_qat_simt_exact(ctx, oracle, syn):
    rng = np.random.default_rng(9)
    inp, out, rows, bits = 96, 40, 5, 4
    codes = rng.integers(0, 16, size=(out, inp))
    w = syn.pack_codes(codes, bits)
    x = rng.standard_normal((rows, inp)).astype(np.float32)
    s = rng.uniform(0.002, 0.02, out).astype(np.float32)
    assert np.array_equal(ctx.qat_linear(x, w, s, bits=bits), oracle.packed_qat_linear(x, w, s, inp, out, bits))


def test_qat_linear_activation_quantisation(ctx, oracle, syn):
    """s_in > 0 quantises activations (integer codes on the tensor cores),
    s_out > 0 quantises outputs; one-quantum flips at rounding ties are the
    only allowed differences."""
    x, w, s, _ = syn.qat_linear_case(1, rows=128)
    for s_in, s_out in [(0.03, 0.0), (0.0, 0.4), (0.03, 0.4)]:
        ref = oracle.qat_i8_linear(x, w, s, s_in, s_out)
        got = ctx.qat_linear(x, w, s, s_in, s_out)
        if s_out == 0:
            assert_parity(ref, got, what=f"s_in={s_in}")
        else:
            flips = np.abs(got - ref) > 1e-6
            assert flips.mean() < 1e-3 and np.abs(got - ref).max() <= s_out * 1.001, (s_in, s_out)


def test_qat_linear_rejects_bad_bits(ctx, native):
    x = np.zeros((2, 64), np.float32)
    with pytest.raises(native.G4MError) as e:
        ctx.qat_linear(x, np.zeros((8, 64), np.uint8), np.ones(8, np.float32), bits=3)
    assert e.value.status == 1


def test_linear_prepare_run_device_pointers(ctx, oracle, syn, native):
    import ctypes
    import torch
    x, w, s, b = syn.qat_linear_case(2, rows=512)
    L = native.lib()
    h = ctypes.c_void_p()
    native.check(L.g4m_linear_prepare(ctx.h, 0, native.ptr(w), 0, 768, 768, native.ptr(s), 0.0, 0.0, native.ptr(b),
                                      ctypes.byref(h)))
    try:
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((512, 768), dtype=torch.float32, device="cuda")
        st = torch.cuda.current_stream().cuda_stream
        native.check(L.g4m_linear_run(h, ctypes.c_void_p(xd.data_ptr()), 512, ctypes.c_void_p(yd.data_ptr()),
                                      ctypes.c_void_p(st)))
        torch.cuda.synchronize()
        got = yd.cpu().numpy()
    finally:
        L.g4m_linear_free(h)
    assert_parity(oracle.add_bias_rows(oracle.qat_i8_linear(x, w, s), b), got, what="resident linear")
