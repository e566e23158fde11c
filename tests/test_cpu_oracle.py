"""CPU tests: the oracle against the reference's literal probe examples and
against an independent numpy restatement (tests/np_ref.py)."""
import json
import os

import numpy as np
import pytest

import np_ref

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def close(a, b, rtol):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    scale = max(np.abs(b).max(), 1e-30)
    return float(np.abs(a - b).max() / scale) <= rtol


# ---------------------------------------------------------------- integer pins

def test_integer_pins_from_reference_probes(oracle):
    pins = json.load(open(os.path.join(GOLD, "integer_pins.json")))
    for case in pins["image_layouts"]:
        got = oracle.image_token_layout(case["height"], case["width"], case["patchSize"], case["maxSoftTokens"],
                                        case["poolingKernelSize"])
        exp = case["expected"]
        assert got["target"] == exp["target"], case
        assert got["patchGrid"] == exp["patchGrid"], case
        assert got["maxPatches"] == exp["maxPatches"] and got["softTokens"] == exp["softTokens"], case
    for case in pins["audio_soft_tokens"]:
        assert oracle.audio_soft_token_count(case["samples"], 320, 160, 750) == case["expected"], case


def test_layout_errors(oracle):
    with pytest.raises(oracle.LayoutError, match="positive"):
        oracle.image_token_layout(0, 10)
    with pytest.raises(oracle.LayoutError, match="0 x 0"):
        oracle.image_token_layout(1, 1, 16, 0, 3)


def test_soft_tokens_from_mask_matches_count(oracle):
    # a fully valid mask of F frames gives the same token count as the formula
    for n in [320, 1280, 16000, 80000, 160000, 479999, 480000]:
        pre = oracle.preprocess_audio(np.zeros(n, np.float32) + 0.01, pad_to_multiple_of=None)
        assert pre["softTokens"] == oracle.audio_soft_token_count(n)


def test_checksum_semantics(oracle):
    v = np.array([0.5e-6, -0.5e-6, 1.25, -3.0000005, 1e3], np.float32)
    # Math.round ties toward +infinity: round(0.5) = 1, round(-0.5) = -0
    c = 0.0
    for i, x in enumerate(v):
        y = float(x) * 1e6
        r = np.floor(y)
        r = r + 1 if y - r >= 0.5 else r
        c = np.fmod(c + r * (i + 1), 1000000007.0)
        c = c + 1000000007.0 if c < 0 else c
    assert oracle.checksum_floats(v) == int(c)


# ---------------------------------------------------- numpy cross-checks

def test_qat_i8_linear(oracle, syn):
    x, w, s, _ = syn.qat_linear_case(0, rows=16, inp=768, out=256)
    for s_in, s_out in [(0.0, 0.0), (0.03, 0.0), (0.0, 0.5), (0.03, 0.5)]:
        got = oracle.qat_i8_linear(x, w, s, s_in, s_out)
        ref = np_ref.qat_i8(x, w, s, s_in, s_out)
        if s_out == 0:
            assert close(got, ref, 1e-5), (s_in, s_out)
        else:  # output quantisation: allow rare one-quantum flips at rounding ties
            assert np.mean(np.abs(got - ref) > 1e-6) < 1e-3


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_packed_qat_linear(oracle, syn, bits):
    rng = np.random.default_rng(bits)
    inp, out = 256, 64
    codes = rng.integers(0, 2 ** bits, size=(out, inp))
    w = syn.pack_codes(codes, bits) if bits != 8 else codes.astype(np.uint8)
    assert oracle.derive_packed_bits(w.nbytes, inp, out) == bits
    x = rng.standard_normal((8, inp)).astype(np.float32)
    s = rng.uniform(0.002, 0.02, out).astype(np.float32)
    got = oracle.packed_qat_linear(x, w, s, inp, out, bits)
    ref = np_ref.packed_qat(x, w, s, inp, bits)
    assert close(got, ref, 1e-4)
    for o, c in [(3, 5), (63, 255)]:
        assert oracle.lib().g4mo_packed_weight_code(oracle._p(np.ascontiguousarray(w)), o, c, inp, bits) == codes[o, c]


def test_rmsnorm_rope_attention(oracle):
    rng = np.random.default_rng(1)
    rows, heads, hd = 36, 12, 64
    x = rng.standard_normal((rows, 768)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(768)).astype(np.float32)
    assert close(oracle.rmsnorm(x, w), np_ref.rmsnorm(x, w), 1e-6)
    pos = np.stack(np.divmod(np.arange(rows), 6)[::-1], 1).astype(np.int32)
    assert close(oracle.vision_rope(x, pos, heads, hd), np_ref.rope(x, pos, heads, hd), 1e-6)
    q, k, v = (rng.standard_normal((rows, 768)).astype(np.float32) for _ in range(3))
    assert close(oracle.vision_attention(q, k, v, heads, hd), np_ref.attention(q, k, v, heads, hd), 1e-5)


def test_gelu_pool_patch_embedder(oracle):
    rng = np.random.default_rng(2)
    g, u = rng.standard_normal((2, 50)).astype(np.float32) * 3
    assert close(oracle.gelu_gate(g, u), np_ref.gelu_gate(g, u), 1e-6)
    gh, gw = 6, 9
    h = rng.standard_normal((gh * gw, 768)).astype(np.float32)
    pos = np.stack(np.divmod(np.arange(gh * gw), gw)[::-1], 1).astype(np.int32)
    assert close(oracle.vision_pooler(h, pos, (gh // 3) * (gw // 3)), np_ref.pooler(h, gh, gw), 1e-6)
    patches = rng.uniform(0, 1, (gh * gw, 768)).astype(np.float32)
    pw = (0.02 * rng.standard_normal((768, 768))).astype(np.float32)
    px = (0.02 * rng.standard_normal((gw, 768))).astype(np.float32)
    py = (0.02 * rng.standard_normal((gh, 768))).astype(np.float32)
    assert close(oracle.vision_patch_embed(patches, pw, pos, px, py), np_ref.patch_embed(patches, pw, pos, px, py), 1e-6)
    ew = (0.02 * rng.standard_normal((1536, 768))).astype(np.float32)
    assert close(oracle.embedder(h[:4], ew), np_ref.embedder(h[:4], ew), 1e-6)


def test_audio_kernels(oracle):
    rng = np.random.default_rng(3)
    # subsample conv with a masked tail
    t, f = 21, 16
    x = rng.standard_normal(t * f).astype(np.float32)
    mask = np.ones(t, np.uint8)
    mask[17:] = 0
    w = (0.1 * rng.standard_normal((8, 1, 3, 3))).astype(np.float32)
    nw = (1 + 0.02 * rng.standard_normal(8)).astype(np.float32)
    y, m, ot, of = oracle.audio_subsample_conv_layer(x, mask, t, f, 1, w, nw, 8)
    yr, mr = np_ref.subsample_conv(x, mask, t, f, 1, w, nw, 8)
    assert (m == mr).all() and close(y, yr, 1e-5)
    assert close(oracle.audio_relpos(13, 1024), np_ref.relpos(13, 1024), 1e-6)
    rows, heads, hd = 30, 8, 128
    q, k, v = (rng.standard_normal((rows, heads * hd)).astype(np.float32) * 0.5 for _ in range(3))
    rk = rng.standard_normal((13, heads * hd)).astype(np.float32) * 0.5
    pds = (0.1 * rng.standard_normal(hd)).astype(np.float32)
    got = oracle.audio_attention(q, k, v, rk, pds, heads, hd)
    assert close(got, np_ref.audio_attention(q, k, v, rk, pds, heads, hd), 1e-5)
    g = rng.standard_normal((rows, 2048)).astype(np.float32)
    assert close(oracle.glu(g, 1024), g[:, :1024] / (1 + np.exp(-g[:, 1024:].astype(np.float64))), 1e-6)
    dw = rng.standard_normal((1024, 1, 5)).astype(np.float32)
    assert close(oracle.depthwise_causal(g[:, :1024], dw), np_ref.depthwise(g[:, :1024], dw), 1e-5)


def test_logmel_against_numpy_fft(oracle, syn):
    x = syn.audio_samples(0, 16000)
    pre = oracle.preprocess_audio(x, pad_to_multiple_of=None)
    ref = np_ref.logmel(x)
    assert pre["frames"] == ref.shape[0] == 99 and pre["validFrames"] == 99
    assert np.abs(pre["inputFeatures"] - ref).max() < 2e-4


def test_preprocess_audio_padding_mask(oracle):
    # padding to a multiple of 128 samples adds frames whose mask is 0 and
    # whose features are 0 (src/preprocess/audio.ts:45-52, 98-105)
    x = np.full(1000, 0.1, np.float32)
    a = oracle.preprocess_audio(x, pad_to_multiple_of=None)
    b = oracle.preprocess_audio(x, pad_to_multiple_of=128)
    assert b["frames"] >= a["frames"] and b["validFrames"] == a["validFrames"]
    assert (b["inputFeatures"][b["inputFeaturesMask"] == 0] == 0).all()
    assert np.array_equal(a["inputFeatures"], b["inputFeatures"][: a["frames"]])
