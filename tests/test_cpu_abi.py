"""CPU tests of the C ABI library: it loads, exports every symbol declared in
include/g4m.h, and its host-side helpers (no GPU work) are bit-exact with
the oracle."""
import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "g4m.h")).read()
    return sorted(set(re.findall(r"G4M_API\s+[\w\s\*]+?\b(g4m_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol(native):
    L = native.lib()
    names = declared_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    # the Python bindings cover exactly the declared ABI
    assert sorted(native.exported_names()) == names
    assert native.version().startswith("g4m sm_100a")


def test_image_layout_matches_oracle(native, oracle):
    rng = np.random.default_rng(0)
    cases = [(1024, 768, 280), (48, 48, 1), (1, 1000, 280), (1000, 1, 280), (7, 13, 70), (4000, 3000, 280)]
    cases += [(int(h), int(w), int(s)) for h, w, s in zip(rng.integers(1, 4000, 200), rng.integers(1, 4000, 200),
                                                           rng.integers(1, 300, 200))]
    for h, w, s in cases:
        try:
            exp = oracle.image_token_layout(h, w, 16, s, 3)
        except oracle.LayoutError:
            try:
                native.image_token_layout(h, w, 16, s, 3)
            except native.G4MError as e:
                assert e.status == 10
                continue
            raise AssertionError(f"layout {h}x{w}/{s} should fail")
        got = native.image_token_layout(h, w, 16, s, 3)
        assert got == [exp["target"]["height"], exp["target"]["width"], exp["patchGrid"]["height"],
                       exp["patchGrid"]["width"], exp["maxPatches"], exp["softTokens"]], (h, w, s)


def test_audio_token_count_matches_oracle(native, oracle):
    for n in list(range(0, 2000, 7)) + [80000, 160000, 479999, 480000, 480001, 10 ** 7]:
        assert native.audio_soft_token_count(n, 320, 160, 750) == oracle.audio_soft_token_count(n), n


def test_checksum_matches_oracle(native, oracle):
    rng = np.random.default_rng(1)
    for scale in (1e-3, 1.0, 50.0):
        v = (rng.standard_normal(5000) * scale).astype(np.float32)
        assert native.checksum_floats(v) == oracle.checksum_floats(v)


def test_public_api_layout_and_count(g4m):
    lay = g4m.computeGemma4ImageTokenLayout({"height": 1024, "width": 768, "patchSize": 16, "maxSoftTokens": 280,
                                             "poolingKernelSize": 3})
    assert lay["target"] == {"height": 912, "width": 672} and lay["softTokens"] == 266
    assert g4m.computeGemma4AudioSoftTokenCount({"samples": 80000, "frameLength": 320, "hopLength": 160,
                                                 "audioSeqLength": 750}) == 125


def test_embed_without_gpu_returns_error_object(g4m, monkeypatch):
    # The embed entry points never raise (src/vision/index.ts:131-147): with no
    # checkpoint configured they return ok=False and zeroed fields.
    monkeypatch.delenv("G4M_WEIGHTS", raising=False)
    g4m.configure(None)
    r = g4m.computeGemma4VisionImageEmbeddings({"blob": {"pixels": np.zeros((48, 48, 3), np.uint8), "width": 48,
                                                         "height": 48}, "maxSoftTokens": 1})
    assert r["ok"] is False and r["rows"] == 0 and r["checksum"] is None and "error" in r
    r = g4m.computeGemma4AudioEmbeddings({"samples": np.zeros(1600, np.float32)})
    assert r["ok"] is False and r["stages"]["frames"] == 0
    r = g4m.computeGemma4VisionImageEmbeddings({"blob": {"pixels": np.zeros((48, 48, 3), np.uint8)}, "layerCount": 17})
    assert r["ok"] is False and "layer count" in r["error"]


def test_preprocess_image_blob(g4m, oracle):
    px = (np.arange(96 * 96 * 4) % 251).astype(np.uint8).reshape(96, 96, 4)
    got = g4m.preprocessGemma4ImageBlob({"pixels": px, "width": 96, "height": 96}, {"maxSoftTokens": 4})
    exp = oracle.preprocess_image_pixels(px, max_soft_tokens=4)
    assert np.array_equal(got["pixelValues"].reshape(exp["pixelValues"].shape), exp["pixelValues"])
    assert np.array_equal(got["imagePositionIds"].reshape(-1, 2), exp["imagePositionIds"])
    assert got["numSoftTokens"] == 4 and got["patchPixels"] == 768


def test_synthetic_checkpoint_round_trip(syn, tmp_path):
    """Scalar activation scales stay 0-d (shape []) as scalarF32FromTensor
    requires (src/io/safetensors.ts:170-175)."""
    W = syn.vision_weights(0, layers=1)
    p = str(tmp_path / "v.safetensors")
    syn.write_safetensors(p, W)
    R = syn.read_safetensors(p)
    assert set(R) == set(W)
    for k, v in W.items():
        assert R[k].shape == v.shape and R[k].dtype == v.dtype and np.array_equal(R[k], v), k
    assert R["model.vision_tower.encoder.layers.0.self_attn.q_proj.linear.input_activation_scale"].shape == ()
