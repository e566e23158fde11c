"""Full-configuration parity against the oracle.

Vision: one 768 x 768 image (2304 patches, 256 tokens) through the patch
embedding, all 16 encoder layers, the 3 x 3 pooler and the embedder.
Audio: one 10 s clip (160000 samples, 999 frames, 250 encoder rows) through
the log-mel front end, the subsample convs, all 12 conformer layers, the
output projection and the embedder.  Weights are the seeded random-init
towers of the full depth.

Checks, per tower:
- every layer anchored (the reference's gpuAnchored probes,
  src/vision/probes.ts:1372-1497, src/audio/probes.ts:758): the device runs
  layer i on the oracle's input of layer i, and its output meets the
  north-star bound (row cosine >= 0.999, max-abs <= 1e-2 * RMS) against the
  oracle's output of layer i.  Beside it, both are measured against a float64
  evaluation of the same layer on the same input.
- end to end (propagated): the device output against the oracle.  The random
  -init towers amplify rounding-level differences layer over layer, so two
  correct f32-grade implementations with different summation orders drift
  apart; the gate is the north-star bound, or, where the oracle itself -- the
  reference's f32 arithmetic -- is farther than that bound from a float64
  evaluation of the same tower on the same input, the device must be no
  farther from float64 than twice the oracle is (max-abs and 1 - cosine).
"""
import numpy as np
import pytest

from conftest import assert_float64_envelope, assert_parity, report, row_metrics

pytestmark = pytest.mark.gpu


# --------------------------------------------------------------------- vision


@pytest.fixture(scope="module")
def vision_cfg1(native, syn, oracle, tmp_path_factory):
    """The 16-layer tower, the 768 x 768 image, and the oracle and float64
    chains over it (computed once for the module)."""
    import np_ref
    W = syn.vision_weights(0, layers=16)
    path = str(tmp_path_factory.mktemp("vision_cfg1") / "vision16.safetensors")
    syn.write_safetensors(path, W)
    pix = syn.image_pixels(0, 768, 768)
    pre = oracle.preprocess_image_pixels(pix)
    assert pre["numSoftTokens"] == 256
    patches, pos = oracle.valid_image_patch_input(pre)
    hs = [oracle.vision_patch_embeddings(W, patches, pos)]
    for i in range(16):
        hs.append(oracle.vision_layer(W, i, hs[-1], pos))
    emb = oracle.embedder(oracle.vision_pooler(hs[-1], pos, 256), W["model.embed_vision.embedding_projection.weight"])
    h64 = [np_ref.vision_patch_embeddings(W, patches, pos)]
    for i in range(16):
        h64.append(np_ref.vision_layer(W, i, h64[-1], pos))
    emb64 = np_ref.embedder(np_ref.pooler(h64[-1], 48, 48), W["model.embed_vision.embedding_projection.weight"])
    c = native.Context()
    c.load_weights(path)
    c.set_debug(True)
    yield dict(c=c, W=W, pix=pix, pos=pos, hs=hs, emb=emb, h64=h64, emb64=emb64)
    c.close()


def test_vision_cfg1_every_layer_anchored(vision_cfg1):
    """All 16 layers at 2304 patches, each fed the oracle's input of that
    layer, at the north-star bound; the device's float64 error per layer is
    printed beside the oracle's own."""
    import np_ref
    v = vision_cfg1
    worst = (1.0, 0.0)
    for i in range(16):
        got = v["c"].vision_layers(v["hs"][i], 1, 768, 768, i, 1)
        cos, ma = assert_parity(v["hs"][i + 1], got, what=f"vision layer {i} anchored (2304 patches)")
        ref64 = np_ref.vision_layer(v["W"], i, v["hs"][i], v["pos"])
        _, d64 = row_metrics(ref64, got)
        _, o64 = row_metrics(ref64, v["hs"][i + 1])
        report(f"vision layer {i}", cos=cos, maxabs=ma, dev_vs_f64=d64, oracle_vs_f64=o64)
        worst = (min(worst[0], cos), max(worst[1], ma))
    report("vision 16 anchored layers, worst", cos=worst[0], maxabs=worst[1])


def test_vision_cfg1_end_to_end(vision_cfg1):
    """Patch embedding, 16 propagated layers, pooler and embedder on the
    768 x 768 image, through the batch call."""
    v = vision_cfg1
    outs, rows = v["c"].vision_embed([v["pix"]], 280, 16)
    assert rows[0] == 256 and outs[0].shape == (256, 1536)
    h0 = v["c"].vision_debug_hidden(0, 2304)
    assert_parity(v["hs"][0], h0, cos_min=0.99999, maxabs=1e-4, what="patch embeddings")
    hl = v["c"].vision_debug_hidden(1, 2304)
    assert_float64_envelope(v["hs"][16], hl, v["h64"][16], "vision cfg1 hidden after 16 layers")
    assert_float64_envelope(v["emb"], outs[0], v["emb64"], "vision cfg1 embeddings")


# ---------------------------------------------------------------------- audio


@pytest.fixture(scope="module")
def audio_cfg2(native, syn, oracle, tmp_path_factory):
    import np_ref
    W = syn.audio_weights(0, layers=12)
    path = str(tmp_path_factory.mktemp("audio_cfg2") / "audio12.safetensors")
    syn.write_safetensors(path, W)
    x = syn.audio_samples(0, 160000)
    hid = []
    ref = oracle.audio_embed(W, x, layer_count=12, hidden_out=hid)
    assert ref["frames"] == 999 and ref["validSubsampleRows"] == 250
    h64 = [np.asarray(hid[0], np.float64)]
    for i in range(12):
        h64.append(np_ref.audio_layer(W, i, h64[-1]))
    proj = h64[-1] @ np.asarray(W["model.audio_tower.output_proj.weight"], np.float64).T + \
        np.asarray(W["model.audio_tower.output_proj.bias"], np.float64)
    emb64 = np_ref.embedder(proj, W["model.embed_audio.embedding_projection.weight"])
    c = native.Context()
    c.load_weights(path)
    yield dict(c=c, W=W, x=x, hid=hid, emb=ref["embeddings"], h64=h64, emb64=emb64)
    c.close()


def test_audio_cfg2_every_layer_anchored(audio_cfg2):
    """All 12 conformer layers on the 10 s clip's 250 rows, each fed the
    oracle's input of that layer: the north-star bound, or -- where the
    oracle's own packed-code sums (sum code*a - zp*sum a, which cancel) put it
    farther than the bound from float64 -- no farther from float64 than twice
    the oracle."""
    import np_ref
    a = audio_cfg2
    for i in range(12):
        got = a["c"].audio_layers(a["hid"][i], [250], i, 1)
        ref64 = np_ref.audio_layer(a["W"], i, a["hid"][i])
        assert_float64_envelope(a["hid"][i + 1], got, ref64, f"audio layer {i} anchored (250 rows)")


def test_audio_cfg2_end_to_end(audio_cfg2):
    """Log-mel, subsample, 12 propagated layers, output projection and
    embedder on the 10 s clip, through the batch call."""
    a = audio_cfg2
    a["c"].set_debug(True)
    try:
        outs, rows = a["c"].audio_embed([a["x"]], 16000, 12)
        assert rows[0] == 250
        enc_in = a["c"].audio_debug_hidden(250, which=0)
        enc_out = a["c"].audio_debug_hidden(250, which=1)
    finally:
        a["c"].set_debug(False)
    assert_parity(a["hid"][0], enc_in, cos_min=0.999999, maxabs=1e-4, what="audio encoder input (front end)")
    assert_float64_envelope(a["hid"][12], enc_out, a["h64"][12], "audio cfg2 encoder output after 12 layers")
    assert_float64_envelope(a["emb"], outs[0], a["emb64"], "audio cfg2 embeddings")
