"""Static input-activation quantisation (input_activation_scale != 0,
srqScalar in src/kernels/qat.ts:489-492) inside both towers.

Every QAT linear's input scale is calibrated to absmax/127 of the input it
sees on an oracle pass over the test's own input (the calibrated mode), then
the scales of projections that share an input are spread apart (k, v, up)
so the per-projection code planes are exercised with distinct values.

Quantisation makes the random-init towers hypersensitive: a code that rounds
the other way moves one input by 1/127 of the calibration absmax, and the
oracle run on its own input perturbed by 1e-6 relative already leaves 30-60 %
of the rows of one vision layer outside the north-star bound.  Layer and
end-to-end checks therefore compare the device with the oracle's own
envelope under 1e-5 input perturbations (conftest.assert_within_envelope);
the quantised q | k | v projection, which no attention follows, is checked
against a float64 evaluation."""
import numpy as np
import pytest

from conftest import assert_within_envelope, perturbed, row_metrics_all

pytestmark = pytest.mark.gpu

EPS = 1e-5
SEEDS = (0, 1, 2)
VIS_SPREAD = {"self_attn.k_proj": 1.5, "self_attn.v_proj": 0.75, "mlp.up_proj": 1.25}
AUD_SPREAD = {"self_attn.k_proj": 1.5, "self_attn.v_proj": 0.75}


def _spread(W, prefix_fmt, layers, factors):
    """Multiply selected input scales by fixed factors (distinct per projection)."""
    W = dict(W)
    for i in range(layers):
        for name, f in factors.items():
            key = prefix_fmt.format(i=i, name=name) + ".input_activation_scale"
            W[key] = np.array(np.float32(float(W[key]) * f), np.float32).reshape(())
    return W


@pytest.fixture(scope="module")
def visq(native, syn, oracle, tmp_path_factory):
    """Two vision layers calibrated on one 768 x 768 image (2304 patches)."""
    layers = 2
    W = syn.vision_weights(3, layers=layers)
    pix = syn.image_pixels(5, 768, 768)
    pre = oracle.preprocess_image_pixels(pix)
    patches, pos = oracle.valid_image_patch_input(pre)
    with oracle.record_linear_inputs() as taps:
        oracle.vision_embed(W, patches, pos, pre["numSoftTokens"], layer_count=layers)
    Wq = _spread(oracle.calibrated_input_scales(W, taps), "model.vision_tower.encoder.layers.{i}.{name}.linear",
                 layers, VIS_SPREAD)
    path = str(tmp_path_factory.mktemp("visionq") / "visionq.safetensors")
    syn.write_safetensors(path, Wq)
    c = native.Context()
    c.load_weights(path)
    yield c, Wq, pix, pre, patches, pos
    c.close()


def test_vision_quantised_scales_are_distinct(visq):
    _, Wq, *_ = visq
    s = [float(Wq[f"model.vision_tower.encoder.layers.0.self_attn.{p}_proj.linear.input_activation_scale"])
         for p in "qkv"]
    g = [float(Wq[f"model.vision_tower.encoder.layers.0.mlp.{p}_proj.linear.input_activation_scale"])
         for p in ("gate", "up")]
    assert min(s) > 0 and len(set(s)) == 3 and min(g) > 0 and g[0] != g[1]


def test_vision_quantised_layers_anchored(visq, oracle):
    """Each layer fed the oracle's input for that layer (2304 rows)."""
    c, Wq, pix, pre, patches, pos = visq
    h = oracle.vision_patch_embeddings(Wq, patches, pos)
    for i in range(2):
        got = c.vision_layers(h, 1, 768, 768, i, 1)
        env = [oracle.vision_layer(Wq, i, perturbed(h, EPS, s), pos) for s in SEEDS]
        h = oracle.vision_layer(Wq, i, h, pos)
        assert_within_envelope(h, got, env, what=f"vision layer {i}, static input quantisation")


def test_vision_quantised_embeddings(visq, oracle):
    """Patch embed -> 2 quantised layers -> pooler -> embedder (256 tokens)."""
    c, Wq, pix, pre, patches, pos = visq
    ref = oracle.vision_embed(Wq, patches, pos, pre["numSoftTokens"], layer_count=2)
    outs, rows = c.vision_embed([pix], 280, 2)
    assert rows[0] == ref.shape[0] == 256
    env = [oracle.vision_embed(Wq, perturbed(patches, EPS, s), pos, pre["numSoftTokens"], layer_count=2)
           for s in SEEDS]
    assert_within_envelope(ref, outs[0], env, what="vision embeddings, static input quantisation, 2 layers")


def test_vision_mixed_group_rejected(native, syn, tmp_path):
    W = syn.vision_weights(0, layers=1)
    W["model.vision_tower.encoder.layers.0.self_attn.k_proj.linear.input_activation_scale"] = \
        np.array(0.05, np.float32).reshape(())
    path = str(tmp_path / "mixed.safetensors")
    syn.write_safetensors(path, W)
    c = native.Context()
    try:
        c.load_weights(path)
        with pytest.raises(native.G4MError) as e:
            c.vision_embed([syn.image_pixels(0, 96, 96)], 4, 1)
        assert e.value.status == 9 and "share one operand" in str(e.value)
    finally:
        c.close()


@pytest.fixture(scope="module")
def audq(native, syn, oracle, tmp_path_factory):
    """Two conformer layers calibrated on one 10 s clip (250 rows)."""
    layers = 2
    W = syn.audio_weights(3, layers=layers)
    x = syn.audio_samples(9, 160000)
    with oracle.record_linear_inputs() as taps:
        oracle.audio_embed(W, x, layer_count=layers)
    Wq = _spread(oracle.calibrated_input_scales(W, taps), "model.audio_tower.layers.{i}.{name}.linear", layers,
                 AUD_SPREAD)
    path = str(tmp_path_factory.mktemp("audioq") / "audioq.safetensors")
    syn.write_safetensors(path, Wq)
    c = native.Context()
    c.load_weights(path)
    pre = oracle.preprocess_audio(x, pad_to_multiple_of=None)
    h, _ = oracle.audio_subsample(Wq, pre["inputFeatures"], pre["inputFeaturesMask"])
    yield c, Wq, x, h
    c.close()


def test_audio_quantised_qkv_projection(audq, oracle, syn, native, tmp_path):
    """The per-projection code planes of the fused q | k | v GEMM (amode 1),
    with only q / k / v quantised: q, k and v of layer 0 against a float64
    evaluation of feed_forward1 -> norm_pre_attn -> srq -> projection.  The
    oracle follows the reference's packed formula (f32 sum(code * a) minus
    zero point * f32 sum(a)), whose cancellation on ffw_layer_2 flips a few
    q-input codes per row; the device must be at least as close to float64
    as the oracle is."""
    import np_ref
    _, Wq, x, h = audq
    W = syn.audio_weights(3, layers=1)
    for p in "qkv":
        key = f"model.audio_tower.layers.0.self_attn.{p}_proj.linear.input_activation_scale"
        W[key] = Wq[key]
    path = str(tmp_path / "qkvq.safetensors")
    syn.write_safetensors(path, W)
    c = native.Context()
    try:
        c.load_weights(path)
        rows = h.shape[0]
        c.audio_layers(h, [rows], 0, 1)
        got = c.audio_debug_hidden(rows, which=2)
    finally:
        c.close()
    pre = "model.audio_tower.layers.0"

    def lin64(name, xx, inp, out):
        w = W[f"{pre}.{name}.weight"]
        return np_ref.packed_qat(xx, w, W[f"{pre}.{name}.weight_scale"], inp, 8,
                                 float(W[f"{pre}.{name}.input_activation_scale"]),
                                 float(W[f"{pre}.{name}.output_activation_scale"]))

    f = np_ref.rmsnorm(h, W[f"{pre}.feed_forward1.pre_layer_norm.weight"])
    f = lin64("feed_forward1.ffw_layer_1.linear", f, 1024, 4096)
    f = lin64("feed_forward1.ffw_layer_2.linear", f / (1 + np.exp(-f)), 4096, 1024)
    h1 = np.asarray(h, np.float64) + 0.5 * np_ref.rmsnorm(f, W[f"{pre}.feed_forward1.post_layer_norm.weight"])
    a64 = np_ref.rmsnorm(h1, W[f"{pre}.norm_pre_attn.weight"])
    h1o = oracle.audio_ffn(W, 0, "feed_forward1", h)
    ao = oracle.rmsnorm(h1o, W[f"{pre}.norm_pre_attn.weight"], 1e-6)
    orc = oracle.audio_qkv(W, 0, ao)
    for j, p in enumerate("qkv"):
        ref64 = lin64(f"self_attn.{p}_proj.linear", a64, 1024, 1024)
        g = got[:, 1024 * j: 1024 * (j + 1)]
        _, ma_g = row_metrics_all(ref64, g)
        _, ma_o = row_metrics_all(ref64, orc[j])
        print(f"audio {p} from codes vs float64: device median {np.median(ma_g):.2e} max {ma_g.max():.2e}; "
              f"oracle median {np.median(ma_o):.2e} max {ma_o.max():.2e}")
        assert np.median(ma_g) <= 1.5 * np.median(ma_o) + 1e-5 and ma_g.max() <= 1.5 * ma_o.max() + 1e-4


def test_audio_quantised_layers_anchored(audq, oracle):
    """Each conformer layer fed the oracle's input for that layer, with
    calibrated and spread input scales on every QAT linear."""
    c, Wq, x, h = audq
    for i in range(2):
        got = c.audio_layers(h, [h.shape[0]], i, 1)
        env = [oracle.audio_layer(Wq, i, perturbed(h, EPS, s)) for s in SEEDS]
        h = oracle.audio_layer(Wq, i, h)
        assert_within_envelope(h, got, env, what=f"audio layer {i}, static input quantisation")


def test_audio_quantised_embeddings(audq, oracle):
    c, Wq, x, _ = audq
    ref = oracle.audio_embed(Wq, x, layer_count=1)
    outs, rows = c.audio_embed([x], 16000, 1)
    assert rows[0] == ref["validSubsampleRows"] == 250
    env = [oracle.audio_embed(Wq, perturbed(x, EPS, s), layer_count=1)["embeddings"] for s in SEEDS]
    assert_within_envelope(ref["embeddings"], outs[0], env, what="audio embeddings, static input quantisation")
