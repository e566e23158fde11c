"""Device resize to the token layout's target size (the canvas drawImage step
of preprocessGemma4ImageSource, src/preprocess/image.ts:104-162) and the
any-size image entry point.  The browser's smoothing is unspecified, so the
resize is checked against its own numpy restatement and for the properties a
resampler must have (identity at the target size, constants preserved,
monotone ramps); the embeddings of resized images are checked against the
oracle fed with the same resized pixels."""
import numpy as np
import pytest

from conftest import assert_parity

pytestmark = pytest.mark.gpu


def _img(seed, h, w, c=3):
    return np.random.default_rng(seed).integers(0, 256, (h, w, c), dtype=np.uint8)


def test_resize_identity_constant_ramp(ctx):
    x = _img(0, 96, 144)
    y = ctx.resize_rgb(x, 96, 144)
    assert np.array_equal(y, (x.astype(np.float64) * (1 / 255)).astype(np.float32))
    c = np.full((700, 1000, 4), 77, np.uint8)
    assert np.all(ctx.resize_rgb(c, 336, 480) == np.float32(77 / 255))
    ramp = np.tile(np.arange(1000, dtype=np.float64)[None, :, None] * 255 / 999, (50, 1, 3)).round().astype(np.uint8)
    r = ctx.resize_rgb(ramp, 48, 336)
    assert np.all(np.diff(r[0, :, 0]) >= 0) and r[0, 0, 0] < 0.01 and r[0, -1, 0] > 0.99


@pytest.mark.parametrize("hw,thw", [((700, 1000), (336, 480)), ((240, 320), (672, 912)), ((1024, 768), (912, 672))])
def test_resize_matches_restatement(ctx, hw, thw):
    import np_ref
    x = _img(1, *hw)
    got = ctx.resize_rgb(x, *thw)
    ref = np_ref.resize_rgb(x, *thw)
    d = np.abs(got - ref) * 255
    # f32 (device) and float64 (restatement) sums round exact half steps apart:
    # integer pixels and rational weights make ties common; never more than one step
    assert d.max() <= 1.0 + 1e-3 and (d > 0.5).mean() < 1e-2


def test_images_of_any_size(vis_ctx, oracle, native):
    c, W = vis_ctx
    imgs = [_img(2, 700, 1000), _img(3, 96, 96), _img(4, 700, 1000)]
    outs, rows, status = c.vision_embed_images(imgs, 280, 1)
    assert list(status) == [0, 0, 0]
    for im, e, r in zip(imgs, outs, rows):
        th, tw, gh, gw, mp, st = native.image_token_layout(im.shape[0], im.shape[1], 16, 280, 3)
        assert r == st and e.shape == (st, 1536)
        pix = c.resize_rgb(im, th, tw)
        pre = oracle.preprocess_image_pixels(pix)
        patches, pos = oracle.valid_image_patch_input(pre)
        ref = oracle.vision_embed(W, patches, pos, pre["numSoftTokens"], layer_count=1)
        assert_parity(ref, e, what=f"resized {im.shape[:2]} -> {th}x{tw}")
    single, _, _ = c.vision_embed_images([imgs[2]], 280, 1)
    assert np.array_equal(single[0], outs[2])


def test_images_bad_layout_status(vis_ctx):
    """maxSoftTokens 0 rounds every layout to 0 x 0 (src/preprocess/image.ts:237)."""
    c, _ = vis_ctx
    outs, rows, status = c.vision_embed_images([_img(5, 100, 50), _img(6, 96, 96)], 0, 1)
    assert list(status) == [10, 10] and list(rows) == [0, 0]


@pytest.fixture(scope="module")
def vis_ctx(native, syn, tmp_path_factory):
    W = syn.vision_weights(0, layers=1)
    path = str(tmp_path_factory.mktemp("resize") / "v1.safetensors")
    syn.write_safetensors(path, W)
    c = native.Context()
    c.load_weights(path)
    yield c, W
    c.close()
