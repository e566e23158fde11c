"""Batch calls on a context over two GPUs (one host thread per device,
contiguous image blocks, length-balanced clips): every item's embedding is
bitwise the one computed on a single device.  Skipped with fewer than two
GPUs."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_device_batches_match_one(native, syn, tmp_path):
    W = dict(syn.vision_weights(0, layers=2))
    W.update(syn.audio_weights(0, layers=2))
    path = str(tmp_path / "w.safetensors")
    syn.write_safetensors(path, W)
    one, two = native.Context([0]), native.Context([0, 1])
    try:
        one.load_weights(path)
        two.load_weights(path)
        pix = [syn.image_pixels(s, 96, 96) for s in range(5)]
        a, ra = one.vision_embed(pix, 4, 2)
        b, rb = two.vision_embed(pix, 4, 2)
        assert list(ra) == list(rb)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)
        clips = [syn.audio_samples(30 + i, n) for i, n in enumerate([16000, 48000, 3000, 32000, 8000])]
        a, ra = one.audio_embed(clips, 16000, 2)
        b, rb = two.audio_embed(clips, 16000, 2)
        assert list(ra) == list(rb)
        for x, y in zip(a, b):
            assert np.array_equal(x, y)
    finally:
        one.close()
        two.close()
