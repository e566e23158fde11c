"""Pipelined batch calls split a device's items into chunks (head, middle
and tail) whose copies overlap the compute.  Every row of the embeddings is
independent of the other items in its chunk, so a batch large enough to be
split must give bitwise the embeddings of one forward over all items
(the device-pointer entry points run a single forward)."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ctx2(native, syn, tmp_path_factory):
    W = dict(syn.vision_weights(1, layers=2))
    W.update(syn.audio_weights(1, layers=2))
    path = str(tmp_path_factory.mktemp("chunks") / "w.safetensors")
    syn.write_safetensors(path, W)
    c = native.Context([0])
    c.load_weights(path)
    yield c
    c.close()


def test_vision_batch_chunks_match_one_forward(ctx2, syn):
    """13 images: chunks of 4, 5 and 4 images."""
    n, h, w = 13, 96, 96
    pix = [syn.image_pixels(100 + i, h, w) for i in range(n)]
    got, rows = ctx2.vision_embed(pix, 4, 2)
    tokens = int(rows[0])
    dev = torch.from_numpy(np.stack(pix)).cuda()
    out = torch.empty((n, tokens, 1536), dtype=torch.float32, device="cuda")
    ctx2.vision_embed_device(dev.data_ptr(), n, h, w, out.data_ptr(), 4, 2)
    torch.cuda.synchronize()
    ref = out.cpu().numpy()
    for i in range(n):
        assert np.array_equal(got[i], ref[i]), f"image {i}"


def test_audio_batch_chunks_match_one_forward(ctx2, syn, native):
    """48 clips of 1..30 s (~18k encoder rows): a head and a tail chunk of at
    most 4736 rows around one middle chunk."""
    lens = [16000 * (1 + (7 * i) % 30) + 37 * i for i in range(48)]
    clips = [syn.audio_samples(200 + i, L) for i, L in enumerate(lens)]
    got, rows = ctx2.audio_embed(clips, 16000, 2)
    assert sum(int(r) for r in rows) > 3 * 4736
    flat = np.concatenate(clips).astype(np.float32)
    offs = np.cumsum([0] + lens[:-1]).astype(np.int64)
    dev = torch.from_numpy(flat).cuda()
    total = int(sum(int(r) for r in rows))
    out = torch.empty((total, 1536), dtype=torch.float32, device="cuda")
    drows = ctx2.audio_embed_device(dev.data_ptr(), offs, np.array(lens, np.int64), out.data_ptr(), 16000, 2)
    torch.cuda.synchronize()
    assert list(drows) == list(rows)
    ref = out.cpu().numpy()
    r0 = 0
    for i, r in enumerate(rows):
        assert np.array_equal(got[i][:r], ref[r0:r0 + r]), f"clip {i}"
        r0 += int(r)
