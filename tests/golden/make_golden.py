"""Writes tests/golden/oracle_small.npz: seeded small cases evaluated by the
oracle (the CPU restatement of the reference's CPU twins), used as committed
regression vectors for the oracle (tests/test_cpu_golden.py) and as device
parity targets that need no oracle run (tests/test_gpu_golden.py).

Cases (all weights from synthetic.py, seeds fixed):
  qat_i8      cfg0-shaped int8 QAT linear on 16 rows: x [16,768], W int8
              [768,768], scales, bias -> y [16,768]
  packed4     4-bit packed QAT linear [16,1024] -> [16,256]
  vision48    one 48 x 48 image, maxSoftTokens 1 (9 patches, 1 token, the
              reference probe case of src/vision/probes.ts:1378-1405), one
              encoder layer -> embedding [1,1536]
  audio_tone  0.08 s 440 + 660 Hz tone (src/audio/probes.ts:20-27), one
              conformer layer -> embeddings [2,1536]
  logmel      log-mel features of 1280 samples -> [7,128]

Run from the repository root:  python tests/golden/make_golden.py
"""
import importlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

syn = importlib.import_module("gemma-4-webgpu-kernels-multimodal_b200.synthetic")


def tone(seconds, f1=440.0, f2=660.0, a1=0.16, a2=0.05, rate=16000):
    t = np.arange(int(rate * seconds)) / rate
    return (a1 * np.sin(2 * np.pi * f1 * t) + a2 * np.sin(2 * np.pi * f2 * t)).astype(np.float32)


def qat_inputs():
    """cfg0-shaped int8 QAT linear, 16 rows (synthetic seed 0)."""
    return syn.qat_linear_case(0, rows=16)


def packed4_inputs():
    """4-bit packed QAT linear [16, 1024] -> [16, 256] (synthetic streams, seed 4)."""
    codes = syn.int_uniform(4, "golden.packed4.codes", 256 * 1024, 0, 15).reshape(256, 1024)
    wp = syn.pack_codes(codes, 4)
    xp = syn.normal(4, "golden.packed4.x", 16 * 1024).astype(np.float32).reshape(16, 1024)
    sp = (0.002 + 0.018 * syn.uniform(4, "golden.packed4.s", 256)).astype(np.float32)
    return xp, wp, sp


def input_checksum(*arrays):
    """FNV-1a over the raw bytes: detects drift of the seeded generators."""
    h = 0xCBF29CE484222325
    for a in arrays:
        for byte in np.ascontiguousarray(a).tobytes()[::97]:
            h = ((h ^ byte) * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return np.array(h, dtype=np.uint64)


def cases():
    out = {}
    x, w, s, b = qat_inputs()
    out["qat_i8/input_checksum"] = input_checksum(x, w, s, b)
    out["qat_i8/y"] = oracle.add_bias_rows(oracle.qat_i8_linear(x, w, s), b)
    xp, wp, sp = packed4_inputs()
    out["packed4/input_checksum"] = input_checksum(xp, wp, sp)
    out["packed4/y"] = oracle.packed_qat_linear(xp, wp, sp, 1024, 256, 4)
    Wv = syn.vision_weights(0, layers=1)
    pix = syn.image_pixels(0, 48, 48)
    pre = oracle.preprocess_image_pixels(pix, max_soft_tokens=1)
    patches, pos = oracle.valid_image_patch_input(pre)
    out["vision48/pixels"] = pix
    out["vision48/embedding"] = oracle.vision_embed(Wv, patches, pos, pre["numSoftTokens"], layer_count=1)
    Wa = syn.audio_weights(0, layers=1)
    xt = tone(0.08)
    out["audio_tone/samples"] = xt
    out["audio_tone/embeddings"] = oracle.audio_embed(Wa, xt, layer_count=1)["embeddings"]
    xs = syn.audio_samples(3, 1280)
    out["logmel/samples"] = xs
    out["logmel/features"] = oracle.preprocess_audio(xs, pad_to_multiple_of=None)["inputFeatures"]
    return out


if __name__ == "__main__":
    c = cases()
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle_small.npz")
    np.savez_compressed(path, **c)
    print(path, {k: v.shape for k, v in c.items()})
