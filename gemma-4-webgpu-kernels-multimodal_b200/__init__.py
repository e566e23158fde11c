"""B200-native (sm_100a) Gemma 4 E2B vision and audio embedding towers.

Host-side mirror of the public API of ClinDesk-AI/gemma-4-webgpu-kernels-multimodal
(src/index.ts:1-42): same function names, argument meanings, result objects
and error behaviour, running on the CUDA library libg4m.so (C ABI in
include/g4m.h) instead of WebGPU.

Differences forced by the host language:
  * images are passed as decoded pixels ({"pixels", "width", "height"}) --
    the reference's README shape -- since there is no Blob / canvas here;
  * weights come from a local safetensors file (configure(weights_path=...))
    instead of HTTP Range requests to the Hugging Face hub;
  * batched variants (...Batch) take lists and shard them over the
    configured GPUs.
The embed calls never raise: failures return {"ok": False, "error": ...}
with zeroed fields (src/vision/index.ts:131-147, src/audio/index.ts:159-181);
the layout / count / preprocess functions raise, as the reference does.
"""
from __future__ import annotations

import math
import os
import time
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import _native
from ._native import G4MError

GEMMA4_MEDIA_MODEL_ID = "google/gemma-4-E2B-it-qat-mobile-transformers"
GEMMA4_MEDIA_MODEL_URL = "https://huggingface.co/google/gemma-4-E2B-it-qat-mobile-transformers"
UPSTREAM_WEBGPU_KERNEL_SPACE_URL = "https://huggingface.co/spaces/webml-community/gemma-4-webgpu-kernels"
GEMMA4_MEDIA_KERNEL_PENDING_MESSAGE = (
    "Image and audio support must be implemented against google/gemma-4-E2B-it-qat-mobile-transformers.")

VISION_ENCODER_LAYER_COUNT = 16
AUDIO_ENCODER_LAYER_COUNT = 12

_default = {"ctx": None, "weights": None, "devices": None}


def configure(weights_path: Optional[str] = None, devices: Optional[Sequence[int]] = None) -> None:
    """Select the checkpoint (local safetensors) and GPUs used by the API calls."""
    close()
    _default["weights"] = weights_path
    _default["devices"] = list(devices) if devices else None


def close() -> None:
    if _default["ctx"] is not None:
        _default["ctx"].close()
    _default["ctx"] = None


def context() -> _native.Context:
    if _default["ctx"] is None:
        path = _default["weights"] or os.environ.get("G4M_WEIGHTS")
        if not path:
            raise G4MError(8, "no checkpoint configured: call configure(weights_path=...) or set G4M_WEIGHTS")
        ctx = _native.Context(_default["devices"])
        ctx.load_weights(path)
        _default["ctx"] = ctx
    return _default["ctx"]


def build() -> str:
    """Compile libg4m.so in-tree (sm_100a)."""
    from ._build import build as _build
    return _build()


# ---------------------------------------------------------------------------
# Layout and counts (src/preprocess/image.ts:4-30, src/preprocess/audio.ts:4-20)
# ---------------------------------------------------------------------------

def computeGemma4ImageTokenLayout(input: Dict) -> Dict:
    th, tw, gh, gw, mp, st = _native.image_token_layout(input["height"], input["width"], input["patchSize"],
                                                        input["maxSoftTokens"], input["poolingKernelSize"])
    return {"input": {"height": input["height"], "width": input["width"]}, "target": {"height": th, "width": tw},
            "patchGrid": {"height": gh, "width": gw}, "maxPatches": mp, "softTokens": st}


def computeGemma4AudioSoftTokenCount(input: Dict) -> int:
    return _native.audio_soft_token_count(input["samples"], input["frameLength"], input["hopLength"],
                                          input["audioSeqLength"])


def checksumFloats(values) -> int:
    return _native.checksum_floats(values)


def _rounded_sample(v: np.ndarray) -> List[float]:
    out = []
    for x in np.asarray(v, dtype=np.float32).reshape(-1)[:8]:
        y = float(x) * 1_000_000
        f = math.floor(y)
        out.append((f + 1 if y - f >= 0.5 else f) / 1_000_000)
    return out


# ---------------------------------------------------------------------------
# Image preprocessing (src/preprocess/image.ts:32-162)
# ---------------------------------------------------------------------------

def preprocessGemma4ImageBlob(blob: Dict, options: Optional[Dict] = None) -> Dict:
    """blob = {"pixels": uint8 [h, w, 3|4] of any size, or float32 [h, w, 3]
    in [0, 1] already at the token layout's target size; "width", "height"}.
    uint8 images off the target size are resized on the GPU (g4m_resize_rgb:
    antialiased linear filter, 8-bit rounding, 1/255 rescale) in place of the
    reference's browser-canvas drawImage, whose smoothing is unspecified."""
    o = options or {}
    patch = o.get("patchSize", 16)
    max_soft = o.get("maxSoftTokens", 280)
    pool = o.get("poolingKernelSize", 3)
    rescale = o.get("rescaleFactor", 1 / 255)
    px = np.asarray(blob["pixels"])
    h, w = int(blob.get("height", px.shape[0])), int(blob.get("width", px.shape[1]))
    layout = computeGemma4ImageTokenLayout({"height": h, "width": w, "patchSize": patch, "maxSoftTokens": max_soft,
                                            "poolingKernelSize": pool})
    th, tw = layout["target"]["height"], layout["target"]["width"]
    if (th, tw) != (h, w):
        if px.dtype != np.uint8 or rescale != 1 / 255:
            raise ValueError(f"float pixels must already be at the token layout's target size {th} x {tw}")
        rgb = context().resize_rgb(px, th, tw)
    else:
        rgb = (px[..., :3].astype(np.float64) * rescale).astype(np.float32) if px.dtype == np.uint8 else \
            np.ascontiguousarray(px[..., :3], dtype=np.float32)
    gh, gw = layout["patchGrid"]["height"], layout["patchGrid"]["width"]
    pp = patch * patch * 3
    pv = np.zeros((layout["maxPatches"], pp), np.float32)
    ids = np.full((layout["maxPatches"] * 2,), -1, np.int32)
    pv[: gh * gw] = rgb.reshape(gh, patch, gw, patch, 3).transpose(0, 2, 1, 3, 4).reshape(gh * gw, pp)
    yy, xx = np.divmod(np.arange(gh * gw), gw)
    ids[0: 2 * gh * gw: 2] = xx
    ids[1: 2 * gh * gw: 2] = yy
    return {"layout": layout, "pixelValues": pv.reshape(-1), "imagePositionIds": ids,
            "numSoftTokens": layout["softTokens"], "maxPatches": layout["maxPatches"], "patchPixels": pp,
            "rgb": rgb}


# ---------------------------------------------------------------------------
# Embedding entry points
# ---------------------------------------------------------------------------

def _vision_failure(started, layer_count, err) -> Dict:
    return {"ok": False, "modelId": GEMMA4_MEDIA_MODEL_ID, "durationMs": round((time.perf_counter() - started) * 1000),
            "source": {"width": 0, "height": 0}, "layout": None, "layerCount": layer_count, "rows": 0, "dim": 0,
            "embeddings": np.zeros(0, np.float32), "finite": False, "checksum": None, "firstValues": [],
            "error": str(err)}


def computeGemma4VisionImageEmbeddingsBatch(inputs: List[Dict]) -> List[Dict]:
    """Batched computeGemma4VisionImageEmbeddings, sharded across the
    configured GPUs.  uint8 images may have any sizes (resized on the GPU,
    grouped by token layout); float32 pixels must share one target size."""
    started = time.perf_counter()
    if not inputs:
        return []
    layer_count = inputs[0].get("layerCount", VISION_ENCODER_LAYER_COUNT)
    max_soft = inputs[0].get("maxSoftTokens", 280)
    if all(np.asarray(i["blob"]["pixels"]).dtype == np.uint8 for i in inputs):
        return _vision_images(inputs, layer_count, max_soft, started)
    try:
        if not isinstance(layer_count, int) or layer_count < 1 or layer_count > VISION_ENCODER_LAYER_COUNT:
            raise ValueError(f"Vision encoder layer count must be 1-{VISION_ENCODER_LAYER_COUNT}, got {layer_count}.")
        pre = [preprocessGemma4ImageBlob(i["blob"], {"maxSoftTokens": max_soft, "poolingKernelSize": 3}) for i in inputs]
        if len({(p["layout"]["target"]["height"], p["layout"]["target"]["width"]) for p in pre}) != 1:
            raise ValueError("images of one batch must share a token layout")
        outs, rows = context().vision_embed([p["rgb"] for p in pre], max_soft, layer_count)
    except Exception as e:  # never raise, as the reference
        return [_vision_failure(started, layer_count, e) for _ in inputs]
    ms = round((time.perf_counter() - started) * 1000)
    res = []
    for p, e, r in zip(pre, outs, rows):
        finite = bool(np.isfinite(e).all())
        res.append({"ok": finite, "modelId": GEMMA4_MEDIA_MODEL_ID, "durationMs": ms,
                    "source": {"width": p["layout"]["input"]["width"], "height": p["layout"]["input"]["height"]},
                    "layout": p["layout"], "layerCount": layer_count, "rows": int(r), "dim": 1536,
                    "embeddings": e.reshape(-1), "finite": finite, "checksum": checksumFloats(e),
                    "firstValues": _rounded_sample(e)})
    return res


def _vision_images(inputs, layer_count, max_soft, started) -> List[Dict]:
    """Decoded 8-bit images of any sizes through g4m_vision_embed_images."""
    try:
        if not isinstance(layer_count, int) or layer_count < 1 or layer_count > VISION_ENCODER_LAYER_COUNT:
            raise ValueError(f"Vision encoder layer count must be 1-{VISION_ENCODER_LAYER_COUNT}, got {layer_count}.")
        imgs = [np.asarray(i["blob"]["pixels"]) for i in inputs]
        outs, rows, status = context().vision_embed_images(imgs, max_soft, layer_count)
    except Exception as e:  # never raise, as the reference
        return [_vision_failure(started, layer_count, e) for _ in inputs]
    ms = round((time.perf_counter() - started) * 1000)
    res = []
    for im, e, r, st in zip(imgs, outs, rows, status):
        if st != 0:
            res.append(_vision_failure(started, layer_count, f"{_native.STATUS_NAMES.get(int(st), st)}"))
            continue
        lay = computeGemma4ImageTokenLayout({"height": im.shape[0], "width": im.shape[1], "patchSize": 16,
                                             "maxSoftTokens": max_soft, "poolingKernelSize": 3})
        finite = bool(np.isfinite(e).all())
        res.append({"ok": finite, "modelId": GEMMA4_MEDIA_MODEL_ID, "durationMs": ms,
                    "source": {"width": int(im.shape[1]), "height": int(im.shape[0])}, "layout": lay,
                    "layerCount": layer_count, "rows": int(r), "dim": 1536, "embeddings": e.reshape(-1),
                    "finite": finite, "checksum": checksumFloats(e), "firstValues": _rounded_sample(e)})
    return res


def computeGemma4VisionImageEmbeddings(input: Dict) -> Dict:
    """computeGemma4VisionImageEmbeddings (src/vision/index.ts:12-148).
    input = {"blob": {"pixels", "width", "height"}, "maxSoftTokens"?, "layerCount"?}."""
    return computeGemma4VisionImageEmbeddingsBatch([input])[0]


def computeGemma4AudioEmbeddingsBatch(inputs: List[Dict]) -> List[Dict]:
    started = time.perf_counter()
    if not inputs:
        return []
    layer_count = inputs[0].get("layerCount", AUDIO_ENCODER_LAYER_COUNT)
    rate = inputs[0].get("samplingRate", 16000)
    max_samples = inputs[0].get("maxSamples", 0) or 0
    try:
        if not isinstance(layer_count, int) or layer_count < 1 or layer_count > AUDIO_ENCODER_LAYER_COUNT:
            raise ValueError(f"Audio encoder layer count must be 1-{AUDIO_ENCODER_LAYER_COUNT}, got {layer_count}.")
        clips = [np.asarray(i["samples"], dtype=np.float32) for i in inputs]
        outs, rows = context().audio_embed(clips, rate, layer_count, max_samples)
    except Exception as e:
        ms = round((time.perf_counter() - started) * 1000)
        return [{"ok": False, "modelId": GEMMA4_MEDIA_MODEL_ID, "durationMs": ms, "source": {"samples": 0, "samplingRate": rate},
                 "layerCount": layer_count, "rows": 0, "dim": 0, "embeddings": np.zeros(0, np.float32), "finite": False,
                 "checksum": None, "firstValues": [], "stages": {"frames": 0, "validFrames": 0, "subsampleRows": 0,
                 "validSubsampleRows": 0, "stackFinite": False, "outputProjectionFinite": False}, "error": str(e)}
                for _ in inputs]
    ms = round((time.perf_counter() - started) * 1000)
    res = []
    cap = max_samples if max_samples else 480000
    for c, e, r in zip(inputs, outs, rows):
        n = min(len(c["samples"]), cap)
        finite = bool(np.isfinite(e).all())
        frames = (160 + n - 321) // 160 + 1 if 160 + n >= 321 else 0
        res.append({"ok": finite, "modelId": GEMMA4_MEDIA_MODEL_ID, "durationMs": ms,
                    "source": {"samples": n, "samplingRate": rate}, "layerCount": layer_count, "rows": int(r),
                    "dim": 1536, "embeddings": e.reshape(-1), "finite": finite, "checksum": checksumFloats(e),
                    "firstValues": _rounded_sample(e),
                    "stages": {"frames": int(frames), "validFrames": int(frames), "subsampleRows": int(r),
                               "validSubsampleRows": int(r), "stackFinite": finite, "outputProjectionFinite": finite}})
    return res


def computeGemma4AudioEmbeddings(input: Dict) -> Dict:
    """computeGemma4AudioEmbeddings (src/audio/index.ts:12-183).
    input = {"samples", "samplingRate"?, "layerCount"?, "maxSamples"?}."""
    return computeGemma4AudioEmbeddingsBatch([input])[0]


__all__ = [
    "GEMMA4_MEDIA_MODEL_ID", "GEMMA4_MEDIA_MODEL_URL", "UPSTREAM_WEBGPU_KERNEL_SPACE_URL",
    "GEMMA4_MEDIA_KERNEL_PENDING_MESSAGE", "configure", "close", "context", "build",
    "computeGemma4ImageTokenLayout", "computeGemma4AudioSoftTokenCount", "preprocessGemma4ImageBlob",
    "computeGemma4VisionImageEmbeddings", "computeGemma4VisionImageEmbeddingsBatch",
    "computeGemma4AudioEmbeddings", "computeGemma4AudioEmbeddingsBatch", "checksumFloats", "G4MError",
]
