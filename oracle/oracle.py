"""CPU oracle for the Gemma 4 E2B media towers -- TEST INFRASTRUCTURE ONLY.

Python side of the oracle: ctypes bindings to liboracle_g4m.so (the C
restatement of the reference's CPU twins, g4m_oracle.c) and the tower
dataflow composed in the reference's order.  Only tests/, the smoke check
and bench.py's CPU-baseline leg import this module, and only as the checker
or the timed CPU baseline; the product library never does.

Dataflow sources (ClinDesk-AI/gemma-4-webgpu-kernels-multimodal):
  vision entry      src/vision/index.ts:12-148
  vision layer      src/vision/encoder.ts:189-298 (+ attention 681-765, MLP 1040-1092)
  pooler, embedder  src/vision/kernels.ts:815-833, src/embedder/index.ts:111-145
  audio entry       src/audio/index.ts:12-183
  audio layer       src/audio/encoder.ts:761-839 (+ FFN 841-921, light conv 923-1009,
                    attention 1011-1071, strip 1097-1110)
  preprocessing     src/preprocess/image.ts:4-30,104-162,181-197,217-252;
                    src/preprocess/audio.ts:4-226

Parity status: integer paths are pinned to the reference's literal probe
examples; the floating-point paths are "parity unpinned" (the reference ships
no golden vectors and its TypeScript cannot run here) beyond an independent
numpy restatement used as a cross-check in tests/.
"""
from __future__ import annotations

import ctypes
import math
import os
import subprocess
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_g4m.so")
_lib = None

F32P = ctypes.POINTER(ctypes.c_float)


def build() -> str:
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.g4mo_checksum_floats.restype = ctypes.c_double
        L.g4mo_audio_soft_token_count.restype = ctypes.c_long
        L.g4mo_audio_frame_count.restype = ctypes.c_long
        L.g4mo_preprocess_audio.restype = ctypes.c_long
        _lib = L
    return _lib


def set_threads(n: int) -> None:
    lib().g4mo_set_threads(int(n))


def max_threads() -> int:
    return int(lib().g4mo_max_threads())


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _d(x: float):
    return ctypes.c_double(float(x))


def _f(x: float):
    return ctypes.c_float(float(x))


def _chk(rc: int, what: str) -> None:
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its input (rc={rc})")


def f32_from_bf16(bits: np.ndarray) -> np.ndarray:
    """float32FromBf16Bytes, src/io/safetensors.ts:151-164."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


# ---------------------------------------------------------------------------
# Kernel twins
# ---------------------------------------------------------------------------

def qat_i8_linear(x, w, s_w, s_in=0.0, s_out=0.0) -> np.ndarray:
    x = _f32(x)
    w = np.ascontiguousarray(w, dtype=np.int8)
    rows, inp = x.shape
    out = w.shape[0]
    y = np.empty((rows, out), np.float32)
    _chk(lib().g4mo_qat_i8_linear(_p(x), _p(w), _p(_f32(s_w).reshape(-1)), rows, inp, out, _f(s_in), _f(s_out), _p(y)), "qat_i8_linear")
    return y


def packed_qat_linear(x, w_u8, s_w, inp: int, out: int, bits: int, s_in=0.0, s_out=0.0) -> np.ndarray:
    x = _f32(x)
    w = np.ascontiguousarray(w_u8, dtype=np.uint8)
    rows = x.shape[0]
    if w.nbytes != out * inp * bits // 8:
        raise ValueError("packed QAT weight length does not match dimensions")
    y = np.empty((rows, out), np.float32)
    _chk(lib().g4mo_packed_qat_linear(_p(x), _p(w), _p(_f32(s_w).reshape(-1)), rows, inp, out, bits, _f(s_in), _f(s_out), _p(y)), "packed_qat_linear")
    return y


def derive_packed_bits(nbytes: int, inp: int, out: int) -> int:
    """derivePackedQatBits, src/kernels/qat.ts:199-213."""
    bits = nbytes * 8 / (inp * out)
    if bits not in (2, 4, 8):
        raise ValueError(f"derived unsupported {bits}-bit QAT weights from {nbytes} bytes")
    bits = int(bits)
    if (inp * bits) % 8 != 0 or (inp * bits) % 32 != 0:
        raise ValueError("packed QAT row is not byte and u32 aligned")
    return bits


def f32_linear_rows(x, w) -> np.ndarray:
    x = _f32(x)
    w = _f32(w)
    rows, inp = x.shape
    out = w.shape[0]
    y = np.empty((rows, out), np.float32)
    lib().g4mo_f32_linear_rows(_p(x), _p(w), rows, inp, out, _p(y))
    return y


def embedder(h, w, eps=1e-6) -> np.ndarray:
    h = _f32(h)
    w = _f32(w)
    rows, inp = h.shape
    out = w.shape[0]
    y = np.empty((rows, out), np.float32)
    lib().g4mo_embedder(_p(h), _p(w), rows, inp, out, _d(eps), _p(y))
    return y


def rmsnorm(x, w, eps=1e-6) -> np.ndarray:
    x = _f32(x)
    w = _f32(w).reshape(-1)
    d = x.shape[-1]
    if w.size != d:
        raise ValueError("Vision RMSNorm weight length does not match hidden size.")
    rows = x.size // d
    y = np.empty_like(x)
    lib().g4mo_rmsnorm(_p(x), _p(w), rows, d, _d(eps), _p(y))
    return y


def vision_rope(v, pos, heads, hd, theta=100.0) -> np.ndarray:
    v = _f32(v)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    rows = v.size // (heads * hd)
    y = np.empty_like(v)
    _chk(lib().g4mo_vision_rope(_p(v), _p(pos), rows, heads, hd, _d(theta), _p(y)), "vision_rope")
    return y


def vision_attention(q, k, v, heads, hd, scaling=1.0) -> np.ndarray:
    q, k, v = _f32(q), _f32(k), _f32(v)
    rows = q.size // (heads * hd)
    o = np.empty_like(q)
    lib().g4mo_vision_attention(_p(q), _p(k), _p(v), rows, heads, hd, _d(scaling), _p(o))
    return o


def residual_add(r, v) -> np.ndarray:
    r, v = _f32(r), _f32(v)
    y = np.empty_like(r)
    lib().g4mo_residual_add(_p(r), _p(v), ctypes.c_long(r.size), _p(y))
    return y


def gelu_gate(g, u) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    y = np.empty_like(g)
    lib().g4mo_gelu_gate(_p(g), _p(u), ctypes.c_long(g.size), _p(y))
    return y


def vision_pool_indices(pos, out_len, k=3) -> np.ndarray:
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    idx = np.empty(out_len * k * k, np.int32)
    _chk(lib().g4mo_vision_pool_indices(_p(pos), pos.shape[0], out_len, k, _p(idx)), "vision_pool_indices")
    return idx


def vision_pooler(h, pos, out_len, k=3) -> np.ndarray:
    h = _f32(h)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    d = h.shape[-1]
    y = np.empty((out_len, d), np.float32)
    _chk(lib().g4mo_vision_pooler(_p(h), _p(pos), pos.shape[0], out_len, d, k, _p(y)), "vision_pooler")
    return y


def vision_patch_embed(patches, w, pos, posx_rows, posy_rows) -> np.ndarray:
    patches = _f32(patches)
    w = _f32(w)
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    npatch, pp = patches.shape
    out_rows = w.shape[0]
    d = posx_rows.shape[-1]
    posx, posy = _f32(posx_rows), _f32(posy_rows)
    y = np.empty((npatch, out_rows), np.float32)
    _chk(lib().g4mo_vision_patch_embed(_p(patches), _p(w), _p(pos), npatch, pp, d, out_rows, _p(posx), posx.shape[0],
                                       _p(posy), posy.shape[0], _p(y)), "vision_patch_embed")
    return y


def audio_subsample_conv_layer(x, mask, in_t, in_f, in_c, w, nw, out_c, eps=1e-6):
    x = _f32(x)
    mask = np.ascontiguousarray(mask, dtype=np.uint8)
    L = lib()
    ot = L.g4mo_audio_subsample_output_length(in_t)
    of = L.g4mo_audio_subsample_output_length(in_f)
    y = np.empty(ot * of * out_c, np.float32)
    om = np.empty(max(ot, 0), np.uint8)
    L.g4mo_audio_subsample_conv_layer(_p(x), _p(mask), in_t, in_f, in_c, _p(_f32(w)), _p(_f32(nw)), out_c, _d(eps), _p(y), _p(om))
    return y, om, ot, of


def audio_relpos(plen, d) -> np.ndarray:
    y = np.empty((plen, d), np.float32)
    _chk(lib().g4mo_audio_relpos(plen, d, _p(y)), "audio_relpos")
    return y


def audio_attention(q, k, v, relk, pds, heads, hd, chunk=12, ctx=24, plen=13, softcap=50.0) -> np.ndarray:
    q, k, v, relk, pds = _f32(q), _f32(k), _f32(v), _f32(relk), _f32(pds)
    rows = q.size // (heads * hd)
    o = np.empty_like(q)
    lib().g4mo_audio_attention(_p(q), _p(k), _p(v), _p(relk), _p(pds), rows, heads, hd, chunk, ctx, plen, _d(softcap), _p(o))
    return o


def glu(x, hs) -> np.ndarray:
    x = _f32(x)
    rows = x.size // (2 * hs)
    y = np.empty((rows, hs), np.float32)
    lib().g4mo_glu(_p(x), rows, hs, _p(y))
    return y


def depthwise_causal(x, w, ks=5) -> np.ndarray:
    x = _f32(x)
    rows, hs = x.shape
    y = np.empty_like(x)
    lib().g4mo_depthwise_causal(_p(x), _p(_f32(w).reshape(hs, ks)), rows, hs, ks, _p(y))
    return y


def silu(x) -> np.ndarray:
    x = _f32(x)
    y = np.empty_like(x)
    lib().g4mo_silu(_p(x), ctypes.c_long(x.size), _p(y))
    return y


def scaled_residual_add(r, v, scale) -> np.ndarray:
    r, v = _f32(r), _f32(v)
    y = np.empty_like(r)
    lib().g4mo_scaled_residual_add(_p(r), _p(v), ctypes.c_long(r.size), _d(scale), _p(y))
    return y


def add_bias_rows(y, b) -> np.ndarray:
    y = _f32(y).copy()
    lib().g4mo_add_bias_rows(_p(y), _p(_f32(b)), y.shape[0], y.shape[1])
    return y


def strip_rows_by_mask(values, mask) -> np.ndarray:
    """stripRowsByMask, src/audio/encoder.ts:1097-1110."""
    return np.ascontiguousarray(values[np.asarray(mask) != 0])


def checksum_floats(v) -> int:
    v = _f32(v).reshape(-1)
    return int(lib().g4mo_checksum_floats(_p(v), ctypes.c_long(v.size)))


def rounded_sample(v) -> List[float]:
    v = _f32(v).reshape(-1)
    out = np.zeros(8, np.float64)
    lib().g4mo_rounded_sample(_p(v), ctypes.c_long(v.size), _p(out))
    return [float(x) for x in out[: min(8, v.size)]]


# ---------------------------------------------------------------------------
# Preprocessing
# ---------------------------------------------------------------------------

class LayoutError(ValueError):
    pass


def image_token_layout(height, width, patch_size=16, max_soft_tokens=280, pooling_kernel_size=3) -> Dict:
    """computeGemma4ImageTokenLayout, src/preprocess/image.ts:4-30."""
    out = (ctypes.c_long * 6)()
    rc = lib().g4mo_image_token_layout(_d(height), _d(width), _d(patch_size), _d(max_soft_tokens), _d(pooling_kernel_size), out)
    if rc == -1:
        raise LayoutError("Image height and width must be positive.")
    if rc == -2:
        raise LayoutError(f"Image resize rounded to 0 x 0 for side multiple {pooling_kernel_size * patch_size}.")
    if rc == -3:
        raise LayoutError(f"Image resize exceeds {max_soft_tokens * pooling_kernel_size ** 2} patches.")
    return {
        "input": {"height": height, "width": width},
        "target": {"height": out[0], "width": out[1]},
        "patchGrid": {"height": out[2], "width": out[3]},
        "maxPatches": out[4],
        "softTokens": out[5],
    }


def audio_soft_token_count(samples, frame_length=320, hop_length=160, audio_seq_length=750) -> int:
    """computeGemma4AudioSoftTokenCount, src/preprocess/audio.ts:4-20."""
    return int(lib().g4mo_audio_soft_token_count(_d(samples), _d(frame_length), _d(hop_length), _d(audio_seq_length)))


def audio_soft_tokens_from_mask(mask, seq_len=750) -> int:
    mask = np.ascontiguousarray(mask, dtype=np.uint8)
    return int(lib().g4mo_audio_soft_tokens_from_mask(_p(mask), mask.size, seq_len))


def preprocess_image_pixels(pixels, patch_size=16, max_soft_tokens=280, pooling_kernel_size=3, rescale=1.0 / 255.0) -> Dict:
    """Patchify of preprocessGemma4ImageSource, src/preprocess/image.ts:104-162,
    for pixels already at the layout's target size.  `pixels` is [h, w, 3|4]
    uint8 (rescaled by 1/255 as the reference does) or float32 already in
    [0, 1]."""
    h, w = pixels.shape[0], pixels.shape[1]
    layout = image_token_layout(h, w, patch_size, max_soft_tokens, pooling_kernel_size)
    if layout["target"]["height"] != h or layout["target"]["width"] != w:
        raise LayoutError("pixels must already be at the layout's target size")
    if pixels.dtype == np.uint8:
        rgb = (pixels[..., :3].astype(np.float64) * rescale).astype(np.float32)
    else:
        rgb = np.ascontiguousarray(pixels[..., :3], dtype=np.float32)
    gh, gw = layout["patchGrid"]["height"], layout["patchGrid"]["width"]
    pp = patch_size * patch_size * 3
    pv = np.zeros((layout["maxPatches"], pp), np.float32)
    ids = np.full((layout["maxPatches"], 2), -1, np.int32)
    patches = rgb.reshape(gh, patch_size, gw, patch_size, 3).transpose(0, 2, 1, 3, 4).reshape(gh * gw, pp)
    pv[: gh * gw] = patches
    yy, xx = np.divmod(np.arange(gh * gw), gw)
    ids[: gh * gw, 0] = xx
    ids[: gh * gw, 1] = yy
    return {"layout": layout, "pixelValues": pv, "imagePositionIds": ids, "numSoftTokens": layout["softTokens"],
            "maxPatches": layout["maxPatches"], "patchPixels": pp}


def valid_image_patch_input(pre: Dict) -> Tuple[np.ndarray, np.ndarray]:
    """validImagePatchInput, src/preprocess/image.ts:181-197."""
    ids = pre["imagePositionIds"]
    n = 0
    while n < ids.shape[0] and ids[n, 0] >= 0 and ids[n, 1] >= 0:
        n += 1
    if n == 0:
        raise LayoutError("Image preprocessing produced zero valid patches.")
    return np.ascontiguousarray(pre["pixelValues"][:n]), np.ascontiguousarray(ids[:n])


def preprocess_audio(samples, sampling_rate=16000, feature_size=128, frame_length=320, hop_length=160, fft_length=512,
                     min_frequency=0.0, max_frequency=8000.0, mel_floor=0.001, input_scale_factor=1.0,
                     pad_to_multiple_of: Optional[int] = 128, max_samples=480000, audio_seq_length=750) -> Dict:
    """preprocessGemma4AudioSamples, src/preprocess/audio.ts:22-118."""
    x = _f32(samples).reshape(-1)
    L = lib()
    pad = int(pad_to_multiple_of) if pad_to_multiple_of else 0
    frames = int(L.g4mo_audio_frame_count(ctypes.c_long(x.size), ctypes.c_long(max_samples), ctypes.c_long(pad), frame_length, hop_length))
    feats = np.zeros((max(frames, 0), feature_size), np.float32)
    mask = np.zeros(max(frames, 0), np.uint8)
    vf = ctypes.c_long(0)
    if frames > 0:
        got = L.g4mo_preprocess_audio(_p(x), ctypes.c_long(x.size), _d(input_scale_factor), ctypes.c_long(max_samples), ctypes.c_long(pad),
                                      sampling_rate, feature_size, frame_length, hop_length, fft_length, _d(min_frequency),
                                      _d(max_frequency), _d(mel_floor), _p(feats), _p(mask), ctypes.byref(vf))
        if got < 0:
            raise ValueError("Gemma 4 audio FFT length must be a power of two covering the frame length.")
    return {"inputFeatures": feats, "inputFeaturesMask": mask, "frames": frames, "validFrames": int(vf.value),
            "featureSize": feature_size, "samplingRate": sampling_rate, "fftLength": fft_length,
            "softTokens": audio_soft_tokens_from_mask(mask, audio_seq_length) if frames > 0 else 0}


# ---------------------------------------------------------------------------
# Towers
# ---------------------------------------------------------------------------

VISION = dict(hidden=768, ff=3072, heads=12, head_dim=64, text=1536, pool=3, eps=1e-6, theta=100.0)
AUDIO = dict(hidden=1024, ff=4096, expanded=2048, out=1536, text=1536, heads=8, head_dim=128, chunk=12,
             ctx=24, plen=13, kernel=5, softcap=50.0, residual=0.5, eps=1e-6)


def _vis(W, i, name):
    return f"model.vision_tower.encoder.layers.{i}.{name}"


# Optional recorder of each QAT linear's input absmax (record_linear_inputs),
# for calibrating static input-activation scales on a real pass.
_TAPS: Optional[Dict[str, float]] = None


class record_linear_inputs:
    """Context manager: while active, every QAT linear run by the layer
    compositions below records max |x| of its input under its tensor prefix."""

    def __enter__(self):
        global _TAPS
        _TAPS = {}
        return _TAPS

    def __exit__(self, *exc):
        global _TAPS
        _TAPS = None
        return False


def _tap(prefix, x):
    if _TAPS is not None:
        _TAPS[prefix] = max(_TAPS.get(prefix, 0.0), float(np.abs(np.asarray(x, np.float64)).max()))


def calibrated_input_scales(W: Dict[str, np.ndarray], absmax: Dict[str, float]) -> Dict[str, np.ndarray]:
    """Copy of W whose input_activation_scale is absmax/127 (fround) for every
    recorded linear: the calibrated static-quantisation mode."""
    out = dict(W)
    for prefix, m in absmax.items():
        out[f"{prefix}.input_activation_scale"] = np.array(np.float32(m / 127.0) if m > 0 else 1.0, np.float32).reshape(())
    return out


def _qat_vision(W, prefix, x):
    _tap(prefix, x)
    return qat_i8_linear(x, W[f"{prefix}.weight"], W[f"{prefix}.weight_scale"], float(W[f"{prefix}.input_activation_scale"]),
                         float(W[f"{prefix}.output_activation_scale"]))


def vision_layer(W: Dict[str, np.ndarray], i: int, h: np.ndarray, pos: np.ndarray) -> np.ndarray:
    """computeVisionEncoderLayerWebGpuOnly dataflow, src/vision/encoder.ts:189-298,
    with the attention of 681-765 and the MLP of 1040-1092, on CPU twins."""
    c = VISION
    rows, d = h.shape
    heads, hd, eps = c["heads"], c["head_dim"], c["eps"]
    nw = lambda n: f32_from_bf16(W[_vis(W, i, n)])
    a = rmsnorm(h, nw("input_layernorm.weight"), eps)
    # head norms run over rows*heads rows of head_dim (src/vision/encoder.ts:403-410, 503)
    q = rmsnorm(_qat_vision(W, _vis(W, i, "self_attn.q_proj.linear"), a).reshape(-1, hd), nw("self_attn.q_norm.weight"), eps)
    k = rmsnorm(_qat_vision(W, _vis(W, i, "self_attn.k_proj.linear"), a).reshape(-1, hd), nw("self_attn.k_norm.weight"), eps)
    v = rmsnorm(_qat_vision(W, _vis(W, i, "self_attn.v_proj.linear"), a).reshape(-1, hd), np.ones(hd, np.float32), eps)
    q = vision_rope(q, pos, heads, hd, c["theta"])
    k = vision_rope(k, pos, heads, hd, c["theta"])
    o = vision_attention(q, k, v, heads, hd, 1.0).reshape(rows, d)
    o = _qat_vision(W, _vis(W, i, "self_attn.o_proj.linear"), o)
    h1 = residual_add(h, rmsnorm(o, nw("post_attention_layernorm.weight"), eps))
    f = rmsnorm(h1, nw("pre_feedforward_layernorm.weight"), eps)
    m = gelu_gate(_qat_vision(W, _vis(W, i, "mlp.gate_proj.linear"), f), _qat_vision(W, _vis(W, i, "mlp.up_proj.linear"), f))
    dn = _qat_vision(W, _vis(W, i, "mlp.down_proj.linear"), m)
    return residual_add(h1, rmsnorm(dn, nw("post_feedforward_layernorm.weight"), eps))


def vision_patch_embeddings(W, patches, pos) -> np.ndarray:
    """src/vision/index.ts:46-78 and loadVisionPatchPositionRows,
    src/vision/encoder.ts:8-85."""
    proj = f32_from_bf16(W["model.vision_tower.patch_embedder.input_proj.weight"])
    table = W["model.vision_tower.patch_embedder.position_embedding_table"]
    maxx, maxy = int(pos[:, 0].max()), int(pos[:, 1].max())
    if maxx >= table.shape[1] or maxy >= table.shape[1]:
        raise ValueError(f"Vision patch positions exceed position table length {table.shape[1]}: x={maxx}, y={maxy}.")
    xr = f32_from_bf16(table[0, : maxx + 1])
    yr = f32_from_bf16(table[1, : maxy + 1])
    return vision_patch_embed(patches, proj, pos, xr, yr)


def vision_embed(W: Dict[str, np.ndarray], patches: np.ndarray, pos: np.ndarray, num_soft_tokens: int,
                 layer_count: int = 16, hidden_out: Optional[list] = None) -> np.ndarray:
    """computeGemma4VisionImageEmbeddings compute path, src/vision/index.ts:69-112."""
    c = VISION
    h = vision_patch_embeddings(W, patches, pos)
    for i in range(layer_count):
        h = vision_layer(W, i, h, pos)
        if hidden_out is not None:
            hidden_out.append(h)
    pooled = vision_pooler(h, pos, num_soft_tokens, c["pool"])
    return embedder(pooled, W["model.embed_vision.embedding_projection.weight"], c["eps"])


def _aud(i, name):
    return f"model.audio_tower.layers.{i}.{name}"


def _packed(W, prefix, x, inp, out):
    _tap(prefix, x)
    w = W[f"{prefix}.weight"]
    bits = derive_packed_bits(w.nbytes, inp, out)
    return packed_qat_linear(x, w, W[f"{prefix}.weight_scale"], inp, out, bits, float(W[f"{prefix}.input_activation_scale"]),
                             float(W[f"{prefix}.output_activation_scale"]))


def audio_ffn(W, i, blk, h):
    """computeAudioFeedForwardGpuOnly dataflow, src/audio/encoder.ts:841-921."""
    c = AUDIO
    x = rmsnorm(h, W[_aud(i, f"{blk}.pre_layer_norm.weight")], c["eps"])
    x = silu(_packed(W, _aud(i, f"{blk}.ffw_layer_1.linear"), x, c["hidden"], c["ff"]))
    x = _packed(W, _aud(i, f"{blk}.ffw_layer_2.linear"), x, c["ff"], c["hidden"])
    x = rmsnorm(x, W[_aud(i, f"{blk}.post_layer_norm.weight")], c["eps"])
    return scaled_residual_add(h, x, c["residual"])


def audio_relative_keys(W, i) -> np.ndarray:
    c = AUDIO
    return f32_linear_rows(audio_relpos(c["plen"], c["hidden"]), W[_aud(i, "self_attn.relative_k_proj.weight")])


def audio_qkv(W, i, x):
    """q, k, v projections of audio layer i (src/audio/encoder.ts:1019-1036)."""
    d = AUDIO["hidden"]
    return tuple(_packed(W, _aud(i, f"self_attn.{p}_proj.linear"), x, d, d) for p in "qkv")


def audio_attention_block(W, i, x):
    """computeAudioSelfAttentionGpuOnly dataflow, src/audio/encoder.ts:1011-1071."""
    c = AUDIO
    d = c["hidden"]
    q, k, v = audio_qkv(W, i, x)
    rk = audio_relative_keys(W, i)
    o = audio_attention(q, k, v, rk, W[_aud(i, "self_attn.per_dim_scale")], c["heads"], c["head_dim"], c["chunk"], c["ctx"],
                        c["plen"], c["softcap"])
    return _packed(W, _aud(i, "self_attn.post.linear"), o, d, d)


def audio_light_conv(W, i, h):
    """computeAudioLightConvGpuOnly dataflow, src/audio/encoder.ts:923-1009."""
    c = AUDIO
    d = c["hidden"]
    x = rmsnorm(h, W[_aud(i, "lconv1d.pre_layer_norm.weight")], c["eps"])
    x = _packed(W, _aud(i, "lconv1d.linear_start.linear"), x, d, c["expanded"])
    x = glu(x, d)
    x = depthwise_causal(x, W[_aud(i, "lconv1d.depthwise_conv1d.weight")], c["kernel"])
    x = silu(rmsnorm(x, W[_aud(i, "lconv1d.conv_norm.weight")], c["eps"]))
    x = _packed(W, _aud(i, "lconv1d.linear_end.linear"), x, d, d)
    return residual_add(h, x)


def audio_layer(W, i, h):
    """computeAudioEncoderLayerGpuOnly dataflow, src/audio/encoder.ts:761-839."""
    c = AUDIO
    h1 = audio_ffn(W, i, "feed_forward1", h)
    a = rmsnorm(h1, W[_aud(i, "norm_pre_attn.weight")], c["eps"])
    att = audio_attention_block(W, i, a)
    h2 = residual_add(h1, rmsnorm(att, W[_aud(i, "norm_post_attn.weight")], c["eps"]))
    h3 = audio_light_conv(W, i, h2)
    h4 = audio_ffn(W, i, "feed_forward2", h3)
    return rmsnorm(h4, W[_aud(i, "norm_out.weight")], c["eps"])


def audio_subsample(W, feats, mask):
    """runAudioSubsampleProjectionCpu, src/audio/kernels.ts:22-62."""
    c = AUDIO
    p = "model.audio_tower.subsample_conv_projection"
    frames, fs = feats.shape
    y0, m0, t0, f0 = audio_subsample_conv_layer(feats, mask, frames, fs, 1, W[f"{p}.layer0.conv.weight"], W[f"{p}.layer0.norm.weight"], 128, c["eps"])
    y1, m1, t1, f1 = audio_subsample_conv_layer(y0, m0, t0, f0, 128, W[f"{p}.layer1.conv.weight"], W[f"{p}.layer1.norm.weight"], 32, c["eps"])
    if f1 * 32 != c["hidden"]:
        raise ValueError(f"Audio subsample flattened dim {f1 * 32} does not match hidden size {c['hidden']}.")
    out = f32_linear_rows(y1.reshape(t1, f1 * 32), W[f"{p}.input_proj_linear.weight"])
    return out, m1


def audio_embed(W: Dict[str, np.ndarray], samples: np.ndarray, sampling_rate: int = 16000, layer_count: int = 12,
                max_samples: Optional[int] = None, hidden_out: Optional[list] = None) -> Dict:
    """computeGemma4AudioEmbeddings compute path, src/audio/index.ts:52-133."""
    c = AUDIO
    pre = preprocess_audio(samples, sampling_rate=sampling_rate, max_samples=max_samples if max_samples else 480000,
                           pad_to_multiple_of=None)
    if pre["frames"] == 0:
        raise ValueError("Audio preprocessing produced no frames.")
    h, mask = audio_subsample(W, pre["inputFeatures"], pre["inputFeaturesMask"])
    if hidden_out is not None:
        hidden_out.append(h)
    for i in range(layer_count):
        h = audio_layer(W, i, h)
        if hidden_out is not None:
            hidden_out.append(h)
    proj = add_bias_rows(f32_linear_rows(h, W["model.audio_tower.output_proj.weight"]), W["model.audio_tower.output_proj.bias"])
    rows = strip_rows_by_mask(proj, mask)
    emb = embedder(rows, W["model.embed_audio.embedding_projection.weight"], c["eps"])
    return {"embeddings": emb, "frames": pre["frames"], "validFrames": pre["validFrames"], "subsampleRows": int(mask.size),
            "validSubsampleRows": int(np.count_nonzero(mask)), "mask": mask}
