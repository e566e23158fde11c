"""Seeded synthetic checkpoints and inputs for the Gemma 4 E2B media towers.

The real checkpoint (google/gemma-4-E2B-it-qat-mobile-transformers) cannot be
fetched here, so tests, the smoke run and the benchmark use random-init weights
that carry the reference's tensor names, dtypes and shapes
(src/model.ts:25-296 and the shape asserts in src/vision/encoder.ts,
src/audio/encoder.ts, src/audio/index.ts:62-73, src/vision/index.ts:46-60,
src/embedder/index.ts:26-41).

Every value comes from one documented generator so that any consumer (this
module, the C oracle harness, a future Node harness) can reproduce it without
depending on numpy's RNG: tensor `name` under `seed` uses the counter stream
    u64[i] = splitmix64_mix(key + (i + 1) * 0x9E3779B97F4A7C15),
    key    = splitmix64_mix(seed * 0x100000001B3 ^ crc32(name)),
uniforms are (u64 >> 11) * 2**-53, normals are Box-Muller over consecutive
uniform pairs (u1, u2): sqrt(-2 ln(1 - u1)) * cos(2 pi u2).

Distributions (int8 codes uniform in [-127, 127], per-channel weight scales
U(0.002, 0.02), activation scales 0, norm weights 1 + N(0, 0.02), BF16/F32
projection weights N(0, 0.02)) follow the benchmark configuration of the
reference's int8 linear and towers.
"""
from __future__ import annotations

import json
import struct
import zlib
from typing import Dict, Iterable, Tuple

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)

VISION_LAYERS = 16
AUDIO_LAYERS = 12
VISION_HIDDEN = 768
VISION_FF = 3072
VISION_HEAD_DIM = 64
VISION_POSITION_ROWS = 1024
TEXT_HIDDEN = 1536
AUDIO_HIDDEN = 1024
AUDIO_FF = 4096
AUDIO_HEAD_DIM = 128
AUDIO_KERNEL = 5
AUDIO_OUTPUT = 1536


def _mix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def stream_u64(seed: int, name: str, n: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        key0 = np.array([(seed * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF], dtype=np.uint64)
        key0 ^= np.uint64(zlib.crc32(name.encode()))
        key = _mix(key0 + _GOLDEN)[0]
        idx = np.arange(1, n + 1, dtype=np.uint64)
        return _mix(key + idx * _GOLDEN)


def uniform(seed: int, name: str, n: int) -> np.ndarray:
    """U[0, 1) doubles."""
    return (stream_u64(seed, name, n) >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)


def normal(seed: int, name: str, n: int) -> np.ndarray:
    u = uniform(seed, name, 2 * n).reshape(n, 2)
    return np.sqrt(-2.0 * np.log1p(-u[:, 0])) * np.cos(2.0 * np.pi * u[:, 1])


def int_uniform(seed: int, name: str, n: int, lo: int, hi: int) -> np.ndarray:
    """Integers uniform in [lo, hi] (inclusive)."""
    return (np.floor(uniform(seed, name, n) * (hi - lo + 1)) + lo).astype(np.int64)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bit patterns (round to nearest even), as uint16."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return b.astype(np.uint16)


def f32_from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """float32FromBf16Bytes, src/io/safetensors.ts:151-164."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


# --------------------------------------------------------------------------
# Tensor name tables (src/model.ts)
# --------------------------------------------------------------------------

def qat_names(prefix: str) -> Dict[str, str]:
    return {
        "weight": f"{prefix}.weight",
        "weightScale": f"{prefix}.weight_scale",
        "inputScale": f"{prefix}.input_activation_scale",
        "outputScale": f"{prefix}.output_activation_scale",
    }


def vision_layer_prefix(i: int) -> str:
    return f"model.vision_tower.encoder.layers.{i}"


def audio_layer_prefix(i: int) -> str:
    return f"model.audio_tower.layers.{i}"


VISION_PATCH_PROJ = "model.vision_tower.patch_embedder.input_proj.weight"
VISION_POS_TABLE = "model.vision_tower.patch_embedder.position_embedding_table"
VISION_EMBED = "model.embed_vision.embedding_projection.weight"
AUDIO_SUB = "model.audio_tower.subsample_conv_projection"
AUDIO_OUT_W = "model.audio_tower.output_proj.weight"
AUDIO_OUT_B = "model.audio_tower.output_proj.bias"
AUDIO_EMBED = "model.embed_audio.embedding_projection.weight"


def _qat_i8(seed: int, t: Dict[str, np.ndarray], prefix: str, out: int, inp: int, s_in: float, s_out: float):
    n = qat_names(prefix)
    t[n["weight"]] = int_uniform(seed, n["weight"], out * inp, -127, 127).astype(np.int8).reshape(out, inp)
    t[n["weightScale"]] = (0.002 + 0.018 * uniform(seed, n["weightScale"], out)).astype(np.float32).reshape(out, 1)
    t[n["inputScale"]] = np.array(s_in, dtype=np.float32).reshape(())
    t[n["outputScale"]] = np.array(s_out, dtype=np.float32).reshape(())


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """Pack [out, in] codes into the U8 layout read by packedQatWeightCode
    (src/kernels/qat.ts:249-261): lane j of byte b holds column b*(8/bits)+j
    in bits [j*bits, (j+1)*bits)."""
    out, inp = codes.shape
    vpb = 8 // bits
    c = codes.astype(np.uint8).reshape(out, inp // vpb, vpb)
    packed = np.zeros((out, inp // vpb), dtype=np.uint8)
    for j in range(vpb):
        packed |= (c[:, :, j] & ((1 << bits) - 1)) << (j * bits)
    return packed


def _qat_u8(seed: int, t: Dict[str, np.ndarray], prefix: str, out: int, inp: int, bits: int, s_in: float, s_out: float):
    n = qat_names(prefix)
    zp = 1 << (bits - 1)
    codes = int_uniform(seed, n["weight"], out * inp, 1, 2 * zp - 1).reshape(out, inp)
    t[n["weight"]] = pack_codes(codes, bits) if bits != 8 else codes.astype(np.uint8)
    t[n["weightScale"]] = (0.002 + 0.018 * uniform(seed, n["weightScale"], out)).astype(np.float32).reshape(out, 1)
    t[n["inputScale"]] = np.array(s_in, dtype=np.float32).reshape(())
    t[n["outputScale"]] = np.array(s_out, dtype=np.float32).reshape(())


def _bf16(seed: int, name: str, shape: Tuple[int, ...], mean: float, std: float) -> np.ndarray:
    n = int(np.prod(shape))
    return bf16_bits((mean + std * normal(seed, name, n)).astype(np.float32)).reshape(shape)


def _f32(seed: int, name: str, shape: Tuple[int, ...], mean: float, std: float) -> np.ndarray:
    n = int(np.prod(shape))
    return (mean + std * normal(seed, name, n)).astype(np.float32).reshape(shape)


# Static input-activation quantisation at fixed per-linear scales: absmax/127
# of each linear's input, with the absmax measured once on a seeded 768 x 768
# image (vision) and a 30 s clip (audio) through these random-init towers.
# Used to time the quantised mode (one-term GEMMs on integer codes); parity
# tests calibrate on their own inputs instead.
VISION_INPUT_ABSMAX = {"q_proj": 4.79, "k_proj": 4.79, "v_proj": 4.79, "o_proj": 4.59,
                       "gate_proj": 5.69, "up_proj": 5.69, "down_proj": 13260.0}
AUDIO_INPUT_ABSMAX = {"ffw_layer_1": 4.68, "ffw_layer_2": 188.8, "q_proj": 5.31, "k_proj": 5.31, "v_proj": 5.31,
                      "post": 156.6, "linear_start": 6.08, "linear_end": 10.9}


def _s_in(s_in, table, name):
    """s_in: a number (every linear), or "calibrated" (the fixed table above)."""
    if s_in == "calibrated":
        return float(np.float32(table[name] / 127.0))
    return float(s_in)


def vision_weights(seed: int = 0, layers: int = VISION_LAYERS, s_in=0.0, s_out: float = 0.0) -> Dict[str, np.ndarray]:
    """Vision tower + embedder with the reference dtypes: I8 QAT linears,
    BF16 norms / patch projection / position table, F32 embedder.  s_in is
    one input_activation_scale for every linear or "calibrated"."""
    d, ff, hd = VISION_HIDDEN, VISION_FF, VISION_HEAD_DIM
    t: Dict[str, np.ndarray] = {}
    t[VISION_PATCH_PROJ] = _bf16(seed, VISION_PATCH_PROJ, (d, 768), 0.0, 0.02)
    t[VISION_POS_TABLE] = _bf16(seed, VISION_POS_TABLE, (2, VISION_POSITION_ROWS, d), 0.0, 0.02)
    t[VISION_EMBED] = _f32(seed, VISION_EMBED, (TEXT_HIDDEN, d), 0.0, 0.02)
    for i in range(layers):
        p = vision_layer_prefix(i)
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            _qat_i8(seed, t, f"{p}.self_attn.{proj}.linear", d, d, _s_in(s_in, VISION_INPUT_ABSMAX, proj), s_out)
        _qat_i8(seed, t, f"{p}.mlp.gate_proj.linear", ff, d, _s_in(s_in, VISION_INPUT_ABSMAX, "gate_proj"), s_out)
        _qat_i8(seed, t, f"{p}.mlp.up_proj.linear", ff, d, _s_in(s_in, VISION_INPUT_ABSMAX, "up_proj"), s_out)
        _qat_i8(seed, t, f"{p}.mlp.down_proj.linear", d, ff, _s_in(s_in, VISION_INPUT_ABSMAX, "down_proj"), s_out)
        for nm in ("q_norm", "k_norm"):
            name = f"{p}.self_attn.{nm}.weight"
            t[name] = _bf16(seed, name, (hd,), 1.0, 0.02)
        for nm in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm", "post_feedforward_layernorm"):
            name = f"{p}.{nm}.weight"
            t[name] = _bf16(seed, name, (d,), 1.0, 0.02)
    return t


def audio_weights(seed: int = 0, layers: int = AUDIO_LAYERS, bits: int = 8, s_in=0.0, s_out: float = 0.0) -> Dict[str, np.ndarray]:
    """Audio tower + embedder with the reference dtypes: U8 packed QAT
    linears (zero point 2**(bits-1)), F32 norms, convs and projections.
    s_in is one input_activation_scale for every linear or "calibrated"."""
    d, ff = AUDIO_HIDDEN, AUDIO_FF
    t: Dict[str, np.ndarray] = {}
    t[f"{AUDIO_SUB}.layer0.conv.weight"] = _f32(seed, f"{AUDIO_SUB}.layer0.conv.weight", (128, 1, 3, 3), 0.0, 0.02)
    t[f"{AUDIO_SUB}.layer0.norm.weight"] = _f32(seed, f"{AUDIO_SUB}.layer0.norm.weight", (128,), 1.0, 0.02)
    t[f"{AUDIO_SUB}.layer1.conv.weight"] = _f32(seed, f"{AUDIO_SUB}.layer1.conv.weight", (32, 128, 3, 3), 0.0, 0.02)
    t[f"{AUDIO_SUB}.layer1.norm.weight"] = _f32(seed, f"{AUDIO_SUB}.layer1.norm.weight", (32,), 1.0, 0.02)
    t[f"{AUDIO_SUB}.input_proj_linear.weight"] = _f32(seed, f"{AUDIO_SUB}.input_proj_linear.weight", (d, d), 0.0, 0.02)
    t[AUDIO_OUT_W] = _f32(seed, AUDIO_OUT_W, (AUDIO_OUTPUT, d), 0.0, 0.02)
    t[AUDIO_OUT_B] = _f32(seed, AUDIO_OUT_B, (AUDIO_OUTPUT,), 0.0, 0.02)
    t[AUDIO_EMBED] = _f32(seed, AUDIO_EMBED, (TEXT_HIDDEN, AUDIO_OUTPUT), 0.0, 0.02)
    for i in range(layers):
        p = audio_layer_prefix(i)
        for blk in ("feed_forward1", "feed_forward2"):
            _qat_u8(seed, t, f"{p}.{blk}.ffw_layer_1.linear", ff, d, bits, _s_in(s_in, AUDIO_INPUT_ABSMAX, "ffw_layer_1"), s_out)
            _qat_u8(seed, t, f"{p}.{blk}.ffw_layer_2.linear", d, ff, bits, _s_in(s_in, AUDIO_INPUT_ABSMAX, "ffw_layer_2"), s_out)
            for nm in ("pre_layer_norm", "post_layer_norm"):
                name = f"{p}.{blk}.{nm}.weight"
                t[name] = _f32(seed, name, (d,), 1.0, 0.02)
        for proj in ("q_proj", "k_proj", "v_proj", "post"):
            _qat_u8(seed, t, f"{p}.self_attn.{proj}.linear", d, d, bits, _s_in(s_in, AUDIO_INPUT_ABSMAX, proj), s_out)
        t[f"{p}.self_attn.per_dim_scale"] = _f32(seed, f"{p}.self_attn.per_dim_scale", (AUDIO_HEAD_DIM,), 0.0, 0.02)
        t[f"{p}.self_attn.relative_k_proj.weight"] = _f32(seed, f"{p}.self_attn.relative_k_proj.weight", (d, d), 0.0, 0.02)
        _qat_u8(seed, t, f"{p}.lconv1d.linear_start.linear", 2 * d, d, bits, _s_in(s_in, AUDIO_INPUT_ABSMAX, "linear_start"), s_out)
        _qat_u8(seed, t, f"{p}.lconv1d.linear_end.linear", d, d, bits, _s_in(s_in, AUDIO_INPUT_ABSMAX, "linear_end"), s_out)
        for nm in ("pre_layer_norm", "conv_norm"):
            name = f"{p}.lconv1d.{nm}.weight"
            t[name] = _f32(seed, name, (d,), 1.0, 0.02)
        t[f"{p}.lconv1d.depthwise_conv1d.weight"] = _f32(seed, f"{p}.lconv1d.depthwise_conv1d.weight", (d, 1, AUDIO_KERNEL), 0.0, 0.2)
        for nm in ("norm_pre_attn", "norm_post_attn", "norm_out"):
            name = f"{p}.{nm}.weight"
            t[name] = _f32(seed, name, (d,), 1.0, 0.02)
    return t


# --------------------------------------------------------------------------
# Inputs
# --------------------------------------------------------------------------

def qat_linear_case(seed: int = 0, rows: int = 256, inp: int = 768, out: int = 768):
    """int8 QAT linear: x ~ N(0,1) f32 [rows,in], W int8 U[-127,127] [out,in],
    s_w ~ U(0.002,0.02) [out], bias ~ N(0,0.02) [out]."""
    x = normal(seed, "qat.x", rows * inp).astype(np.float32).reshape(rows, inp)
    w = int_uniform(seed, "qat.w", out * inp, -127, 127).astype(np.int8).reshape(out, inp)
    s = (0.002 + 0.018 * uniform(seed, "qat.s", out)).astype(np.float32)
    b = (0.02 * normal(seed, "qat.b", out)).astype(np.float32)
    return x, w, s, b


def image_pixels(seed: int, height: int, width: int) -> np.ndarray:
    """RGB float32 [h, w, 3] with values U[0, 1]."""
    return uniform(seed, f"image.{height}x{width}", height * width * 3).astype(np.float32).reshape(height, width, 3)


def audio_samples(seed: int, n: int, std: float = 0.1) -> np.ndarray:
    """Mono float32 waveform ~ N(0, std)."""
    return (std * normal(seed, f"audio.{n}", n)).astype(np.float32)


def audio_batch_lengths(seed: int, count: int, lo_s: float = 1.0, hi_s: float = 30.0, rate: int = 16000) -> np.ndarray:
    """Clip lengths in samples, uniform in [lo_s, hi_s] seconds."""
    u = uniform(seed, "audio.batch.lengths", count)
    return np.floor((lo_s + (hi_s - lo_s) * u) * rate).astype(np.int64)


# --------------------------------------------------------------------------
# safetensors
# --------------------------------------------------------------------------

_DTYPE = {np.dtype(np.int8): "I8", np.dtype(np.uint8): "U8", np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32"}
_NP = {"I8": np.int8, "U8": np.uint8, "BF16": np.uint16, "F32": np.float32}


def write_safetensors(path: str, tensors: Dict[str, np.ndarray], dtypes: Dict[str, str] | None = None) -> None:
    """Write a safetensors file.  uint16 arrays are written as BF16."""
    header = {}
    off = 0
    order = sorted(tensors)
    arrays = {}
    for name in order:
        a = np.asarray(tensors[name])
        arrays[name] = a if a.flags.c_contiguous else a.copy()  # keeps 0-d scalars 0-d
    for name in order:
        a = arrays[name]
        dt = (dtypes or {}).get(name) or _DTYPE[a.dtype]
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    header["__metadata__"] = {"format": "pt", "generator": "synthetic-splitmix64"}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for name in order:
            f.write(arrays[name].tobytes())


def read_safetensors(path: str) -> Dict[str, np.ndarray]:
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
        out = {}
        for name, info in header.items():
            if name == "__metadata__":
                continue
            f.seek(base + info["data_offsets"][0])
            nb = info["data_offsets"][1] - info["data_offsets"][0]
            out[name] = np.frombuffer(f.read(nb), dtype=_NP[info["dtype"]]).reshape(info["shape"])
        return out


def merge(*dicts: Iterable[Dict[str, np.ndarray]]) -> Dict[str, np.ndarray]:
    out: Dict[str, np.ndarray] = {}
    for d in dicts:
        out.update(d)
    return out
