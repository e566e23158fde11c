"""ctypes bindings to libg4m.so, the CUDA (sm_100a) library behind the API.

There is no CPU fallback: if the library is missing or cannot load, every
entry point raises.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libg4m.so")

G4M_OK = 0
STATUS_NAMES = {0: "OK", 1: "E_ARG", 2: "E_SHAPE", 3: "E_DTYPE", 4: "E_CUDA", 5: "E_TIMEOUT", 6: "E_CANCELLED",
                7: "E_IO", 8: "E_NOT_LOADED", 9: "E_UNSUPPORTED", 10: "E_LAYOUT"}

# (name, restype, argtypes) for every function declared in include/g4m.h
_VP = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
_I64 = ctypes.c_int64
_SIGS = [
    ("g4m_create", _VP, [_VP, _I]),
    ("g4m_destroy", None, [_VP]),
    ("g4m_device_count", _I, [_VP]),
    ("g4m_last_error", ctypes.c_char_p, []),
    ("g4m_load_weights", _I, [_VP, ctypes.c_char_p]),
    ("g4m_loaded_towers", _I, [_VP]),
    ("g4m_cancel", None, [_VP]),
    ("g4m_clear_cancel", None, [_VP]),
    ("g4m_set_debug", _I, [_VP, _I]),
    ("g4m_qat_linear", _I, [_VP, _I, _VP, _I, _I, _I, _VP, _I, _VP, _F, _F, _VP, _VP]),
    ("g4m_linear_prepare", _I, [_VP, _I, _VP, _I, _I, _I, _VP, _F, _F, _VP, ctypes.POINTER(_VP)]),
    ("g4m_linear_run", _I, [_VP, _VP, _I, _VP, _VP]),
    ("g4m_linear_free", None, [_VP]),
    ("g4m_linear_run_noalloc", _I, [_VP, _VP, _I, _VP, _VP]),
    ("g4m_vision_embed_images", _I, [_VP, _I, _VP, _VP, _VP, _I, _I, _I, _VP, _VP, _VP]),
    ("g4m_resize_rgb", _I, [_VP, _I, _VP, _I, _I, _I, _I, _I, _VP]),
    ("g4m_selftest_wait_timeout", _I, [_VP, _I, ctypes.c_longlong]),
    ("g4m_vision_embed_batch", _I, [_VP, _I, _VP, _I, _I, _I, _I, _VP, _VP, _VP]),
    ("g4m_vision_embed_device", _I, [_VP, _I, _I, _VP, _I, _I, _I, _I, _VP, _VP]),
    ("g4m_vision_debug_hidden", _I, [_VP, _I, _I, _VP, ctypes.c_size_t]),
    ("g4m_vision_layers", _I, [_VP, _I, _I, _I, _I, _I, _I, _VP]),
    ("g4m_audio_embed_batch", _I, [_VP, _I, _VP, _VP, _I, _I, _I64, _VP, _VP, _VP]),
    ("g4m_audio_embed_device", _I, [_VP, _I, _I, _VP, _VP, _VP, _I, _I, _I64, _VP, _VP, _VP]),
    ("g4m_audio_debug_hidden", _I, [_VP, _I, _I, _VP, ctypes.c_size_t]),
    ("g4m_audio_layers", _I, [_VP, _I, _I, _VP, _I, _I, _VP]),
    ("g4m_image_token_layout", _I, [_I, _I, _I, _I, _I, ctypes.POINTER(_I64)]),
    ("g4m_audio_soft_token_count", _I64, [_I64, _I, _I, _I]),
    ("g4m_checksum_floats", ctypes.c_double, [_VP, _I64]),
    ("g4m_profile_begin", _I, [_VP, _I]),
    ("g4m_profile_end", _I, [_VP, _I, ctypes.c_char_p, ctypes.c_size_t]),
    ("g4m_kernel_launches", ctypes.c_longlong, []),
    ("g4m_version", ctypes.c_char_p, []),
]

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libg4m.so is not built ({LIB_PATH}); run build() first -- there is no CPU fallback")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in _SIGS:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_names():
    return [s[0] for s in _SIGS]


class G4MError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status
        self.message = message


def last_error() -> str:
    m = lib().g4m_last_error()
    return m.decode() if m else ""


def check(rc: int) -> None:
    if rc != G4M_OK:
        raise G4MError(rc, last_error())


def ptr(a: np.ndarray):
    return ctypes.c_void_p(a.ctypes.data)


class Context:
    """Owns a g4m_ctx (resident weights on one or more CUDA devices)."""

    def __init__(self, devices=None):
        L = lib()
        if devices:
            arr = (ctypes.c_int * len(devices))(*devices)
            self.h = L.g4m_create(ctypes.cast(arr, ctypes.c_void_p), len(devices))
        else:
            self.h = L.g4m_create(None, 0)
        if not self.h:
            raise G4MError(4, last_error())

    def close(self):
        if getattr(self, "h", None):
            lib().g4m_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def device_count(self) -> int:
        return lib().g4m_device_count(self.h)

    def load_weights(self, path: str) -> None:
        check(lib().g4m_load_weights(self.h, path.encode()))

    @property
    def loaded_towers(self) -> int:
        return lib().g4m_loaded_towers(self.h)

    def cancel(self):
        lib().g4m_cancel(self.h)

    def clear_cancel(self):
        lib().g4m_clear_cancel(self.h)

    def profile_begin(self, device=0):
        check(lib().g4m_profile_begin(self.h, device))

    def profile_end(self, device=0) -> dict:
        import json
        buf = ctypes.create_string_buffer(1 << 16)
        check(lib().g4m_profile_end(self.h, device, buf, len(buf)))
        return {k: (int(v[0]), float(v[1])) for k, v in json.loads(buf.value.decode()).items()}

    def set_debug(self, on: bool):
        check(lib().g4m_set_debug(self.h, 1 if on else 0))

    def qat_linear(self, x, w, w_scale, s_in=0.0, s_out=0.0, bias=None, bits=0, in_dim=None, device=0) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        rows, inp = x.shape
        if bits == 0:
            w = np.ascontiguousarray(w, dtype=np.int8)
            out = w.shape[0]
        else:
            w = np.ascontiguousarray(w, dtype=np.uint8)
            out = w.shape[0]
        s = np.ascontiguousarray(w_scale, dtype=np.float32).reshape(-1)
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32).reshape(-1)
        y = np.empty((rows, out), np.float32)
        check(lib().g4m_qat_linear(self.h, device, ptr(x), rows, inp, out, ptr(w), bits, ptr(s), float(s_in), float(s_out),
                                   None if b is None else ptr(b), ptr(y)))
        return y

    def vision_embed(self, pixels_list, max_soft_tokens=280, layer_count=16, outs=None):
        """pixels_list: list of float32 [h, w, 3] arrays of one size; `outs`
        optionally supplies the [tokens, 1536] float32 output arrays."""
        n = len(pixels_list)
        if n == 0:
            return [], []
        h, w = pixels_list[0].shape[:2]
        pix = [np.ascontiguousarray(p, dtype=np.float32) for p in pixels_list]
        lay = (ctypes.c_int64 * 6)()
        check(lib().g4m_image_token_layout(h, w, 16, max_soft_tokens, 3, lay))
        tokens = lay[5]
        if outs is None:
            outs = [np.empty((tokens, 1536), np.float32) for _ in range(n)]
        elif any(o.shape != (tokens, 1536) or o.dtype != np.float32 or not o.flags.c_contiguous for o in outs):
            raise ValueError("outs must be C-contiguous float32 [tokens, 1536] arrays")
        pin = (ctypes.c_void_p * n)(*[p.ctypes.data for p in pix])
        pout = (ctypes.c_void_p * n)(*[o.ctypes.data for o in outs])
        rows = np.zeros(n, np.int32)
        status = np.zeros(n, np.int32)
        rc = lib().g4m_vision_embed_batch(self.h, n, ctypes.cast(pin, ctypes.c_void_p), h, w, max_soft_tokens, layer_count,
                                          ctypes.cast(pout, ctypes.c_void_p), ptr(rows), ptr(status))
        check(rc)
        return outs, rows

    def vision_embed_images(self, images, max_soft_tokens=280, layer_count=16):
        """images: list of uint8 [h, w, 3 | 4] arrays of any sizes (one channel
        count).  Returns ([tokens_i, 1536] float32 arrays, rows, statuses);
        per-image failures are reported in the statuses, not raised."""
        n = len(images)
        if n == 0:
            return [], np.zeros(0, np.int32), np.zeros(0, np.int32)
        imgs = [np.ascontiguousarray(im, dtype=np.uint8) for im in images]
        ch = imgs[0].shape[2]
        if any(im.ndim != 3 or im.shape[2] != ch for im in imgs):
            raise ValueError("images must be [h, w, c] uint8 with one channel count")
        hs = np.array([im.shape[0] for im in imgs], np.int32)
        ws = np.array([im.shape[1] for im in imgs], np.int32)
        outs = []
        for im in imgs:
            lay = (ctypes.c_int64 * 6)()
            rc = lib().g4m_image_token_layout(im.shape[0], im.shape[1], 16, max_soft_tokens, 3, lay)
            outs.append(np.empty((max(int(lay[5]), 1) if rc == 0 else 1, 1536), np.float32))
        pin = (ctypes.c_void_p * n)(*[im.ctypes.data for im in imgs])
        pout = (ctypes.c_void_p * n)(*[o.ctypes.data for o in outs])
        rows = np.zeros(n, np.int32)
        status = np.zeros(n, np.int32)
        rc = lib().g4m_vision_embed_images(self.h, n, ctypes.cast(pin, ctypes.c_void_p), ptr(hs), ptr(ws), ch,
                                           max_soft_tokens, layer_count, ctypes.cast(pout, ctypes.c_void_p),
                                           ptr(rows), ptr(status))
        if rc and not (status != 0).any():
            check(rc)
        return [o[: int(r)] for o, r in zip(outs, rows)], rows, status

    def resize_rgb(self, image, target_height: int, target_width: int, device=0) -> np.ndarray:
        im = np.ascontiguousarray(image, dtype=np.uint8)
        out = np.empty((target_height, target_width, 3), np.float32)
        check(lib().g4m_resize_rgb(self.h, device, ptr(im), im.shape[0], im.shape[1], im.shape[2], target_height,
                                   target_width, ptr(out)))
        return out

    def vision_embed_device(self, pixels_ptr: int, n: int, height: int, width: int, out_ptr: int, max_soft_tokens=280,
                            layer_count=16, stream: int = 0, device=0) -> None:
        check(lib().g4m_vision_embed_device(self.h, device, n, ctypes.c_void_p(pixels_ptr), height, width, max_soft_tokens,
                                            layer_count, ctypes.c_void_p(out_ptr), ctypes.c_void_p(stream) if stream else None))

    def vision_debug_hidden(self, which: int, rows: int, device=0) -> np.ndarray:
        out = np.empty((rows, 768), np.float32)
        check(lib().g4m_vision_debug_hidden(self.h, device, which, ptr(out), out.size))
        return out

    def vision_layers(self, h: np.ndarray, n: int, height: int, width: int, first: int, count: int, device=0) -> np.ndarray:
        h = np.ascontiguousarray(h, dtype=np.float32).copy()
        check(lib().g4m_vision_layers(self.h, device, n, height, width, first, count, ptr(h)))
        return h

    def audio_embed(self, clips, sampling_rate=16000, layer_count=12, max_samples=0, outs=None):
        """clips: list of float32 sample arrays; `outs` optionally supplies
        C-contiguous float32 output arrays of at least [rows_i, 1536] each."""
        n = len(clips)
        xs = [np.ascontiguousarray(c, dtype=np.float32).reshape(-1) for c in clips]
        lens = np.array([x.size for x in xs], np.int64)
        cap = max_samples if max_samples else 480000
        need = [int(lib().g4m_audio_soft_token_count(min(x.size, cap), 320, 160, 750)) for x in xs]
        if outs is None:
            outs = [np.empty((max(r, 1), 1536), np.float32) for r in need]
        elif any(o.dtype != np.float32 or not o.flags.c_contiguous or o.ndim != 2 or o.shape[1] != 1536
                 or o.shape[0] < r for o, r in zip(outs, need)):
            raise ValueError("outs must be C-contiguous float32 [>= rows, 1536] arrays")
        pin = (ctypes.c_void_p * n)(*[x.ctypes.data for x in xs])
        pout = (ctypes.c_void_p * n)(*[o.ctypes.data for o in outs])
        rows = np.zeros(n, np.int32)
        status = np.zeros(n, np.int32)
        check(lib().g4m_audio_embed_batch(self.h, n, ctypes.cast(pin, ctypes.c_void_p), ptr(lens), sampling_rate, layer_count,
                                          int(max_samples), ctypes.cast(pout, ctypes.c_void_p), ptr(rows), ptr(status)))
        return [o[: int(r)] for o, r in zip(outs, rows)], rows

    def audio_debug_hidden(self, rows: int, which: int = 1, device=0) -> np.ndarray:
        out = np.empty((rows, 3072 if which == 2 else 1024), np.float32)
        check(lib().g4m_audio_debug_hidden(self.h, device, which, ptr(out), out.size))
        return out

    def audio_layers(self, h: np.ndarray, rows_per_clip, first: int, count: int, device=0) -> np.ndarray:
        h = np.ascontiguousarray(h, dtype=np.float32).copy()
        rows = np.ascontiguousarray(rows_per_clip, dtype=np.int32)
        check(lib().g4m_audio_layers(self.h, device, rows.size, ptr(rows), first, count, ptr(h)))
        return h

    def audio_embed_device(self, samples_ptr: int, offsets: np.ndarray, lengths: np.ndarray, out_ptr: int,
                           sampling_rate=16000, layer_count=12, max_samples=0, stream: int = 0, device=0) -> np.ndarray:
        offsets = np.ascontiguousarray(offsets, dtype=np.int64)
        lengths = np.ascontiguousarray(lengths, dtype=np.int64)
        rows = np.zeros(offsets.size, np.int32)
        check(lib().g4m_audio_embed_device(self.h, device, offsets.size, ctypes.c_void_p(samples_ptr), ptr(offsets),
                                           ptr(lengths), sampling_rate, layer_count, int(max_samples),
                                           ctypes.c_void_p(out_ptr), ptr(rows), ctypes.c_void_p(stream) if stream else None))
        return rows


def image_token_layout(height: int, width: int, patch_size: int, max_soft_tokens: int, pooling_kernel_size: int):
    out = (ctypes.c_int64 * 6)()
    check(lib().g4m_image_token_layout(int(height), int(width), int(patch_size), int(max_soft_tokens),
                                       int(pooling_kernel_size), out))
    return list(out)


def audio_soft_token_count(samples: int, frame_length: int, hop_length: int, audio_seq_length: int) -> int:
    return int(lib().g4m_audio_soft_token_count(int(samples), int(frame_length), int(hop_length), int(audio_seq_length)))


def checksum_floats(values: np.ndarray) -> int:
    v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    return int(lib().g4m_checksum_floats(ptr(v), v.size))


def kernel_launches() -> int:
    return int(lib().g4m_kernel_launches())


def version() -> str:
    return lib().g4m_version().decode()
