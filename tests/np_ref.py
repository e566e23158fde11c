"""Independent float64 numpy restatement of the reference CPU twins.

Written separately from oracle/g4m_oracle.c (vectorised, double precision,
no Math.fround emulation) so the two can cross-check each other; agreement
is expected to f32 rounding level, not bit for bit.  Sources are the same
reference functions the oracle cites.
"""
import numpy as np


def srq(v, s):
    if s == 0:
        return v
    q = v / s
    r = np.floor(q)
    r = np.where(q - r >= 0.5, r + 1, r)
    return np.clip(r, -128, 127) * s


def qat_i8(x, w, s_w, s_in=0.0, s_out=0.0):
    a = srq(np.asarray(x, np.float64), s_in)
    return srq((a @ np.asarray(w, np.float64).T) * np.asarray(s_w, np.float64).reshape(-1), s_out)


def unpack_codes(w_u8, inp, bits):
    vpb = 8 // bits
    w = np.asarray(w_u8, np.uint8)
    out = np.zeros((w.shape[0], inp), np.int64)
    for j in range(vpb):
        out[:, j::vpb] = (w >> (j * bits)) & ((1 << bits) - 1)
    return out


def packed_qat(x, w_u8, s_w, inp, bits, s_in=0.0, s_out=0.0):
    codes = unpack_codes(w_u8, inp, bits).astype(np.float64) - 2 ** (bits - 1)
    a = srq(np.asarray(x, np.float64), s_in)
    return srq((a @ codes.T) * np.asarray(s_w, np.float64).reshape(-1), s_out)


def rmsnorm(x, w, eps=1e-6):
    x = np.asarray(x, np.float64)
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * np.asarray(w, np.float64)


def rope(v, pos, heads, hd, theta=100.0):
    v = np.asarray(v, np.float64).reshape(-1, heads, hd)
    out = np.empty_like(v)
    half = hd // 4
    for part in range(2):
        p = np.asarray(pos, np.float64)[:, part][:, None]
        f = np.arange(half)
        ang = p / theta ** (2 * f / (hd / 2))
        c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
        a = v[..., part * 2 * half: part * 2 * half + half]
        b = v[..., part * 2 * half + half: (part + 1) * 2 * half]
        out[..., part * 2 * half: part * 2 * half + half] = a * c - b * s
        out[..., part * 2 * half + half: (part + 1) * 2 * half] = b * c + a * s
    return out.reshape(-1, heads * hd)


def attention(q, k, v, heads, hd):
    q = np.asarray(q, np.float64).reshape(-1, heads, hd).transpose(1, 0, 2)
    k = np.asarray(k, np.float64).reshape(-1, heads, hd).transpose(1, 0, 2)
    v = np.asarray(v, np.float64).reshape(-1, heads, hd).transpose(1, 0, 2)
    s = q @ k.transpose(0, 2, 1)
    s = np.exp(s - s.max(-1, keepdims=True))
    s /= s.sum(-1, keepdims=True)
    return (s @ v).transpose(1, 0, 2).reshape(-1, heads * hd)


def gelu_gate(g, u):
    g = np.asarray(g, np.float64)
    return 0.5 * g * (1 + np.tanh(0.7978845608028654 * (g + 0.044715 * g ** 3))) * np.asarray(u, np.float64)


def pooler(h, gh, gw, k=3):
    h = np.asarray(h, np.float64)
    d = h.shape[-1]
    t = h.reshape(gh // k, k, gw // k, k, d).sum((1, 3)).reshape(-1, d)
    return t / (k * k) * np.sqrt(d)


def embedder(x, w, eps=1e-6):
    x = np.asarray(x, np.float64)
    x = x / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return x @ np.asarray(w, np.float64).T


def patch_embed(patches, w, pos, posx, posy):
    return (2 * (np.asarray(patches, np.float64) - 0.5)) @ np.asarray(w, np.float64).T + \
        np.asarray(posx, np.float64)[pos[:, 0]] + np.asarray(posy, np.float64)[pos[:, 1]]


def subsample_conv(x, mask, in_t, in_f, in_c, w, nw, out_c, eps=1e-6):
    x = np.asarray(x, np.float64).reshape(in_t, in_f, in_c)
    x = x * (np.asarray(mask) != 0)[:, None, None]
    ot, of = (in_t - 1) // 2 + 1, (in_f - 1) // 2 + 1
    xp = np.zeros((in_t + 2, in_f + 2, in_c))
    xp[1:-1, 1:-1] = x
    w = np.asarray(w, np.float64).reshape(out_c, in_c, 3, 3)
    y = np.zeros((ot, of, out_c))
    for kt in range(3):
        for kf in range(3):
            patch = xp[kt: kt + 2 * ot: 2, kf: kf + 2 * of: 2, :]
            y += patch @ w[:, :, kt, kf].T
    mean = y.mean(-1, keepdims=True)
    var = ((y - mean) ** 2).mean(-1, keepdims=True)
    y = (y - mean) / np.sqrt(var + eps) * np.asarray(nw, np.float64)
    m = np.array([mask[2 * i] if 2 * i < in_t else 0 for i in range(ot)], np.uint8)
    return np.maximum(y, 0).reshape(-1), m


def relpos(plen, d):
    half = d // 2
    inc = np.log(10000) / max(half - 1, 1)
    p = (plen - 1 - np.arange(plen))[:, None] * np.exp(np.arange(half) * -inc)[None, :]
    return np.concatenate([np.sin(p), np.cos(p)], 1)


def audio_attention(q, k, v, relk, pds, heads, hd, chunk=12, ctx=24, plen=13, softcap=50.0):
    rows = q.shape[0]
    q = np.asarray(q, np.float64).reshape(rows, heads, hd)
    k = np.asarray(k, np.float64).reshape(rows, heads, hd)
    v = np.asarray(v, np.float64).reshape(rows, heads, hd)
    rk = np.asarray(relk, np.float64).reshape(plen, heads, hd)
    sp = np.log1p(np.exp(np.asarray(pds, np.float64)))
    qs = q * (hd ** -0.5 / np.log(2)) * sp
    ks = k * (np.log(1 + np.e) / np.log(2))
    out = np.zeros_like(q)
    for r in range(rows):
        blk, qp = r // chunk, r % chunk
        src = blk * chunk + np.arange(ctx) - (ctx - chunk)
        ok = (src >= 0) & (src < rows)
        rel = np.arange(ctx) - qp
        rok = (rel >= 0) & (rel < plen)
        s = np.zeros((heads, ctx))
        s[:, ok] += np.einsum("hd,chd->hc", qs[r], ks[src[ok]])
        s[:, rok] += np.einsum("hd,chd->hc", qs[r], rk[rel[rok]])
        s = np.tanh(s / softcap) * softcap
        p = np.exp(s - s.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        out[r] = np.einsum("hc,chd->hd", p[:, ok], v[src[ok]])
    return out.reshape(rows, heads * hd)


def depthwise(x, w, ks=5):
    x = np.asarray(x, np.float64)
    w = np.asarray(w, np.float64).reshape(x.shape[1], ks)
    xp = np.concatenate([np.zeros((ks - 1, x.shape[1])), x], 0)
    return sum(xp[k: k + x.shape[0]] * w[:, k] for k in range(ks))


def logmel(samples, frame_len=320, hop=160, fft=512, nmel=128, sr=16000, fmin=0.0, fmax=8000.0, floor=1e-3):
    x = np.asarray(samples, np.float64)
    wav = np.concatenate([np.zeros(frame_len // 2), x])
    frames = (len(wav) - (frame_len + 1)) // hop + 1 if len(wav) >= frame_len + 1 else 0
    win = 0.5 - 0.5 * np.cos(2 * np.pi * np.arange(frame_len) / frame_len)
    bins = fft // 2 + 1
    mel = lambda f: 2595 * np.log10(1 + f / 700)
    imel = lambda m: 700 * (10 ** (m / 2595) - 1)
    ff = imel(mel(fmin) + (mel(fmax) - mel(fmin)) * np.arange(nmel + 2) / (nmel + 1))
    f = sr / ((bins - 1) * 2) * np.arange(bins)[:, None]
    up = (f - ff[None, :-2]) / (ff[None, 1:-1] - ff[None, :-2])
    dn = (ff[None, 2:] - f) / (ff[None, 2:] - ff[None, 1:-1])
    filt = np.maximum(0, np.minimum(up, dn))
    idx = np.arange(frames)[:, None] * hop + np.arange(frame_len)[None, :]
    spec = np.abs(np.fft.rfft(wav[idx] * win, n=fft, axis=1))
    return np.log(spec @ filt + floor)


def audio_layer(W, i, h):
    """One conformer layer in float64 (src/audio/encoder.ts:761-1071 dataflow)."""
    p = f"model.audio_tower.layers.{i}"
    D = 1024

    def lin(prefix, x, inp, out):
        w = W[f"{prefix}.weight"]
        bits = int(w.nbytes * 8 // (inp * out))
        return packed_qat(x, w, W[f"{prefix}.weight_scale"], inp, bits,
                          float(W[f"{prefix}.input_activation_scale"]), float(W[f"{prefix}.output_activation_scale"]))

    def ffn(blk, h):
        x = rmsnorm(h, W[f"{p}.{blk}.pre_layer_norm.weight"])
        x = lin(f"{p}.{blk}.ffw_layer_1.linear", x, D, 4096)
        x = x / (1 + np.exp(-x))
        x = lin(f"{p}.{blk}.ffw_layer_2.linear", x, 4096, D)
        return h + 0.5 * rmsnorm(x, W[f"{p}.{blk}.post_layer_norm.weight"])

    h = np.asarray(h, np.float64)
    h1 = ffn("feed_forward1", h)
    a = rmsnorm(h1, W[f"{p}.norm_pre_attn.weight"])
    q = lin(f"{p}.self_attn.q_proj.linear", a, D, D)
    k = lin(f"{p}.self_attn.k_proj.linear", a, D, D)
    v = lin(f"{p}.self_attn.v_proj.linear", a, D, D)
    rk = relpos(13, D) @ np.asarray(W[f"{p}.self_attn.relative_k_proj.weight"], np.float64).T
    o = audio_attention(q, k, v, rk, W[f"{p}.self_attn.per_dim_scale"], 8, 128)
    o = lin(f"{p}.self_attn.post.linear", o, D, D)
    h2 = h1 + rmsnorm(o, W[f"{p}.norm_post_attn.weight"])
    x = rmsnorm(h2, W[f"{p}.lconv1d.pre_layer_norm.weight"])
    x = lin(f"{p}.lconv1d.linear_start.linear", x, D, 2 * D)
    x = x[:, :D] / (1 + np.exp(-x[:, D:]))
    x = depthwise(x, W[f"{p}.lconv1d.depthwise_conv1d.weight"])
    x = rmsnorm(x, W[f"{p}.lconv1d.conv_norm.weight"])
    x = x / (1 + np.exp(-x))
    h3 = h2 + lin(f"{p}.lconv1d.linear_end.linear", x, D, D)
    h4 = ffn("feed_forward2", h3)
    return rmsnorm(h4, W[f"{p}.norm_out.weight"])


def resize_rgb(img, th, tw):
    """Antialiased linear (triangle) resize of uint8 [h, w, c] to float
    [th, tw, 3] in [0, 1] with 8-bit rounding: the filter the device uses for
    the canvas drawImage step (radius max(scale, 1), centre (i + 0.5) scale)."""
    img = np.asarray(img, np.float64)[..., :3]

    def axis(n_in, n_out):
        s = n_in / n_out
        r = max(s, 1.0)
        m = np.zeros((n_out, n_in))
        for i in range(n_out):
            c = (i + 0.5) * s
            x = np.arange(max(0, int(np.floor(c - r))), min(n_in - 1, int(np.ceil(c + r))) + 1)
            w = np.maximum(0.0, 1.0 - np.abs(x + 0.5 - c) / r)
            m[i, x] = w / w.sum()
        return m

    h, w = img.shape[:2]
    tmp = np.einsum("ox,yxc->yoc", axis(w, tw), img)
    out = np.einsum("oy,yxc->oxc", axis(h, th), tmp)
    return (np.clip(np.floor(out + 0.5), 0, 255) / 255.0).astype(np.float32)


def bf16_to_f64(bits):
    """BF16 bit patterns (uint16) -> float64."""
    b = np.asarray(bits).astype(np.uint32) << 16
    return b.view(np.float32).astype(np.float64)


def vision_layer(W, i, h, pos):
    """One vision encoder layer in float64 (src/vision/encoder.ts:189-298
    dataflow: input norm, q / k / v with head norms and 2-D RoPE, attention
    with scale 1, o_proj, post-attention norm + residual, pre-feedforward
    norm, gelu-gate MLP, post-feedforward norm + residual)."""
    p = f"model.vision_tower.encoder.layers.{i}"
    heads, hd = 12, 64

    def lin(name, x):
        pre = f"{p}.{name}.linear"
        return qat_i8(x, W[f"{pre}.weight"], W[f"{pre}.weight_scale"], float(W[f"{pre}.input_activation_scale"]),
                      float(W[f"{pre}.output_activation_scale"]))

    nw = lambda n: bf16_to_f64(W[f"{p}.{n}.weight"])
    h = np.asarray(h, np.float64)
    a = rmsnorm(h, nw("input_layernorm"))
    q = rmsnorm(lin("self_attn.q_proj", a).reshape(-1, hd), nw("self_attn.q_norm")).reshape(-1, heads * hd)
    k = rmsnorm(lin("self_attn.k_proj", a).reshape(-1, hd), nw("self_attn.k_norm")).reshape(-1, heads * hd)
    v = rmsnorm(lin("self_attn.v_proj", a).reshape(-1, hd), np.ones(hd)).reshape(-1, heads * hd)
    q, k = rope(q, pos, heads, hd), rope(k, pos, heads, hd)
    o = lin("self_attn.o_proj", attention(q, k, v, heads, hd))
    h1 = h + rmsnorm(o, nw("post_attention_layernorm"))
    f = rmsnorm(h1, nw("pre_feedforward_layernorm"))
    m = gelu_gate(lin("mlp.gate_proj", f), lin("mlp.up_proj", f))
    return h1 + rmsnorm(lin("mlp.down_proj", m), nw("post_feedforward_layernorm"))


def vision_patch_embeddings(W, patches, pos):
    t = W["model.vision_tower.patch_embedder.position_embedding_table"]
    return patch_embed(patches, bf16_to_f64(W["model.vision_tower.patch_embedder.input_proj.weight"]), pos,
                       bf16_to_f64(t[0]), bf16_to_f64(t[1]))


def vision_embed(W, patches, pos, grid_h, grid_w, layer_count=16, hidden_out=None):
    """Vision tower in float64: patch embedding, layers, 3x3 pooler,
    embedder (src/vision/index.ts:69-112)."""
    h = vision_patch_embeddings(W, patches, pos)
    for i in range(layer_count):
        h = vision_layer(W, i, h, pos)
        if hidden_out is not None:
            hidden_out.append(h)
    return embedder(pooler(h, grid_h, grid_w), W["model.embed_vision.embedding_projection.weight"])
