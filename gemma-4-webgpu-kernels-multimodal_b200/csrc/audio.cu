// Audio tower runtime: weights, the packed-clip forward pass and the audio
// C ABI entry points.
//
// Dataflow of computeGemma4AudioEmbeddings (src/audio/index.ts:52-133) with
// the conformer layer of computeAudioEncoderLayerGpuOnly
// (src/audio/encoder.ts:761-1071): log-mel -> subsample convs -> input
// projection -> 12 x [FFN(1/2) -> attention -> light conv -> FFN(1/2) ->
// norm_out] -> output projection (+bias) -> embedder.  Clips are packed back
// to back (no padding rows), each row-coupled kernel honouring its clip's
// boundaries, so every clip gets exactly the reference's result for that
// clip alone.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <numeric>
#include <string>
#include <thread>
#include <vector>

#include "../../include/g4m.h"
#include "g4m_kernels.h"
#include "runtime_internal.h"
#include "safetensors.h"

namespace g4m {

namespace {

constexpr int D = 1024, FF = 4096, OUT = 1536, HD = 128, PLEN = 13;

const TensorInfo* need_f32(const SafeTensors& f, const std::string& name, std::vector<int64_t> shape,
                           const std::string& label, int* rc) {
  const TensorInfo* t = f.find(name);
  if (!t) {
    *rc = fail(G4M_E_IO, "Safetensors tensor not found: " + name);
    return nullptr;
  }
  if (t->dtype != "F32" || t->shape != shape) {  // assertF32Tensor, src/io/safetensors.ts:184-190
    *rc = fail(G4M_E_DTYPE, "Unexpected " + label + " tensor: " + shape_str(*t) + ".");
    return nullptr;
  }
  return t;
}

float* up(Device& d, const TensorInfo* t, const SafeTensors& f) {
  return upload_f32(d, (const float*)f.data(*t), (size_t)t->numel());
}

// audioRelativePositionEmbeddings (src/audio/kernels.ts:415-430), f32 stored.
std::vector<float> relpos(int plen, int dim) {
  std::vector<float> y((size_t)plen * dim);
  const int half = dim / 2;
  const double li = log(10000.0) / (double)std::max(half - 1, 1);
  for (int pi = 0; pi < plen; ++pi) {
    const double p = (double)(plen - 1 - pi);
    for (int k = 0; k < half; ++k) {
      const double s = p * exp((double)k * -li);
      y[(size_t)pi * dim + k] = (float)sin(s);
      y[(size_t)pi * dim + half + k] = (float)cos(s);
    }
  }
  return y;
}

double softplus_d(double v) {  // src/audio/kernels.ts:514-518
  if (v > 20) return v;
  if (v < -20) return exp(v);
  return log(1 + exp(v));
}

}  // namespace

int load_audio(Device& d, const SafeTensors& f) {
  auto lp = [](int i) { return "model.audio_tower.layers." + std::to_string(i); };
  int layers = 0;
  while (layers < 12 && f.find(lp(layers) + ".feed_forward1.ffw_layer_1.linear.weight")) ++layers;
  if (layers == 0) return G4M_OK;
  AudioWeights& aw = d.aw;
  aw.L.assign(layers, AudioLayer());
  int rc = G4M_OK;
  DevBuf staging, map_dev;
  const std::string sub = "model.audio_tower.subsample_conv_projection";
  // src/audio/index.ts:62-73
  const TensorInfo* c0 = need_f32(f, sub + ".layer0.conv.weight", {128, 1, 3, 3}, "audio embedding subsample layer0 conv", &rc);
  if (!c0) return rc;
  const TensorInfo* c0n = need_f32(f, sub + ".layer0.norm.weight", {128}, "audio embedding subsample layer0 norm", &rc);
  if (!c0n) return rc;
  const TensorInfo* c1 = need_f32(f, sub + ".layer1.conv.weight", {32, 128, 3, 3}, "audio embedding subsample layer1 conv", &rc);
  if (!c1) return rc;
  const TensorInfo* c1n = need_f32(f, sub + ".layer1.norm.weight", {32}, "audio embedding subsample layer1 norm", &rc);
  if (!c1n) return rc;
  const TensorInfo* inp = need_f32(f, sub + ".input_proj_linear.weight", {D, D}, "audio embedding subsample input projection", &rc);
  if (!inp) return rc;
  const TensorInfo* ow = need_f32(f, "model.audio_tower.output_proj.weight", {OUT, D}, "audio output projection weight", &rc);
  if (!ow) return rc;
  const TensorInfo* ob = need_f32(f, "model.audio_tower.output_proj.bias", {OUT}, "audio output projection bias", &rc);
  if (!ob) return rc;
  const TensorInfo* ew = need_f32(f, "model.embed_audio.embedding_projection.weight", {1536, OUT}, "audio embedder projection", &rc);
  if (!ew) return rc;
  aw.c0w = up(d, c0, f);
  aw.c0n = up(d, c0n, f);
  {  // layer-0 LayerNorm statistics from the taps: wbar_k = mean_c w[c][k], G_kl = (1 or 2) mean_c w[c][k] w[c][l]
    const float* w = (const float*)f.data(*c0);
    std::vector<double> stv(54, 0.0);
    for (int k = 0; k < 9; ++k) {
      for (int c = 0; c < 128; ++c) stv[k] += (double)w[c * 9 + k];
      stv[k] /= 128.0;
    }
    int q = 9;
    for (int k = 0; k < 9; ++k)
      for (int l = k; l < 9; ++l) {
        double g = 0.0;
        for (int c = 0; c < 128; ++c) g += (double)w[c * 9 + k] * (double)w[c * 9 + l];
        stv[q++] = (k == l ? 1.0 : 2.0) * g / 128.0;
      }
    aw.c0stat = (double*)dalloc(d, stv.size() * sizeof(double));
    if (!aw.c0stat || cudaMemcpy(aw.c0stat, stv.data(), stv.size() * sizeof(double), cudaMemcpyHostToDevice))
      return fail(G4M_E_CUDA, "audio subsample statistics upload failed");
  }
  aw.c1n = up(d, c1n, f);
  {  // layer-1 conv as tap-major rows [kt * 3 + kf][c_out][c_in], fp16 hi / lo (the conv GEMM's B operand)
    const float* w = (const float*)f.data(*c1);
    std::vector<float> t((size_t)9 * 32 * 128);
    for (int co = 0; co < 32; ++co)
      for (int ci = 0; ci < 128; ++ci)
        for (int k = 0; k < 9; ++k) t[((size_t)k * 32 + co) * 128 + ci] = w[((size_t)co * 128 + ci) * 9 + k];
    aw.c1_hi = (__half*)dalloc(d, t.size() * 2);
    aw.c1_lo = (__half*)dalloc(d, t.size() * 2);
    if (!aw.c1_hi || !aw.c1_lo || ensure(staging, t.size() * 4) != cudaSuccess ||
        cudaMemcpy(staging.p, t.data(), t.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        prep_w(staging.p, 2, 0, 9 * 32, 128, nullptr, aw.c1_hi, aw.c1_lo, 0) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess)
      return fail(G4M_E_CUDA, "audio subsample weight upload failed");
  }
  aw.out_b = up(d, ob, f);
  auto split_upload = [&](const TensorInfo* t, int rows, int cols, __half** hi, __half** lo) -> int {
    *hi = (__half*)dalloc(d, (size_t)rows * cols * 2);
    *lo = (__half*)dalloc(d, (size_t)rows * cols * 2);
    if (!*hi || !*lo || ensure(staging, f.bytes(*t)) != cudaSuccess ||
        cudaMemcpy(staging.p, f.data(*t), f.bytes(*t), cudaMemcpyHostToDevice) != cudaSuccess ||
        prep_w(staging.p, 2, 0, rows, cols, nullptr, *hi, *lo, 0) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess)
      return fail(G4M_E_CUDA, "audio projection upload failed");
    return G4M_OK;
  };
  if ((rc = split_upload(inp, D, D, &aw.in_hi, &aw.in_lo))) return rc;
  if ((rc = split_upload(ow, OUT, D, &aw.out_hi, &aw.out_lo))) return rc;
  if ((rc = split_upload(ew, 1536, OUT, &aw.emb_hi, &aw.emb_lo))) return rc;

  std::vector<float> rp = relpos(PLEN, D);
  for (int i = 0; i < layers; ++i) {
    AudioLayer& L = aw.L[i];
    const std::string p = lp(i);
    const char* blk[2] = {"feed_forward1", "feed_forward2"};
    for (int b = 0; b < 2; ++b) {
      L.w_ff1[b] = (__half*)dalloc(d, (size_t)FF * D * 2);
      L.w_ff2[b] = (__half*)dalloc(d, (size_t)D * FF * 2);
      if (!L.w_ff1[b] || !L.w_ff2[b]) return fail(G4M_E_CUDA, "audio weight allocation failed");
      std::vector<float> s1(FF), s2(D);
      std::vector<int> m1(FF), m2(D);
      std::iota(m1.begin(), m1.end(), 0);
      std::iota(m2.begin(), m2.end(), 0);
      if ((rc = load_qat(d, f, p + "." + blk[b] + ".ffw_layer_1.linear", "ffw_layer_1", FF, D, true, L.w_ff1[b], m1, s1,
                         L.sin_ff[b][0], L.sout_ff[b][0], staging, map_dev)))
        return rc;
      if ((rc = load_qat(d, f, p + "." + blk[b] + ".ffw_layer_2.linear", "ffw_layer_2", D, FF, true, L.w_ff2[b], m2, s2,
                         L.sin_ff[b][1], L.sout_ff[b][1], staging, map_dev)))
        return rc;
      L.s_ff1[b] = upload_f32(d, s1.data(), s1.size());
      L.s_ff2[b] = upload_f32(d, s2.data(), s2.size());
      const TensorInfo* a = need_f32(f, p + "." + blk[b] + ".pre_layer_norm.weight", {D},
                                     "audio layer " + std::to_string(i) + " " + blk[b] + " pre layernorm", &rc);
      if (!a) return rc;
      const TensorInfo* c = need_f32(f, p + "." + blk[b] + ".post_layer_norm.weight", {D},
                                     "audio layer " + std::to_string(i) + " " + blk[b] + " post layernorm", &rc);
      if (!c) return rc;
      L.n_ff_pre[b] = up(d, a, f);
      L.n_ff_post[b] = up(d, c, f);
    }
    // attention
    L.wqkv = (__half*)dalloc(d, (size_t)3 * D * D * 2);
    L.wpost = (__half*)dalloc(d, (size_t)D * D * 2);
    if (!L.wqkv || !L.wpost) return fail(G4M_E_CUDA, "audio weight allocation failed");
    std::vector<float> sqkv(3 * D), spost(D);
    const char* qkv[3] = {"q_proj", "k_proj", "v_proj"};
    for (int j = 0; j < 3; ++j) {
      std::vector<int> m(D);
      std::iota(m.begin(), m.end(), j * D);
      if ((rc = load_qat(d, f, p + ".self_attn." + qkv[j] + ".linear", qkv[j], D, D, true, L.wqkv, m, sqkv, L.sin_qkv[j],
                         L.sout_qkv[j], staging, map_dev)))
        return rc;
    }
    {
      std::vector<int> m(D);
      std::iota(m.begin(), m.end(), 0);
      if ((rc = load_qat(d, f, p + ".self_attn.post.linear", "post", D, D, true, L.wpost, m, spost, L.sin_post,
                         L.sout_post, staging, map_dev)))
        return rc;
    }
    L.sqkv = upload_f32(d, sqkv.data(), sqkv.size());
    L.spost = upload_f32(d, spost.data(), spost.size());
    const TensorInfo* pds = need_f32(f, p + ".self_attn.per_dim_scale", {HD},
                                     "audio layer " + std::to_string(i) + " attention per-dim scale", &rc);
    if (!pds) return rc;
    const TensorInfo* rkw = need_f32(f, p + ".self_attn.relative_k_proj.weight", {D, D},
                                     "audio layer " + std::to_string(i) + " relative key projection", &rc);
    if (!rkw) return rc;
    {
      // per-dim query multiplier: headDim^-0.5 / ln 2 * softplus(per_dim_scale)
      // (audioSelfAttentionScore, src/audio/kernels.ts:486-494)
      const float* pv = (const float*)f.data(*pds);
      std::vector<float> qm(HD);
      for (int k = 0; k < HD; ++k) qm[k] = (float)((pow((double)HD, -0.5) / log(2.0)) * softplus_d(pv[k]));
      L.pds = upload_f32(d, qm.data(), HD);
      // relative keys depend only on weights: projected once here
      // (runF32LinearRowsCpu of the position embeddings, src/audio/encoder.ts:1049-1056)
      const float* w = (const float*)f.data(*rkw);
      std::vector<float> rk((size_t)PLEN * D);
      for (int r = 0; r < PLEN; ++r)
        for (int o = 0; o < D; ++o) {
          double s = 0;
          const float* wr = w + (size_t)o * D;
          const float* xr = rp.data() + (size_t)r * D;
          for (int c = 0; c < D; ++c) s += (double)xr[c] * (double)wr[c];
          rk[(size_t)r * D + o] = (float)s;
        }
      L.relk = upload_f32(d, rk.data(), rk.size());
    }
    // light conv
    L.wstart = (__half*)dalloc(d, (size_t)2 * D * D * 2);
    L.wend = (__half*)dalloc(d, (size_t)D * D * 2);
    if (!L.wstart || !L.wend) return fail(G4M_E_CUDA, "audio weight allocation failed");
    std::vector<float> sst(2 * D), send(D);
    {
      // GLU halves (value rows [0, 1024), gate rows [1024, 2048)) interleaved in 128-row groups
      std::vector<int> m(2 * D);
      std::vector<int> a = map_interleave(D, 0), b = map_interleave(D, 1);
      for (int r = 0; r < D; ++r) {
        m[r] = a[r];
        m[D + r] = b[r];
      }
      float sout_start = 0;
      if ((rc = load_qat(d, f, p + ".lconv1d.linear_start.linear", "linear_start", 2 * D, D, true, L.wstart, m, sst,
                         L.sin_start, sout_start, staging, map_dev)))
        return rc;
      L.sout_start[0] = L.sout_start[1] = sout_start;
      std::vector<int> me(D);
      std::iota(me.begin(), me.end(), 0);
      if ((rc = load_qat(d, f, p + ".lconv1d.linear_end.linear", "linear_end", D, D, true, L.wend, me, send, L.sin_end,
                         L.sout_end, staging, map_dev)))
        return rc;
    }
    L.sstart = upload_f32(d, sst.data(), sst.size());
    L.send = upload_f32(d, send.data(), send.size());
    const std::string li = "audio layer " + std::to_string(i);
    const TensorInfo* t1 = need_f32(f, p + ".lconv1d.pre_layer_norm.weight", {D}, li + " lconv pre layernorm", &rc);
    if (!t1) return rc;
    const TensorInfo* t2 = need_f32(f, p + ".lconv1d.conv_norm.weight", {D}, li + " lconv norm", &rc);
    if (!t2) return rc;
    const TensorInfo* t3 = need_f32(f, p + ".lconv1d.depthwise_conv1d.weight", {D, 1, 5}, li + " lconv depthwise conv", &rc);
    if (!t3) return rc;
    const TensorInfo* t4 = need_f32(f, p + ".norm_pre_attn.weight", {D}, li + " pre-attention norm", &rc);
    if (!t4) return rc;
    const TensorInfo* t5 = need_f32(f, p + ".norm_post_attn.weight", {D}, li + " post-attention norm", &rc);
    if (!t5) return rc;
    const TensorInfo* t6 = need_f32(f, p + ".norm_out.weight", {D}, li + " output norm", &rc);
    if (!t6) return rc;
    L.n_lpre = up(d, t1, f);
    L.n_conv = up(d, t2, f);
    {  // depthwise weights transposed to [5][1024] (four channels per vector load)
      const float* w = (const float*)f.data(*t3);
      std::vector<float> wt(5 * D);
      for (int c = 0; c < D; ++c)
        for (int k = 0; k < 5; ++k) wt[k * D + c] = w[c * 5 + k];
      L.dw = upload_f32(d, wt.data(), wt.size());
    }
    L.n_pre_attn = up(d, t4, f);
    L.n_post_attn = up(d, t5, f);
    L.n_out = up(d, t6, f);
    if (!L.s_ff1[0] || !L.sqkv || !L.spost || !L.pds || !L.relk || !L.sstart || !L.send || !L.n_lpre || !L.n_conv ||
        !L.dw || !L.n_pre_attn || !L.n_post_attn || !L.n_out)
      return fail(G4M_E_CUDA, "audio weight upload failed");
  }
  // front-end tables: periodic Hann window, FFT twiddles
  {
    std::vector<float> win(320);
    for (int i = 0; i < 320; ++i) win[i] = (float)(0.5 - 0.5 * cos((2 * M_PI * i) / 320));  // periodicHannWindow
    aw.window = upload_f32(d, win.data(), win.size());
    std::vector<double> tw(512);
    for (int k = 0; k < 256; ++k) {
      tw[2 * k] = cos(-2 * M_PI * k / 512);
      tw[2 * k + 1] = sin(-2 * M_PI * k / 512);
    }
    aw.twiddle = (double2*)dalloc(d, tw.size() * sizeof(double));
    if (!aw.twiddle || cudaMemcpy(aw.twiddle, tw.data(), tw.size() * sizeof(double), cudaMemcpyHostToDevice))
      return fail(G4M_E_CUDA, "twiddle upload failed");
  }
  release(staging);
  release(map_dev);
  aw.layers = layers;
  return G4M_OK;
}

// createHtkMelFilterBank (src/preprocess/audio.ts:128-157) for a sampling rate.
static int ensure_mel(Device& d, int sr) {
  if (d.aw.mel && d.aw_mel_sr == sr) return G4M_OK;
  const int bins = 257, nmel = 128;
  auto hz2mel = [](double f) { return 2595 * log10(1 + f / 700); };
  auto mel2hz = [](double m) { return 700 * (pow(10, m / 2595) - 1); };
  const double mmin = hz2mel(0), mmax = hz2mel(8000);
  std::vector<double> ff(nmel + 2);
  for (int i = 0; i < nmel + 2; ++i) ff[i] = mel2hz(mmin + ((mmax - mmin) * i) / (nmel + 1));
  std::vector<float> filt((size_t)bins * nmel);
  const double bw = (double)sr / ((bins - 1) * 2.0);
  for (int b = 0; b < bins; ++b) {
    const double fr = bw * b;
    for (int m = 0; m < nmel; ++m) {
      const double l = ff[m], c = ff[m + 1], r = ff[m + 2];
      const double u = c == l ? 0 : (fr - l) / (c - l);
      const double dn = r == c ? 0 : (r - fr) / (r - c);
      filt[(size_t)b * nmel + m] = (float)std::max(0.0, std::min(u, dn));
    }
  }
  // non-zero bin range of every channel: the device sums only those terms, in
  // bin order, which leaves each double sum bit-identical to the dense one
  std::vector<int> rng(2 * nmel);
  for (int m = 0; m < nmel; ++m) {
    int lo = bins, hi = -1;
    for (int b = 0; b < bins; ++b)
      if (filt[(size_t)b * nmel + m] != 0.0f) {
        lo = std::min(lo, b);
        hi = b;
      }
    rng[2 * m] = lo;
    rng[2 * m + 1] = hi;  // empty channel: lo > hi
  }
  if (!d.aw.mel) d.aw.mel = (float*)dalloc(d, filt.size() * 4);
  if (!d.aw.mel_rng) d.aw.mel_rng = (int*)dalloc(d, rng.size() * 4);
  if (!d.aw.mel || !d.aw.mel_rng ||
      cudaMemcpy(d.aw.mel, filt.data(), filt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(d.aw.mel_rng, rng.data(), rng.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(G4M_E_CUDA, "mel filter upload failed");
  d.aw_mel_sr = sr;
  return G4M_OK;
}

// Frames / subsample rows of an unpadded clip of n samples
// (src/preprocess/audio.ts:54-57, audioSubsampleOutputLength).
struct ClipShape {
  long samples = 0;
  int frames = 0, t0 = 0, t1 = 0;
};

ClipShape clip_shape(long n) {
  ClipShape s;
  s.samples = n;
  const long wl = 160 + n;
  s.frames = wl >= 321 ? (int)((wl - 321) / 160 + 1) : 0;
  if (s.frames > 0) {
    s.t0 = (s.frames - 1) / 2 + 1;
    s.t1 = (s.t0 - 1) / 2 + 1;
  }
  return s;
}

#define G4M_LAUNCH_A(x)                                                                          \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) return fail(G4M_E_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// q / k / v share one operand: all three use static input quantisation or
// none of them; every other linear is independent.
static int audio_check_quant(const AudioWeights& aw, int layers) {
  for (int i = 0; i < layers; ++i)
    if (quant_group(aw.L[i].sin_qkv, 3) < 0)
      return fail(G4M_E_UNSUPPORTED, "audio layer " + std::to_string(i) +
                                         ": q/k/v projections mix zero and non-zero input_activation_scale; they "
                                         "share one operand");
  return G4M_OK;
}

static GemmArgs aargs(Device& d, long M, int N, int K) {
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.M = (int)M;
  a.N = N;
  a.K = K;
  a.row_scale = 1.0f;
  a.row_scale_b = 1.0f;
  a.row_scale_c = 1.0f;
  a.eps = 1e-6f;
  a.err = d.err;
  return a;
}

// Next-operand fields of a row pass whose consumers have input scales s[0..n)
// (integer code planes a_hi, a_lo, a_c when they are non-zero).
static void next_scales(RowArgs& r, const float* s, int n, __half* a_c) {
  r.s_in_next = s ? s[0] : 0.0f;
  r.s_in_b = (s && n > 1) ? s[1] : 0.0f;
  r.s_in_c = (s && n > 2) ? s[2] : 0.0f;
  r.a_c = (s && n > 2 && s[0] != 0.0f) ? a_c : nullptr;
}

// Row metadata of a packed batch: clip of every row, first row and row count
// of every clip, attention runs (clip, first of up to kAudioAttnRun blocks
// of 12 rows).
static int audio_setup_rows(Device& d, const std::vector<int>& rows, long* M_out, int* nruns, cudaStream_t st,
                            HostKeep* keep = nullptr) {
  const int n = (int)rows.size();
  std::vector<int> row0(n);
  std::vector<int> bclip, bidx;
  long M = 0;
  for (int i = 0; i < n; ++i) {
    row0[i] = (int)M;
    M += rows[i];
    for (int b = 0; b < (rows[i] + 11) / 12; b += kAudioAttnRun) {
      bclip.push_back(i);
      bidx.push_back(b);
    }
  }
  std::vector<int> row_clip(M);
  for (int i = 0; i < n; ++i)
    for (int r = 0; r < rows[i]; ++r) row_clip[row0[i] + r] = i;
  AudioBuffers& b = d.ab;
  if (ensure(b.clip_row0, n * 4) || ensure(b.clip_rows, n * 4) || ensure(b.row_clip, M * 4 + 4) ||
      ensure(b.t1_off, bclip.size() * 4 + 4) || ensure(b.t1_len, bidx.size() * 4 + 4) || ensure(b.h, M * D * 4) ||
      ensure(b.y, M * D * 4) || ensure(b.qkv, M * 3 * D * 4) || ensure(b.g, M * D * 4) || ensure(b.a_hi, M * D * 2) ||
      ensure(b.a_lo, M * D * 2) || ensure(b.f_hi, M * FF * 2) || ensure(b.f_lo, M * FF * 2) ||
      ensure(b.proj, M * OUT * 4) || ensure(b.e_hi, M * OUT * 2) || ensure(b.e_lo, M * OUT * 2))
    return fail(G4M_E_CUDA, "audio activation allocation failed (" + std::to_string(M) + " rows)");
  bool codes3 = false;  // a third code plane for layers with quantised q / k / v
  for (int i = 0; i < d.aw.layers; ++i) codes3 = codes3 || d.aw.L[i].sin_qkv[0] != 0.0f;
  if (codes3 && ensure(b.a_c, M * D * 2))
    return fail(G4M_E_CUDA, "audio activation allocation failed (" + std::to_string(M) + " rows)");
  G4M_LAUNCH_A(upload_meta(b.clip_row0.p, row0.data(), n * 4, st, keep));
  G4M_LAUNCH_A(upload_meta(b.clip_rows.p, rows.data(), n * 4, st, keep));
  G4M_LAUNCH_A(upload_meta(b.row_clip.p, row_clip.data(), M * 4, st, keep));
  G4M_LAUNCH_A(upload_meta(b.t1_off.p, bclip.data(), bclip.size() * 4, st, keep));
  G4M_LAUNCH_A(upload_meta(b.t1_len.p, bidx.data(), bidx.size() * 4, st, keep));
  if (!keep) G4M_LAUNCH_A(cudaStreamSynchronize(st));  // the host vectors above are the copy sources
  *M_out = M;
  *nruns = (int)bclip.size();
  return G4M_OK;
}

// Conformer layers [first, first+count) on the packed rows: on entry ab.h
// holds the residual stream and ab.a_* the feed_forward1 pre-norm operand of
// layer `first`; on exit ab.h holds the output of the last layer (after
// norm_out) and, if another layer follows, ab.a_* its first operand.
static int audio_layer_range(g4m_ctx* ctx, Device& d, long M, int nruns, int first, int count, bool next_operand,
                             cudaStream_t st) {
  AudioWeights& aw = d.aw;
  AudioBuffers& b = d.ab;
  const int* drow0 = (const int*)b.clip_row0.p;
  const int* drows = (const int*)b.clip_rows.p;
  const int* drc = (const int*)b.row_clip.p;
  __half *ah = (__half*)b.a_hi.p, *al = (__half*)b.a_lo.p;
  float *h = (float*)b.h.p, *y = (float*)b.y.p;
  RowArgs r;
  memset(&r, 0, sizeof(r));
  r.rows = M;
  r.d = D;
  r.eps = 1e-6f;
  r.a_hi = ah;
  r.a_lo = al;
  r.lda = D;
  GemmArgs a;
  GemmOperands op;
  int rc = G4M_OK;
  __half* ac = (__half*)b.a_c.p;
  // Feed-forward block `blk`; its final row pass also produces the operand
  // of the next linear (norm w_next, input scales s_next[0..n_next)).
  auto ffn = [&](const AudioLayer& L, int blk, const float* w_next, const float* s_next, int n_next,
                 const float* w_out) -> int {
    const float s1 = L.sin_ff[blk][0], s2 = L.sin_ff[blk][1];
    GemmArgs g = aargs(d, M, FF, D);
    g.col_scale = L.s_ff1[blk];
    g.s_out = L.sout_ff[blk][0];
    g.out_hi = (__half*)b.f_hi.p;
    g.out_lo = (__half*)b.f_lo.p;
    g.ldh = FF;
    g.s_code = s2;  // ffw_layer_2's input scale: store codes
    if (s1 != 0.0f) g.row_scale = s1;
    GemmOperands o{ah, al, L.w_ff1[blk], nullptr};
    G4M_RUN("gemm_ffw1", gemm_launch(256, s1 != 0.0f ? 1 : 2, EPI_SILU, o, g, st));
    g = aargs(d, M, D, FF);
    g.col_scale = L.s_ff2[blk];
    g.s_out = L.sout_ff[blk][1];
    g.out_f32 = y;
    g.ldo = D;
    if (s2 != 0.0f) g.row_scale = s2;
    o = GemmOperands{(const __half*)b.f_hi.p, (const __half*)b.f_lo.p, L.w_ff2[blk], nullptr};
    G4M_RUN("gemm_ffw2", gemm_launch(256, s2 != 0.0f ? 1 : 2, EPI_F32, o, g, st));
    RowArgs q = r;
    q.h_in = h;
    q.h_out = h;
    q.y = y;
    q.w_post = L.n_ff_post[blk];
    q.res_scale = 0.5f;  // AUDIO_FEED_FORWARD_RESIDUAL_WEIGHT, src/model.ts:91
    q.w_out = w_out;
    q.w_next = w_next;
    next_scales(q, s_next, n_next, ac);
    G4M_RUN("rows", fused_rows(q, st));
    return G4M_OK;
  };
  for (int i = first; i < first + count; ++i) {
    if (ctx->cancel.load()) return fail(G4M_E_CANCELLED, "Aborted");
    const AudioLayer& L = aw.L[i];
    if ((rc = ffn(L, 0, L.n_pre_attn, L.sin_qkv, 3, nullptr))) return rc;
    // self attention (src/audio/encoder.ts:1011-1071)
    const bool qkv_codes = L.sin_qkv[0] != 0.0f;  // all-zero or all-non-zero (audio_check_quant)
    a = aargs(d, M, 3 * D, D);
    a.col_scale = L.sqkv;
    if (qkv_codes) {
      a.row_scale = L.sin_qkv[0];
      a.row_scale_b = L.sin_qkv[1];
      a.row_scale_c = L.sin_qkv[2];
    }
    a.proj_width = D;
    a.s_out = L.sout_qkv[0];
    a.s_out_b = L.sout_qkv[1];
    a.s_out_c = L.sout_qkv[2];
    a.out_f32 = (float*)b.qkv.p;
    a.ldo = 3 * D;
    op = GemmOperands{ah, al, L.wqkv, nullptr, ac};
    if (qkv_codes) G4M_RUN("gemm_qkv", gemm_launch(256, 1, EPI_F32, op, a, st, 0, 1));
    else G4M_RUN("gemm_qkv", gemm_launch(256, 2, EPI_F32, op, a, st));
    G4M_RUN("attention", audio_attention_blocks((const float*)b.qkv.p, L.relk, L.pds, (const int*)b.t1_off.p,
                                                (const int*)b.t1_len.p, nruns, drow0, drows,
                                                (float)(log(1.0 + exp(1.0)) / log(2.0)), 50.0f, ah, al, L.sin_post,
                                                st));
    a = aargs(d, M, D, D);
    a.col_scale = L.spost;
    a.s_out = L.sout_post;
    a.out_f32 = y;
    a.ldo = D;
    if (L.sin_post != 0.0f) a.row_scale = L.sin_post;
    op = GemmOperands{ah, al, L.wpost, nullptr};
    G4M_RUN("gemm_post", gemm_launch(256, L.sin_post != 0.0f ? 1 : 2, EPI_F32, op, a, st));
    RowArgs q = r;
    q.y = y;
    q.w_post = L.n_post_attn;
    q.res_scale = 1.0f;
    q.h_in = h;
    q.h_out = h;
    q.w_next = L.n_lpre;
    next_scales(q, &L.sin_start, 1, nullptr);
    G4M_RUN("rows", fused_rows(q, st));
    // light conv (src/audio/encoder.ts:923-1009)
    a = aargs(d, M, 2 * D, D);
    a.col_scale = L.sstart;
    a.s_out = L.sout_start[0];
    a.s_out_b = L.sout_start[1];
    a.out_f32 = (float*)b.g.p;
    a.ldo = D;
    if (L.sin_start != 0.0f) a.row_scale = a.row_scale_b = L.sin_start;
    op = GemmOperands{ah, al, L.wstart, nullptr};
    G4M_RUN("gemm_lconv_start", gemm_launch(256, L.sin_start != 0.0f ? 1 : 2, EPI_GLU, op, a, st));
    G4M_RUN("lconv",
            audio_lconv_rows((const float*)b.g.p, L.dw, L.n_conv, drc, drow0, M, 1e-6f, ah, al, L.sin_end,
                             d.err, st));
    a = aargs(d, M, D, D);
    a.col_scale = L.send;
    a.s_out = L.sout_end;
    a.out_f32 = y;
    a.ldo = D;
    if (L.sin_end != 0.0f) a.row_scale = L.sin_end;
    op = GemmOperands{ah, al, L.wend, nullptr};
    G4M_RUN("gemm_lconv_end", gemm_launch(256, L.sin_end != 0.0f ? 1 : 2, EPI_F32, op, a, st));
    q = r;
    q.y = y;
    q.w_post = nullptr;
    q.res_scale = 1.0f;
    q.h_in = h;
    q.h_out = h;
    q.w_next = L.n_ff_pre[1];
    next_scales(q, &L.sin_ff[1][0], 1, nullptr);
    G4M_RUN("rows", fused_rows(q, st));
    const bool more = i + 1 < first + count || (next_operand && i + 1 < aw.layers);
    if ((rc = ffn(L, 1, more ? aw.L[i + 1].n_ff_pre[0] : nullptr, more ? &aw.L[i + 1].sin_ff[0][0] : nullptr, 1,
                  L.n_out)))
      return rc;
  }
  return G4M_OK;
}

// Packed forward for clips whose samples sit in samples_dev at offsets
// soff.  shapes[i].t1 rows per clip.
int audio_forward(g4m_ctx* ctx, Device& d, const std::vector<ClipShape>& shapes, const float* samples_dev,
                  const std::vector<long>& soff, int sr, int layers, float* out_dev, cudaStream_t st,
                  HostKeep* keep = nullptr) {
  (void)cudaGetLastError();  // a failed earlier call must not leak into this one
  AudioWeights& aw = d.aw;
  if (aw.layers == 0) return fail(G4M_E_NOT_LOADED, "audio tower weights are not loaded");
  if (layers < 1 || layers > 12)
    return fail(G4M_E_ARG, "Audio encoder layer count must be 1-12, got " + std::to_string(layers) + ".");
  if (layers > aw.layers)
    return fail(G4M_E_NOT_LOADED, "checkpoint holds " + std::to_string(aw.layers) + " audio layers, " +
                                      std::to_string(layers) + " requested");
  int rc = audio_check_quant(aw, layers);
  if (rc) return rc;
  rc = ensure_mel(d, sr);
  if (rc) return rc;
  const int n = (int)shapes.size();
  if (n == 0) return G4M_OK;
  std::vector<int> foff(n), fcnt(n), rows(n), t0off(n);
  std::vector<long> slen(n);
  long FR = 0, T0S = 0;
  int max_t0 = 0;
  for (int i = 0; i < n; ++i) {
    foff[i] = (int)FR;
    fcnt[i] = shapes[i].frames;
    rows[i] = shapes[i].t1;
    slen[i] = shapes[i].samples;
    FR += shapes[i].frames;
    const int t0 = (shapes[i].frames - 1) / 2 + 1;  // layer-0 rows (src/audio/kernels.ts:1242-1244)
    t0off[i] = (int)T0S + 1;                        // a zero row before every clip
    T0S += t0 + 1;
    max_t0 = std::max(max_t0, t0);
  }
  T0S += 1;            // and one after the last
  T0S += T0S & 1;      // an even row count (the conv's TMA view pairs rows)
  long M = 0;
  int nruns = 0;
  if ((rc = audio_setup_rows(d, rows, &M, &nruns, st, keep))) return rc;
  AudioBuffers& b = d.ab;
  if (ensure(b.sample_off, n * 8) || ensure(b.sample_len, n * 8) || ensure(b.frame_off, n * 4) ||
      ensure(b.frames, n * 4) || ensure(b.feats, FR * 128 * 4) || ensure(b.t0_off, n * 4) ||
      ensure(b.l0, (size_t)T0S * 64 * 128 * 2 * 2))
    return fail(G4M_E_CUDA, "audio front-end allocation failed");
  G4M_LAUNCH_A(upload_meta(b.sample_off.p, soff.data(), n * 8, st, keep));
  G4M_LAUNCH_A(upload_meta(b.sample_len.p, slen.data(), n * 8, st, keep));
  G4M_LAUNCH_A(upload_meta(b.frame_off.p, foff.data(), n * 4, st, keep));
  G4M_LAUNCH_A(upload_meta(b.frames.p, fcnt.data(), n * 4, st, keep));
  G4M_LAUNCH_A(upload_meta(b.t0_off.p, t0off.data(), n * 4, st, keep));
  if (!keep) G4M_LAUNCH_A(cudaStreamSynchronize(st));
  const int* dfoff = (const int*)b.frame_off.p;
  const int* dfcnt = (const int*)b.frames.p;
  __half *ah = (__half*)b.a_hi.p, *al = (__half*)b.a_lo.p;
  float* h = (float*)b.h.p;
  // front end (preprocessGemma4AudioSamples + runAudioSubsampleProjectionCpu)
  G4M_RUN("logmel", audio_logmel(samples_dev, (const long*)b.sample_off.p, (const long*)b.sample_len.p, dfoff, dfcnt, n,
                                 (int)FR, aw.window, aw.mel, aw.mel_rng, aw.twiddle, (float*)b.feats.p, st));
  const int max_rows = *std::max_element(rows.begin(), rows.end());
  __half* l0h = (__half*)b.l0.p;
  __half* l0l = l0h + (size_t)T0S * 64 * 128;
  G4M_RUN("subsample", audio_subsample_tc((const float*)b.feats.p, dfoff, dfcnt, (const int*)b.t0_off.p, T0S,
                                          (const int*)b.clip_row0.p, (const int*)b.clip_rows.p, n, max_t0, max_rows,
                                          aw.c0w, aw.c0stat, aw.c0n, aw.c1_hi, aw.c1_lo, aw.c1n, 1e-6f, l0h, l0l, ah, al, d.err,
                                          st));
  GemmArgs a = aargs(d, M, D, D);
  a.out_f32 = h;
  a.ldo = D;
  GemmOperands op{ah, al, aw.in_hi, aw.in_lo};
  G4M_RUN("gemm_in_proj", gemm_launch(128, 3, EPI_F32, op, a, st));
  if (ctx->debug) {  // encoder input, for front-end parity checks
    if (ensure(b.h0, M * D * 4)) return fail(G4M_E_CUDA, "debug buffer allocation failed");
    G4M_LAUNCH_A(cudaMemcpyAsync(b.h0.p, h, M * D * 4, cudaMemcpyDeviceToDevice, st));
  }
  RowArgs r;
  memset(&r, 0, sizeof(r));
  r.rows = M;
  r.d = D;
  r.eps = 1e-6f;
  r.h_in = h;
  r.w_next = aw.L[0].n_ff_pre[0];
  next_scales(r, &aw.L[0].sin_ff[0][0], 1, nullptr);
  r.a_hi = ah;
  r.a_lo = al;
  r.lda = D;
  G4M_RUN("rows", fused_rows(r, st));
  if ((rc = audio_layer_range(ctx, d, M, nruns, 0, layers, false, st))) return rc;
  // output projection + bias (src/audio/kernels.ts:380-413), then the embedder
  G4M_RUN("prep_a", prep_a(h, M, D, 0.0f, nullptr, ah, al, st));
  a = aargs(d, M, OUT, D);
  a.bias = aw.out_b;
  a.out_f32 = (float*)b.proj.p;
  a.ldo = OUT;
  op = GemmOperands{ah, al, aw.out_hi, aw.out_lo};
  G4M_RUN("gemm_out_proj", gemm_launch(128, 3, EPI_F32, op, a, st));
  G4M_RUN("embed_operand", row_inv_rms_operand((const float*)b.proj.p, M, OUT, 1e-6f, (__half*)b.e_hi.p,
                                               (__half*)b.e_lo.p, st));
  a = aargs(d, M, 1536, OUT);
  a.out_f32 = out_dev;
  a.ldo = 1536;
  op = GemmOperands{(const __half*)b.e_hi.p, (const __half*)b.e_lo.p, aw.emb_hi, aw.emb_lo};
  G4M_RUN("gemm_embed", gemm_launch(128, 3, EPI_F32, op, a, st));
  d.last_audio_rows = M;
  return G4M_OK;
}

// Run audio layers [first, first+count) on host hidden states h (packed rows,
// rows_per_clip[i] rows for clip i) in place.
int audio_layers_host(g4m_ctx* ctx, Device& d, const std::vector<int>& rows, int first, int count, float* h) {
  AudioWeights& aw = d.aw;
  if (aw.layers == 0) return fail(G4M_E_NOT_LOADED, "audio tower weights are not loaded");
  if (first < 0 || count < 1 || first + count > aw.layers) return fail(G4M_E_ARG, "layer range outside the checkpoint");
  int rc = audio_check_quant(aw, first + count);
  if (rc) return rc;
  cudaStream_t st = d.st;
  long M = 0;
  int nruns = 0;
  if ((rc = audio_setup_rows(d, rows, &M, &nruns, st))) return rc;
  AudioBuffers& b = d.ab;
  G4M_LAUNCH_A(cudaMemcpyAsync(b.h.p, h, M * D * 4, cudaMemcpyHostToDevice, st));
  RowArgs r;
  memset(&r, 0, sizeof(r));
  r.rows = M;
  r.d = D;
  r.eps = 1e-6f;
  r.h_in = (const float*)b.h.p;
  r.w_next = aw.L[first].n_ff_pre[0];
  next_scales(r, &aw.L[first].sin_ff[0][0], 1, nullptr);
  r.a_hi = (__half*)b.a_hi.p;
  r.a_lo = (__half*)b.a_lo.p;
  r.lda = D;
  G4M_RUN("rows", fused_rows(r, st));
  if ((rc = audio_layer_range(ctx, d, M, nruns, first, count, false, st))) return rc;
  G4M_LAUNCH_A(cudaMemcpyAsync(h, b.h.p, M * D * 4, cudaMemcpyDeviceToHost, st));
  d.last_audio_rows = M;
  return finish(d, st);
}

}  // namespace g4m

using namespace g4m;

extern "C" {

int g4m_audio_embed_device(g4m_ctx* ctx, int di, int n, const float* samples_dev, const int64_t* offsets,
                           const int64_t* lengths, int sampling_rate, int layer_count, int64_t max_samples,
                           float* out_dev, int* rows_out, void* stream) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || n < 0 || (n > 0 && (!samples_dev || !offsets || !lengths || !out_dev)))
    return fail(G4M_E_ARG, "bad argument");
  if (sampling_rate <= 0) return fail(G4M_E_ARG, "sampling rate must be positive");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  const long cap = max_samples > 0 ? (long)max_samples : 480000;
  std::vector<ClipShape> shapes(n);
  std::vector<long> soff(n);
  for (int i = 0; i < n; ++i) {
    shapes[i] = clip_shape(std::min<long>((long)lengths[i], cap));
    soff[i] = (long)offsets[i];
    if (shapes[i].frames == 0) return fail(G4M_E_SHAPE, "Audio preprocessing produced no frames.");
    if (rows_out) rows_out[i] = shapes[i].t1;
  }
  cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamLegacy;
  return audio_forward(ctx, d, shapes, samples_dev, soff, sampling_rate, layer_count, out_dev, st);
}

}  // extern "C"

// Chunks [first, last) of one device's clips (longest first) for the
// pipelined batch call.  Only the first chunk's upload and the last chunk's
// download are not hidden behind compute, so the head and the tail hold at
// most kEdgeRows encoder rows each (37 M-tiles: a 1024-column GEMM over them
// is one 148-tile wave), and the middle chunk takes all the rest, keeping the
// GEMMs' tile waves full.  Batches under three edges' worth of rows run as
// one chunk.
static std::vector<std::pair<int, int>> audio_batch_chunks(const std::vector<ClipShape>& sh) {
  constexpr long kEdgeRows = 37 * 128;
  const int m = (int)sh.size();
  long total = 0;
  for (const ClipShape& c : sh) total += c.t1;
  if (m < 3 || total < 3 * kEdgeRows) return {{0, m}};
  int h = 0;
  long rows = 0;
  while (h < m - 2 && (h == 0 || rows + sh[h].t1 <= kEdgeRows)) rows += sh[h++].t1;
  int t = m;
  rows = 0;
  while (t > h + 1 && (t == m || rows + sh[t - 1].t1 <= kEdgeRows)) rows += sh[--t].t1;
  return {{0, h}, {h, t}, {t, m}};
}

extern "C" {

int g4m_audio_embed_batch(g4m_ctx* ctx, int n, const float* const* samples, const int64_t* lengths, int sampling_rate,
                          int layer_count, int64_t max_samples, float* const* out, int* rows_out, int* status) {
  if (!ctx || n < 0 || (n > 0 && (!samples || !lengths || !out))) return fail(G4M_E_ARG, "bad argument");
  if (sampling_rate <= 0) return fail(G4M_E_ARG, "sampling rate must be positive");
  const long cap = max_samples > 0 ? (long)max_samples : 480000;
  std::vector<ClipShape> shapes(n);
  std::vector<int> ok;
  for (int i = 0; i < n; ++i) {
    shapes[i] = clip_shape(std::min<long>((long)lengths[i], cap));
    if (rows_out) rows_out[i] = 0;
    if (shapes[i].frames == 0) {
      if (status) status[i] = G4M_E_SHAPE;
    } else {
      if (status) status[i] = G4M_OK;
      ok.push_back(i);
    }
  }
  // length-balanced assignment: longest first onto the least-loaded device
  const int G = (int)ctx->devs.size();
  std::vector<std::vector<int>> part(G);
  std::vector<long> load(G, 0);
  std::vector<int> order = ok;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return shapes[a].t1 > shapes[b].t1; });
  for (int i : order) {
    const int g = (int)(std::min_element(load.begin(), load.end()) - load.begin());
    part[g].push_back(i);
    load[g] += shapes[i].t1;
  }
  std::vector<int> rcs(G, G4M_OK);
  std::vector<std::string> msgs(G);
  auto work = [&](int g) {
    if (part[g].empty()) return;
    Device& d = *ctx->devs[g];
    std::lock_guard<std::mutex> lk(d.mu);
    cudaSetDevice(d.id);
    std::vector<ClipShape> sh;
    std::vector<long> soff;
    long total = 0, rows = 0;
    for (int i : part[g]) {
      sh.push_back(shapes[i]);
      soff.push_back(total);
      total += shapes[i].samples;
      rows += shapes[i].t1;
    }
    int r = G4M_OK;
    if (ensure(d.ab.samples, std::max<long>(total, 1) * 4) || ensure(d.io_out, std::max<long>(rows, 1) * 1536 * 4))
      r = fail(G4M_E_CUDA, "audio io allocation failed");
    // a short head and tail chunk and one middle chunk (audio_batch_chunks):
    // uploads queue on the copy stream, each chunk's forward waits for its
    // upload, each download for its forward
    const int m = (int)part[g].size();
    const auto chunks = audio_batch_chunks(sh);
    std::vector<cudaEvent_t> up(chunks.size()), done(chunks.size());
    for (size_t c = 0; c < chunks.size(); ++c) {
      cudaEventCreateWithFlags(&up[c], cudaEventDisableTiming);
      cudaEventCreateWithFlags(&done[c], cudaEventDisableTiming);
    }
    for (size_t c = 0; !r && c < chunks.size(); ++c) {
      for (int k = chunks[c].first; !r && k < chunks[c].second; ++k)
        if (cudaMemcpyAsync((float*)d.ab.samples.p + soff[k], samples[part[g][k]], sh[k].samples * 4,
                            cudaMemcpyHostToDevice, d.cst))
          r = fail(G4M_E_CUDA, "sample upload failed");
      if (!r && cudaEventRecord(up[c], d.cst)) r = fail(G4M_E_CUDA, "event record failed");
    }
    HostKeep keep;  // chunk metadata stays alive until the final synchronize
    long ro = 0;
    for (size_t c = 0; !r && c < chunks.size(); ++c) {
      const int k0 = chunks[c].first, k1 = chunks[c].second;
      std::vector<ClipShape> csh(sh.begin() + k0, sh.begin() + k1);
      std::vector<long> coff;
      for (int k = k0; k < k1; ++k) coff.push_back(soff[k] - soff[k0]);
      if (cudaStreamWaitEvent(d.st, up[c], 0)) r = fail(G4M_E_CUDA, "stream wait failed");
      if (!r)
        r = audio_forward(ctx, d, csh, (const float*)d.ab.samples.p + soff[k0], coff, sampling_rate, layer_count,
                          (float*)d.io_out.p + ro * 1536, d.st, &keep);
      if (!r && (cudaEventRecord(done[c], d.st) || cudaStreamWaitEvent(d.cst, done[c], 0)))
        r = fail(G4M_E_CUDA, "event record failed");
      for (int k = k0; !r && k < k1; ++k) {
        if (cudaMemcpyAsync(out[part[g][k]], (float*)d.io_out.p + ro * 1536, (size_t)sh[k].t1 * 1536 * 4,
                            cudaMemcpyDeviceToHost, d.cst))
          r = fail(G4M_E_CUDA, "embedding download failed");
        ro += sh[k].t1;
      }
    }
    const int rs = finish(d, d.st);
    const cudaError_t ce = cudaStreamSynchronize(d.cst);
    for (size_t c = 0; c < chunks.size(); ++c) {
      cudaEventDestroy(up[c]);
      cudaEventDestroy(done[c]);
    }
    if (!r) r = rs;
    if (!r && ce != cudaSuccess) r = fail(G4M_E_CUDA, std::string("copy stream: ") + cudaGetErrorString(ce));
    rcs[g] = r;
    if (r) msgs[g] = tl_err;
  };
  if (G == 1) work(0);
  else {
    std::vector<std::thread> th;
    for (int g = 0; g < G; ++g) th.emplace_back(work, g);
    for (auto& t : th) t.join();
  }
  int first = G4M_OK;
  for (int g = 0; g < G; ++g) {
    for (int i : part[g]) {
      if (rows_out) rows_out[i] = rcs[g] ? 0 : shapes[i].t1;
      if (status) status[i] = rcs[g];
    }
    if (rcs[g] && !first) {
      first = rcs[g];
      tl_err = msgs[g];
    }
  }
  if (!first && ok.size() != (size_t)n) first = fail(G4M_E_SHAPE, "Audio preprocessing produced no frames.");
  return first;
}

int g4m_audio_layers(g4m_ctx* ctx, int di, int n, const int* rows_per_clip, int first, int count, float* h) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || n <= 0 || !rows_per_clip || !h)
    return fail(G4M_E_ARG, "bad argument");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  std::vector<int> rows(rows_per_clip, rows_per_clip + n);
  for (int v : rows)
    if (v <= 0) return fail(G4M_E_ARG, "every clip needs at least one row");
  return audio_layers_host(ctx, d, rows, first, count, h);
}

int g4m_audio_debug_hidden(g4m_ctx* ctx, int di, int which, float* host, size_t count) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || !host) return fail(G4M_E_ARG, "bad argument");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  if (which < 0 || which > 2) return fail(G4M_E_ARG, "which must be 0, 1 or 2");
  const size_t need_n = (size_t)d.last_audio_rows * (which == 2 ? 3 * 1024 : 1024);
  const DevBuf& src = which == 0 ? d.ab.h0 : (which == 1 ? d.ab.h : d.ab.qkv);
  if (!src.p || need_n == 0) return fail(G4M_E_ARG, "no audio stage output is available");
  if (count < need_n) return fail(G4M_E_ARG, "host buffer too small");
  if (cudaDeviceSynchronize() || cudaMemcpy(host, src.p, need_n * 4, cudaMemcpyDeviceToHost))
    return fail(G4M_E_CUDA, "stage download failed");
  return G4M_OK;
}

}  // extern "C"
