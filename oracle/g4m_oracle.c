/*
 * g4m_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference library's CPU twins for the Gemma 4 E2B
 * media towers (ClinDesk-AI/gemma-4-webgpu-kernels-multimodal, TypeScript).
 * It is the parity oracle for the CUDA path and the timed CPU baseline; the
 * product library never links, loads or calls it.
 *
 * The reference is TypeScript and cannot run in this image (no JS runtime),
 * so every function here follows its TS counterpart line for line with JS
 * number semantics:
 *   - a TS `number` is a C `double`;
 *   - `Math.fround(x)` and every store into a `Float32Array` is `fr(x)`,
 *     i.e. one rounding of the double to float;
 *   - `Math.round(x)` rounds ties toward +infinity (`js_round`).
 * Build with -ffp-contract=off so no multiply-add is fused behind the
 * reference's back.  Hoisting a loop-invariant expression (for example the
 * quantised activation of one input row, or `fround(score/denominator)` of
 * the attention body) produces bit-identical values and is done for speed.
 *
 * Parity status: the integer paths (token layouts, soft-token counts,
 * checksums) are pinned to the literal examples in the reference's probes.
 * The floating-point paths have no reference golden vectors (the reference
 * ships none and compares CPU twins to WGSL live on the HF checkpoint), so
 * the floating-point restatement is "parity unpinned" beyond the
 * cross-check against an independent numpy restatement in tests/.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float fr(double x) { return (float)x; }

/* JS Math.round: nearest integer, ties toward +infinity. */
static inline double js_round(double x) {
  double f = floor(x);
  return (x - f >= 0.5) ? f + 1.0 : f;
}

/* srqScalar, src/kernels/qat.ts:489-492 */
static inline double srq(double v, double s) {
  if (s == 0.0) return v;
  double r = js_round(v / s);
  if (r > 127.0) r = 127.0;
  if (r < -128.0) r = -128.0;
  return r * s;
}

void g4mo_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int g4mo_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------------------ */
/* Linears                                                                   */
/* ------------------------------------------------------------------------ */

/* runQatI8LinearCpu, src/kernels/qat.ts:458-487.
 * y[r,o] = srq(fround(sum * s_w[o]), s_out), sum = fround-accumulated
 * fround(srq(x, s_in) * w).  Eight outputs are carried side by side; each
 * output's accumulation order over `col` is unchanged. */
int g4mo_qat_i8_linear(const float* x, const int8_t* w, const float* s_w, int rows, int in, int out,
                       float s_in, float s_out, float* y) {
  if (rows < 0 || in <= 0 || out <= 0) return -1;
#pragma omp parallel
  {
    double* a = (double*)malloc(sizeof(double) * (size_t)in);
    double* wt = (double*)malloc(sizeof(double) * (size_t)in * 8);
#pragma omp for schedule(dynamic, 1)
    for (int ob = 0; ob < (out + 7) / 8; ob++) {
      int o0 = ob * 8, nb = (out - o0) < 8 ? (out - o0) : 8;
      for (int c = 0; c < in; c++)
        for (int j = 0; j < 8; j++) wt[(size_t)c * 8 + j] = j < nb ? (double)w[(size_t)(o0 + j) * in + c] : 0.0;
      for (int r = 0; r < rows; r++) {
        for (int c = 0; c < in; c++) a[c] = srq((double)x[(size_t)r * in + c], (double)s_in);
        float sum[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int c = 0; c < in; c++) {
          const double ac = a[c];
          const double* wr = wt + (size_t)c * 8;
          for (int j = 0; j < 8; j++) sum[j] = fr((double)sum[j] + (double)fr(ac * wr[j]));
        }
        for (int j = 0; j < nb; j++)
          y[(size_t)r * out + o0 + j] = fr(srq((double)fr((double)sum[j] * (double)s_w[o0 + j]), (double)s_out));
      }
    }
    free(a);
    free(wt);
  }
  return 0;
}

/* packedQatWeightCode, src/kernels/qat.ts:249-261 */
static inline int packed_code(const uint8_t* w, int o, int col, int in, int bits) {
  int vpb = 8 / bits;
  size_t bpr = (size_t)in * bits / 8;
  size_t bi = (size_t)o * bpr + (size_t)(col / vpb);
  int lane = col % vpb;
  return (w[bi] >> (lane * bits)) & ((1 << bits) - 1);
}

int g4mo_packed_weight_code(const uint8_t* w, int o, int col, int in, int bits) {
  return packed_code(w, o, col, in, bits);
}

/* runPackedQatLinearCpu, src/kernels/qat.ts:215-247.
 * y = srq(fround(s_w * fround(sumQA - fround(zp * sumA))), s_out). */
int g4mo_packed_qat_linear(const float* x, const uint8_t* w, const float* s_w, int rows, int in, int out,
                           int bits, float s_in, float s_out, float* y) {
  if (!(bits == 2 || bits == 4 || bits == 8)) return -1;
  const double zp = (double)(1 << (bits - 1));
#pragma omp parallel
  {
    double* a = (double*)malloc(sizeof(double) * (size_t)in);
    double* wt = (double*)malloc(sizeof(double) * (size_t)in * 8);
#pragma omp for schedule(dynamic, 1)
    for (int ob = 0; ob < (out + 7) / 8; ob++) {
      int o0 = ob * 8, nb = (out - o0) < 8 ? (out - o0) : 8;
      for (int c = 0; c < in; c++)
        for (int j = 0; j < 8; j++) wt[(size_t)c * 8 + j] = j < nb ? (double)packed_code(w, o0 + j, c, in, bits) : 0.0;
      for (int r = 0; r < rows; r++) {
        for (int c = 0; c < in; c++) a[c] = srq((double)x[(size_t)r * in + c], (double)s_in);
        float sqa[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float sa = 0.f;
        for (int c = 0; c < in; c++) {
          const double ac = a[c];
          const double* wr = wt + (size_t)c * 8;
          for (int j = 0; j < 8; j++) sqa[j] = fr((double)sqa[j] + (double)fr(wr[j] * ac));
          sa = fr((double)sa + ac);
        }
        for (int j = 0; j < nb; j++) {
          float inner = fr((double)sqa[j] - (double)fr(zp * (double)sa));
          y[(size_t)r * out + o0 + j] = fr(srq((double)fr((double)s_w[o0 + j] * (double)inner), (double)s_out));
        }
      }
    }
    free(a);
    free(wt);
  }
  return 0;
}

/* runF32LinearRowsCpu, src/kernels/qat.ts:6-33 (double accumulation). */
int g4mo_f32_linear_rows(const float* x, const float* w, int rows, int in, int out, float* y) {
#pragma omp parallel for schedule(dynamic, 1)
  for (int o = 0; o < out; o++) {
    const float* wr = w + (size_t)o * in;
    for (int r = 0; r < rows; r++) {
      const float* xr = x + (size_t)r * in;
      double sum = 0.0;
      for (int c = 0; c < in; c++) sum += (double)xr[c] * (double)wr[c];
      y[(size_t)r * out + o] = fr(sum);
    }
  }
  return 0;
}

/* runMultimodalEmbedderCpu, src/embedder/index.ts:111-145. */
int g4mo_embedder(const float* h, const float* w, int rows, int in, int out, double eps, float* y) {
  double* inv = (double*)malloc(sizeof(double) * (size_t)(rows > 0 ? rows : 1));
  for (int r = 0; r < rows; r++) {
    double ms = 0.0;
    for (int c = 0; c < in; c++) {
      double v = h[(size_t)r * in + c];
      ms += v * v;
    }
    inv[r] = pow(ms / in + eps, -0.5);
  }
#pragma omp parallel for schedule(dynamic, 1)
  for (int o = 0; o < out; o++) {
    const float* wr = w + (size_t)o * in;
    for (int r = 0; r < rows; r++) {
      const float* hr = h + (size_t)r * in;
      double sum = 0.0;
      for (int c = 0; c < in; c++) sum += (double)hr[c] * inv[r] * (double)wr[c];
      y[(size_t)r * out + o] = fr(sum);
    }
  }
  free(inv);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Vision kernels (src/vision/kernels.ts)                                    */
/* ------------------------------------------------------------------------ */

/* runVisionRmsNormCpu, src/vision/kernels.ts:5-32 (also the audio RMSNorm). */
int g4mo_rmsnorm(const float* x, const float* w, int rows, int d, double eps, float* y) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    const float* xr = x + (size_t)r * d;
    double ms = 0.0;
    for (int i = 0; i < d; i++) {
      double v = xr[i];
      ms += v * v;
    }
    double inv = pow(ms / d + eps, -0.5);
    for (int i = 0; i < d; i++) y[(size_t)r * d + i] = fr((double)xr[i] * inv * (double)w[i]);
  }
  return 0;
}

/* runVisionRopeCpu, src/vision/kernels.ts:34-73.  pos is [rows][2] = (x, y). */
int g4mo_vision_rope(const float* v, const int* pos, int rows, int heads, int hd, double theta, float* y) {
  if (hd % 4 != 0) return -1;
  const int part_size = hd / 2, half = part_size / 2;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    for (int h = 0; h < heads; h++) {
      size_t base = ((size_t)r * heads + h) * hd;
      for (int ch = 0; ch < hd; ch++) {
        int part = ch < part_size ? 0 : 1;
        int po = ch - part * part_size;
        int fi = po % half;
        double p = part == 0 ? (double)pos[2 * r] : (double)pos[2 * r + 1];
        double angle = p / pow(theta, (double)(2 * fi) / (double)part_size);
        int paired = po < half ? po + half : po - half;
        double rotated = (po < half ? -1.0 : 1.0) * (double)v[base + part * part_size + paired];
        y[base + ch] = fr((double)v[base + ch] * cos(angle) + rotated * sin(angle));
      }
    }
  }
  return 0;
}

/* runVisionAttentionBodyCpu + visionAttentionScore, src/vision/kernels.ts:75-131.
 * q, k, v, o are [rows][heads][hd]. */
int g4mo_vision_attention(const float* q, const float* k, const float* v, int rows, int heads, int hd,
                          double scaling, float* o) {
#pragma omp parallel
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)rows);
    float* acc = (float*)malloc(sizeof(float) * (size_t)hd);
#pragma omp for schedule(dynamic, 4)
    for (int rh = 0; rh < rows * heads; rh++) {
      int r = rh / heads, h = rh % heads;
      const float* qr = q + ((size_t)r * heads + h) * hd;
      double mx = -INFINITY;
      for (int kr = 0; kr < rows; kr++) {
        const float* kk = k + ((size_t)kr * heads + h) * hd;
        float s = 0.f;
        for (int d = 0; d < hd; d++) s = fr((double)s + (double)fr((double)qr[d] * (double)kk[d]));
        float score = fr((double)s * scaling);
        sc[kr] = score;
        if ((double)score > mx) mx = score;
      }
      float den = 0.f;
      for (int kr = 0; kr < rows; kr++) {
        float wgt = fr(exp((double)fr((double)sc[kr] - mx)));
        sc[kr] = wgt;
        den = fr((double)den + (double)wgt);
      }
      for (int kr = 0; kr < rows; kr++) sc[kr] = fr((double)sc[kr] / (double)den);
      for (int d = 0; d < hd; d++) acc[d] = 0.f;
      for (int kr = 0; kr < rows; kr++) {
        const double wk = sc[kr];
        const float* vv = v + ((size_t)kr * heads + h) * hd;
        for (int d = 0; d < hd; d++) acc[d] = fr((double)acc[d] + (double)fr(wk * (double)vv[d]));
      }
      memcpy(o + ((size_t)r * heads + h) * hd, acc, sizeof(float) * (size_t)hd);
    }
    free(sc);
    free(acc);
  }
  return 0;
}

/* runResidualAddCpu, src/vision/kernels.ts:133-142. */
int g4mo_residual_add(const float* r, const float* v, long n, float* y) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; i++) y[i] = fr((double)r[i] + (double)v[i]);
  return 0;
}

/* geluPytorchTanh, src/vision/kernels.ts:155-159. */
static inline double gelu_tanh(double x) {
  double inner = 0.7978845608028654 * (x + 0.044715 * x * x * x);
  double t = 2.0 / (1.0 + exp(-2.0 * inner)) - 1.0;
  return 0.5 * x * (1.0 + t);
}

/* runVisionMlpActivationCpu, src/vision/kernels.ts:144-153. */
int g4mo_gelu_gate(const float* gate, const float* up, long n, float* y) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; i++) y[i] = fr(gelu_tanh((double)gate[i]) * (double)up[i]);
  return 0;
}

/* visionPoolIndices, src/vision/kernels.ts:955-980.  Returns -1 on a layout error. */
int g4mo_vision_pool_indices(const int* pos, int npos, int out_len, int k, int* idx) {
  if (npos <= 0) return -1;
  int maxx = pos[0], maxy = pos[1];
  for (int i = 1; i < npos; i++) {
    if (pos[2 * i] > maxx) maxx = pos[2 * i];
    if (pos[2 * i + 1] > maxy) maxy = pos[2 * i + 1];
  }
  maxx += 1;
  maxy += 1;
  int cx = maxx / k, cy = maxy / k, kk = k * k;
  if (cx * cy != out_len) return -1;
  for (int i = 0; i < out_len * kk; i++) idx[i] = -1;
  for (int p = 0; p < npos; p++) {
    int x = pos[2 * p], y = pos[2 * p + 1];
    int tok = x / k + cx * (y / k);
    int local = (y % k) * k + (x % k);
    if (tok < 0 || tok >= out_len) return -1;
    idx[tok * kk + local] = p;
  }
  return 0;
}

/* runVisionPoolerCpu, src/vision/kernels.ts:815-833. */
int g4mo_vision_pooler(const float* h, const int* pos, int npos, int out_len, int d, int k, float* y) {
  int kk = k * k;
  int* idx = (int*)malloc(sizeof(int) * (size_t)out_len * kk);
  if (g4mo_vision_pool_indices(pos, npos, out_len, k, idx) != 0) {
    free(idx);
    return -1;
  }
  double scale = sqrt((double)d);
#pragma omp parallel for schedule(static)
  for (int t = 0; t < out_len; t++) {
    for (int c = 0; c < d; c++) {
      double sum = 0.0;
      for (int j = 0; j < kk; j++) {
        int p = idx[t * kk + j];
        if (p >= 0) sum += (double)h[(size_t)p * d + c];
      }
      y[(size_t)t * d + c] = fr((sum / kk) * scale);
    }
  }
  free(idx);
  return 0;
}

/* runVisionPatchEmbeddingCpu, src/vision/kernels.ts:982-1019.
 * patches [npatch][pp], w [out_rows][pp], posx/posy are [nrows][d]. */
int g4mo_vision_patch_embed(const float* patches, const float* w, const int* pos, int npatch, int pp, int d,
                            int out_rows, const float* posx, int nposx, const float* posy, int nposy, float* y) {
  for (int p = 0; p < npatch; p++) {
    if (pos[2 * p] < 0 || pos[2 * p] >= nposx || pos[2 * p + 1] < 0 || pos[2 * p + 1] >= nposy) return -1;
  }
#pragma omp parallel for schedule(static)
  for (int p = 0; p < npatch; p++) {
    const float* pv = patches + (size_t)p * pp;
    size_t xo = (size_t)pos[2 * p] * d, yo = (size_t)pos[2 * p + 1] * d;
    for (int r = 0; r < out_rows; r++) {
      const float* wr = w + (size_t)r * pp;
      double sum = 0.0;
      for (int c = 0; c < pp; c++) {
        double scaled = 2.0 * ((double)pv[c] - 0.5);
        sum += scaled * (double)wr[c];
      }
      y[(size_t)p * out_rows + r] = fr(sum + (double)posx[xo + r] + (double)posy[yo + r]);
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Audio kernels (src/audio/kernels.ts)                                      */
/* ------------------------------------------------------------------------ */

/* audioSubsampleOutputLength, src/audio/kernels.ts:1242-1244. */
int g4mo_audio_subsample_output_length(int n) { return (int)floor((n + 2 - 3) / 2.0) + 1; }

/* computeGemma4AudioSoftTokensFromMask, src/audio/kernels.ts:7-20. */
int g4mo_audio_soft_tokens_from_mask(const uint8_t* mask, int n, int seq_len) {
  uint8_t* cur = (uint8_t*)malloc((size_t)(n > 0 ? n : 1));
  memcpy(cur, mask, (size_t)n);
  int len = n;
  for (int layer = 0; layer < 2; layer++) {
    int ol = (int)floor((len + 2 - 3) / 2.0) + 1;
    if (ol < 0) ol = 0;
    uint8_t* nx = (uint8_t*)malloc((size_t)(ol > 0 ? ol : 1));
    for (int i = 0; i < ol; i++) nx[i] = (i * 2 < len) ? cur[i * 2] : 0;
    free(cur);
    cur = nx;
    len = ol;
  }
  int total = 0;
  for (int i = 0; i < len; i++) total += cur[i];
  free(cur);
  return total < seq_len ? total : seq_len;
}

/* runAudioSubsampleConvLayerCpu + audioSubsampleConvValueCpu + strideAudioMask,
 * src/audio/kernels.ts:112-183, 1246-1252.  Channel-last layout (t*F+f)*C+c. */
int g4mo_audio_subsample_conv_layer(const float* x, const uint8_t* mask, int in_t, int in_f, int in_c,
                                    const float* w, const float* nw, int out_c, double eps, float* y,
                                    uint8_t* out_mask) {
  int ot = g4mo_audio_subsample_output_length(in_t);
  int of = g4mo_audio_subsample_output_length(in_f);
#pragma omp parallel
  {
    float* cv = (float*)malloc(sizeof(float) * (size_t)out_c);
#pragma omp for schedule(static)
    for (int t = 0; t < ot; t++) {
      for (int f = 0; f < of; f++) {
        double mean = 0.0;
        for (int oc = 0; oc < out_c; oc++) {
          double sum = 0.0;
          for (int ic = 0; ic < in_c; ic++) {
            for (int kt = 0; kt < 3; kt++) {
              int st = t * 2 + kt - 1;
              if (st < 0 || st >= in_t || mask[st] == 0) continue;
              for (int kf = 0; kf < 3; kf++) {
                int sf = f * 2 + kf - 1;
                if (sf < 0 || sf >= in_f) continue;
                double iv = x[((size_t)st * in_f + sf) * in_c + ic];
                double wv = w[(((size_t)oc * in_c + ic) * 3 + kt) * 3 + kf];
                sum += iv * wv;
              }
            }
          }
          cv[oc] = fr(sum);
          mean += sum;
        }
        mean /= out_c;
        double var = 0.0;
        for (int oc = 0; oc < out_c; oc++) {
          double c = (double)cv[oc] - mean;
          var += c * c;
        }
        double inv = pow(var / out_c + eps, -0.5);
        for (int oc = 0; oc < out_c; oc++) {
          double nrm = ((double)cv[oc] - mean) * inv * (double)nw[oc];
          y[((size_t)t * of + f) * out_c + oc] = fr(nrm > 0.0 ? nrm : 0.0);
        }
      }
    }
    free(cv);
  }
  for (int i = 0; i < ot; i++) out_mask[i] = (i * 2 < in_t) ? mask[i * 2] : 0;
  return 0;
}

/* audioRelativePositionEmbeddings, src/audio/kernels.ts:415-430. */
int g4mo_audio_relpos(int plen, int d, float* y) {
  if (d % 2 != 0) return -1;
  int half = d / 2;
  double li = log(10000.0) / (double)(half - 1 > 1 ? half - 1 : 1);
  for (int pi = 0; pi < plen; pi++) {
    double p = (double)(plen - 1 - pi);
    for (int dd = 0; dd < half; dd++) {
      double s = p * exp((double)dd * -li);
      y[(size_t)pi * d + dd] = fr(sin(s));
      y[(size_t)pi * d + half + dd] = fr(cos(s));
    }
  }
  return 0;
}

/* softplus, src/audio/kernels.ts:514-518. */
static inline double softplus(double v) {
  if (v > 20) return v;
  if (v < -20) return exp(v);
  return log(1 + exp(v));
}

/* runAudioSelfAttentionBodyCpu + audioSelfAttentionScore +
 * audioSelfAttentionContextSourceRow, src/audio/kernels.ts:432-512.
 * q, k, v, o are [rows][heads][hd]; relk is [plen][heads][hd]. */
int g4mo_audio_attention(const float* q, const float* k, const float* v, const float* relk, const float* pds,
                         int rows, int heads, int hd, int chunk, int ctx, int plen, double softcap, float* o) {
  const double qscale = pow((double)hd, -0.5) / log(2.0);
  const double kscale = log(1.0 + exp(1.0)) / log(2.0);
  const int horizon = ctx - chunk;
#pragma omp parallel
  {
    float* sc = (float*)malloc(sizeof(float) * (size_t)ctx);
    double* qv = (double*)malloc(sizeof(double) * (size_t)hd);
#pragma omp for schedule(static)
    for (int rh = 0; rh < rows * heads; rh++) {
      int r = rh / heads, h = rh % heads;
      const float* qr = q + ((size_t)r * heads + h) * hd;
      for (int d = 0; d < hd; d++) qv[d] = (double)qr[d] * qscale * softplus((double)pds[d]);
      int block = r / chunk, qpos = r % chunk;
      double mx = -INFINITY;
      for (int c = 0; c < ctx; c++) {
        int src = block * chunk + c - horizon;
        int rel = (c >= qpos && c < qpos + plen) ? c - qpos : -1;
        float s = 0.f;
        for (int d = 0; d < hd; d++) {
          if (src >= 0 && src < rows) {
            double key = (double)k[((size_t)src * heads + h) * hd + d] * kscale;
            s = fr((double)s + (double)fr(qv[d] * key));
          }
          if (rel >= 0) {
            double relv = relk[((size_t)rel * heads + h) * hd + d];
            s = fr((double)s + (double)fr(qv[d] * relv));
          }
        }
        double score = tanh((double)s / softcap) * softcap;
        sc[c] = fr(score);
        if (score > mx) mx = score;
      }
      float den = 0.f;
      for (int c = 0; c < ctx; c++) {
        float wgt = fr(exp((double)fr((double)sc[c] - mx)));
        sc[c] = wgt;
        den = fr((double)den + (double)wgt);
      }
      for (int d = 0; d < hd; d++) {
        float sum = 0.f;
        for (int c = 0; c < ctx; c++) {
          int src = block * chunk + c - horizon;
          if (src < 0 || src >= rows) continue;
          float wgt = fr((double)sc[c] / (double)den);
          double val = v[((size_t)src * heads + h) * hd + d];
          sum = fr((double)sum + (double)fr((double)wgt * val));
        }
        o[((size_t)r * heads + h) * hd + d] = sum;
      }
    }
    free(sc);
    free(qv);
  }
  return 0;
}

/* runGluActivationCpu, src/audio/kernels.ts:735-750.  x is [rows][2*hs]. */
int g4mo_glu(const float* x, int rows, int hs, float* y) {
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    for (int d = 0; d < hs; d++) {
      double g = x[(size_t)r * hs * 2 + d];
      double sg = 1.0 / (1.0 + exp(-(double)x[(size_t)r * hs * 2 + hs + d]));
      y[(size_t)r * hs + d] = fr(g * sg);
    }
  }
  return 0;
}

/* runAudioDepthwiseCausalConv1dCpu, src/audio/kernels.ts:855-884.  w is [hs][ks]. */
int g4mo_depthwise_causal(const float* x, const float* w, int rows, int hs, int ks, float* y) {
  int lp = ks - 1;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    for (int d = 0; d < hs; d++) {
      float sum = 0.f;
      for (int k = 0; k < ks; k++) {
        int s = r + k - lp;
        if (s < 0 || s >= rows) continue;
        sum = fr((double)sum + (double)fr((double)x[(size_t)s * hs + d] * (double)w[(size_t)d * ks + k]));
      }
      y[(size_t)r * hs + d] = sum;
    }
  }
  return 0;
}

/* runSiluActivationCpu, src/audio/kernels.ts:1016-1022. */
int g4mo_silu(const float* x, long n, float* y) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; i++) y[i] = fr((double)x[i] / (1.0 + exp(-(double)x[i])));
  return 0;
}

/* runScaledResidualAddCpu, src/audio/kernels.ts:1116-1125. */
int g4mo_scaled_residual_add(const float* r, const float* v, long n, double scale, float* y) {
#pragma omp parallel for schedule(static)
  for (long i = 0; i < n; i++) y[i] = fr((double)r[i] + (double)fr((double)v[i] * scale));
  return 0;
}

/* runAudioOutputProjectionWebGpu host bias step, src/audio/kernels.ts:405-411:
 * y = fround(y + bias) applied to the F32 linear rows. */
int g4mo_add_bias_rows(float* y, const float* b, int rows, int d) {
  for (int r = 0; r < rows; r++)
    for (int i = 0; i < d; i++) y[(size_t)r * d + i] = fr((double)y[(size_t)r * d + i] + (double)b[i]);
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Preprocessing (src/preprocess/audio.ts, src/preprocess/image.ts)          */
/* ------------------------------------------------------------------------ */

/* computeGemma4AudioSoftTokenCount, src/preprocess/audio.ts:4-20. */
long g4mo_audio_soft_token_count(double samples, double frame_len, double hop, double seq_len) {
  double fsu = frame_len + 1;
  double pad_left = floor(frame_len / 2);
  double nmel = floor((samples + pad_left - fsu) / hop) + 1;
  if (nmel <= 0) return 0;
  double ts = nmel;
  for (int l = 0; l < 2; l++) ts = floor((ts + 2 * 1 - 3) / 2) + 1;
  return (long)(ts < seq_len ? ts : seq_len);
}

/* aspectRatioPreservingSize + computeGemma4ImageTokenLayout,
 * src/preprocess/image.ts:4-30, 217-252.
 * out = {target_h, target_w, grid_h, grid_w, max_patches, soft_tokens}.
 * Returns 0, or -1/-2/-3 for the three errors the reference throws. */
int g4mo_image_token_layout(double height, double width, double patch, double max_soft, double pool, long* out) {
  double max_patches = max_soft * pool * pool;
  if (height <= 0 || width <= 0) return -1;
  double total = height * width;
  double target_px = max_patches * patch * patch;
  double factor = sqrt(target_px / total);
  double ih = factor * height, iw = factor * width;
  double side = pool * patch;
  double th = floor(ih / side) * side, tw = floor(iw / side) * side;
  if (th == 0 && tw == 0) return -2;
  double max_side = floor(max_patches / (pool * pool)) * side;
  if (th == 0) {
    th = side;
    double c = floor(width / height) * side;
    tw = c < max_side ? c : max_side;
  } else if (tw == 0) {
    tw = side;
    double c = floor(height / width) * side;
    th = c < max_side ? c : max_side;
  }
  if (th * tw > target_px) return -3;
  double gh = th / patch, gw = tw / patch;
  out[0] = (long)th;
  out[1] = (long)tw;
  out[2] = (long)gh;
  out[3] = (long)gw;
  out[4] = (long)max_patches;
  out[5] = (long)floor((gh * gw) / (pool * pool));
  return 0;
}

/* fftRadix2, src/preprocess/audio.ts:171-214 (Float32Array storage). */
static void fft_radix2(float* re, float* im, int n) {
  int j = 0;
  for (int i = 1; i < n; i++) {
    int bit = n >> 1;
    while (j & bit) {
      j ^= bit;
      bit >>= 1;
    }
    j ^= bit;
    if (i < j) {
      float tr = re[i], ti = im[i];
      re[i] = re[j];
      im[i] = im[j];
      re[j] = tr;
      im[j] = ti;
    }
  }
  for (int size = 2; size <= n; size <<= 1) {
    int half = size >> 1;
    double theta = -2 * M_PI / size;
    double sr = cos(theta), si = sin(theta);
    for (int start = 0; start < n; start += size) {
      double pr = 1, pi = 0;
      for (int off = 0; off < half; off++) {
        int ev = start + off, od = ev + half;
        double orr = (double)re[od] * pr - (double)im[od] * pi;
        double oi = (double)re[od] * pi + (double)im[od] * pr;
        re[od] = fr((double)re[ev] - orr);
        im[od] = fr((double)im[ev] - oi);
        re[ev] = fr((double)re[ev] + orr);
        im[ev] = fr((double)im[ev] + oi);
        double npr = pr * sr - pi * si;
        pi = pr * si + pi * sr;
        pr = npr;
      }
    }
  }
}

/* createHtkMelFilterBank, src/preprocess/audio.ts:128-157.  filters [bins][nmel]. */
int g4mo_htk_mel_filters(int bins, int nmel, double fmin, double fmax, double sr, float* filters) {
  double mmin = 2595 * log10(1 + fmin / 700), mmax = 2595 * log10(1 + fmax / 700);
  double* ff = (double*)malloc(sizeof(double) * (size_t)(nmel + 2));
  for (int i = 0; i < nmel + 2; i++) {
    double mel = mmin + ((mmax - mmin) * i) / (nmel + 1);
    ff[i] = 700 * (pow(10, mel / 2595) - 1);
  }
  double bw = sr / ((bins - 1) * 2.0);
  for (int b = 0; b < bins; b++) {
    double f = bw * b;
    for (int m = 0; m < nmel; m++) {
      double l = ff[m], c = ff[m + 1], r = ff[m + 2];
      double up = c == l ? 0 : (f - l) / (c - l);
      double dn = r == c ? 0 : (r - f) / (r - c);
      double v = up < dn ? up : dn;
      filters[(size_t)b * nmel + m] = fr(v > 0 ? v : 0);
    }
  }
  free(ff);
  return 0;
}

/* Frame count of preprocessGemma4AudioSamples for given options
 * (src/preprocess/audio.ts:46-59). */
long g4mo_audio_frame_count(long n_raw, long max_samples, long pad_multiple, int frame_len, int hop) {
  long src = n_raw < max_samples ? n_raw : max_samples;
  long padded = pad_multiple > 0 ? ((src + pad_multiple - 1) / pad_multiple) * pad_multiple : src;
  long wl = frame_len / 2 + padded;
  return wl >= frame_len + 1 ? (wl - (frame_len + 1)) / hop + 1 : 0;
}

/* preprocessGemma4AudioSamples, src/preprocess/audio.ts:22-118.
 * features [frames][nmel] and mask [frames] must hold g4mo_audio_frame_count
 * entries.  Writes *valid_frames. */
long g4mo_preprocess_audio(const float* raw, long n_raw, double in_scale, long max_samples, long pad_multiple,
                           int sr, int nmel, int frame_len, int hop, int fft_len, double fmin, double fmax,
                           double mel_floor, float* features, uint8_t* mask, long* valid_frames) {
  if (fft_len <= 0 || (fft_len & (fft_len - 1)) != 0 || fft_len < frame_len) return -1;
  long src = n_raw < max_samples ? n_raw : max_samples;
  long padded = pad_multiple > 0 ? ((src + pad_multiple - 1) / pad_multiple) * pad_multiple : src;
  long pad_left = frame_len / 2;
  long wl = pad_left + padded;
  float* wave = (float*)calloc((size_t)wl, sizeof(float));
  uint8_t* am = (uint8_t*)calloc((size_t)wl, 1);
  for (long i = 0; i < src; i++) {
    wave[pad_left + i] = fr((double)raw[i] * in_scale);
    am[pad_left + i] = 1;
  }
  long frames = wl >= frame_len + 1 ? (wl - (frame_len + 1)) / hop + 1 : 0;
  int bins = fft_len / 2 + 1;
  float* win = (float*)malloc(sizeof(float) * (size_t)frame_len);
  for (int i = 0; i < frame_len; i++) win[i] = fr(0.5 - 0.5 * cos((2 * M_PI * i) / frame_len));
  float* filt = (float*)malloc(sizeof(float) * (size_t)bins * nmel);
  g4mo_htk_mel_filters(bins, nmel, fmin, fmax, sr, filt);
  long vf = 0;
#pragma omp parallel reduction(+ : vf)
  {
    float* re = (float*)malloc(sizeof(float) * (size_t)fft_len);
    float* im = (float*)malloc(sizeof(float) * (size_t)fft_len);
    float* mag = (float*)malloc(sizeof(float) * (size_t)bins);
#pragma omp for schedule(static)
    for (long fi = 0; fi < frames; fi++) {
      long fs = fi * hop;
      for (int i = 0; i < fft_len; i++) {
        re[i] = 0.f;
        im[i] = 0.f;
      }
      for (int i = 0; i < frame_len; i++) re[i] = fr((double)wave[fs + i] * (double)win[i]);
      fft_radix2(re, im, fft_len);
      for (int i = 0; i < bins; i++) mag[i] = fr(hypot((double)re[i], (double)im[i]));
      long fe = fs + frame_len + 1 - 1;
      int valid = am[fe] == 1;
      if (valid) vf += 1;
      mask[fi] = valid ? 1 : 0;
      for (int m = 0; m < nmel; m++) {
        double e = 0;
        for (int b = 0; b < bins; b++) e += (double)mag[b] * (double)filt[(size_t)b * nmel + m];
        features[(size_t)fi * nmel + m] = valid ? fr(log(e + mel_floor)) : 0.f;
      }
    }
    free(re);
    free(im);
    free(mag);
  }
  *valid_frames = vf;
  free(wave);
  free(am);
  free(win);
  free(filt);
  return frames;
}

/* ------------------------------------------------------------------------ */
/* Result helpers (src/utils/math.ts)                                        */
/* ------------------------------------------------------------------------ */

/* checksumFloats, src/utils/math.ts:3-12 (double arithmetic as in JS). */
double g4mo_checksum_floats(const float* v, long n) {
  const double mod = 1000000007.0;
  double c = 0;
  long lim = n < 4096 ? n : 4096;
  for (long i = 0; i < lim; i++) {
    c = fmod(c + js_round((double)v[i] * 1000000.0) * (double)(i + 1), mod);
    if (c < 0) c += mod;
  }
  return c;
}

/* roundedSample, src/utils/math.ts:131-133. */
void g4mo_rounded_sample(const float* v, long n, double* out8) {
  for (long i = 0; i < 8 && i < n; i++) out8[i] = js_round((double)v[i] * 1000000.0) / 1000000.0;
}
