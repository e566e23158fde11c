// Audio tower kernels: log-mel front end, fused two-layer subsample conv,
// chunked local self-attention and the light-conv depthwise block.
//
// Clips are packed back to back (ragged rows): clip c owns encoder rows
// [clip_row0[c], clip_row0[c] + clip_rows[c]).  Every row-coupled kernel
// (subsample conv, attention context, causal conv) stops at its clip's
// boundaries exactly as the reference stops at the end of one unpadded clip.
#include "g4m_kernels.h"
#include "g4m_sm100.cuh"

namespace g4m {

__device__ __forceinline__ float warp_sum_a(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max_a(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Log-mel front end: preprocessGemma4AudioSamples (src/preprocess/audio.ts:22-118)
// for unpadded clips: periodic Hann window (320), zero-padded radix-2 FFT
// (512), magnitude, HTK mel filters (257 x 128), log(mel + 1e-3).  One CTA
// (256 threads) per frame.  Frame f of a clip reads waveform samples
// [f*160 - 160, f*160 + 160) (160 leading zeros, frameLength / 2).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) logmel_kernel(const float* __restrict__ samples, const long* __restrict__ soff,
                                                     const long* __restrict__ slen, const int* __restrict__ foff,
                                                     const int* __restrict__ fcount, int clips,
                                                     const float* __restrict__ window, const float* __restrict__ mel,
                                                     const int* __restrict__ mel_rng, const double2* __restrict__ tw,
                                                     float* __restrict__ feats) {
  __shared__ float re[512], im[512], mag[257];
  const int gf = blockIdx.x;
  // clip of this frame: binary search over frame offsets
  int lo = 0, hi = clips - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (foff[mid] <= gf) lo = mid;
    else hi = mid - 1;
  }
  const int clip = lo, f = gf - foff[clip];
  if (f >= fcount[clip]) return;
  const float* x = samples + soff[clip];
  const long L = slen[clip];
  const int t = threadIdx.x;
  // bit-reversed load (9-bit index)
  for (int i = t; i < 512; i += 256) {
    float v = 0.f;
    if (i < 320) {
      const long idx = (long)f * 160 + i - 160;
      if (idx >= 0 && idx < L) v = x[idx] * window[i];
    }
    const int r = __brev(i) >> 23;
    re[r] = v;
    im[r] = 0.f;
  }
  __syncthreads();
  // Butterflies in double, stored to float, as fftRadix2 does with JS
  // numbers and Float32Array storage (src/preprocess/audio.ts:191-212).
  for (int size = 2; size <= 512; size <<= 1) {
    const int half = size >> 1;
    const int g = t / half, k = t % half;
    const int e = g * size + k, o = e + half;
    const double2 w = tw[k * (512 / size)];  // exp(-2 pi i k / size)
    const double orr = (double)re[o] * w.x - (double)im[o] * w.y;
    const double oi = (double)re[o] * w.y + (double)im[o] * w.x;
    const double er = re[e], ei = im[e];
    re[o] = (float)(er - orr);
    im[o] = (float)(ei - oi);
    re[e] = (float)(er + orr);
    im[e] = (float)(ei + oi);
    __syncthreads();
  }
  for (int b = t; b < 257; b += 256) mag[b] = (float)hypot((double)re[b], (double)im[b]);
  __syncthreads();
  if (t < 128) {
    double e = 0.0;  // mel energy in double (JS number), in bin order, over the non-zero bins
    const int b1 = mel_rng[2 * t + 1];
    for (int b = mel_rng[2 * t]; b <= b1; ++b) e += (double)mag[b] * (double)mel[b * 128 + t];
    feats[(long)gf * 128 + t] = (float)log(e + 0.001);
  }
}

cudaError_t audio_logmel(const float* samples, const long* sample_off, const long* sample_len, const int* frame_off,
                         const int* frames, int clips, int total_frames, const float* window, const float* mel,
                         const int* mel_rng, const double2* twiddle, float* features, cudaStream_t st) {
  if (total_frames <= 0) return cudaSuccess;
  logmel_kernel<<<total_frames, 256, 0, st>>>(samples, sample_off, sample_len, frame_off, frames, clips, window, mel,
                                              mel_rng, twiddle, features);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Chunked local self-attention (runAudioSelfAttentionBodyCpu and
// audioSelfAttentionScore, src/audio/kernels.ts:432-512): chunk 12, context
// 24 (12 past-horizon rows), 13 relative positions, per-dim softplus query
// scale, tanh softcap.  Out-of-clip context rows add no key term and no
// value, but their slot stays in the softmax with the relative-only score.
// One CTA per (clip block of 12 rows, head), 128 threads:
//   stage    the 24-row key / value window (keys pre-scaled), the 13
//            relative keys and the block's 12 scaled queries in shared memory
//   dots     the 12 x 24 query-key and 12 x 13 query-relative dot products,
//            each a float4 sequence over the 128 dims, spread over all threads
//   softmax  one warp per query row, lane = context slot: tanh softcap, max,
//            exp, sum; weights of out-of-clip slots kept in the denominator
//   P*V      thread = output dim, 24-term sums for each of the 12 rows
// qkv: [rows][3 * 1024] f32 (q | k | v); relk: [13][1024]; qmul: [128]
// (= 128^-0.5 / ln 2 * softplus(per_dim_scale)); kscale = ln(1 + e) / ln 2.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) audio_attn_kernel(const float* __restrict__ qkv, const float* __restrict__ relk,
                                                         const float* __restrict__ qmul, const int* __restrict__ blk_clip,
                                                         const int* __restrict__ blk_index,
                                                         const int* __restrict__ row0, const int* __restrict__ rows,
                                                         float kscale, float softcap, __half* __restrict__ o_hi,
                                                         __half* __restrict__ o_lo, float s_code) {
  constexpr int HD = 128, CH = 12, CTX = 24, PL = 13, D = 1024, PP = HD + 4;  // PP: padded row pitch
  __shared__ __align__(16) float qs[CH][PP], ks[CTX][PP], rk[PL][PP];
  __shared__ __align__(16) float vs[CTX][HD];
  __shared__ float dk[CH][CTX], dr[CH][PL], wt[CH][CTX];
  const int head = blockIdx.y;
  const int clip = blk_clip[blockIdx.x], blk = blk_index[blockIdx.x];
  const long r0 = row0[clip];
  const int nr = rows[clip];
  const int nq = min(CH, nr - blk * CH);  // query rows of this block
  const int t = threadIdx.x;  // staging: thread = head dim, every row's load in flight at once
  {
    const float qm = qmul[t];
    float kv[CTX], vv[CTX], rv[PL], qv[CH];
#pragma unroll
    for (int c = 0; c < CTX; ++c) {
      const int src = blk * CH + c - (CTX - CH);
      const bool ok = src >= 0 && src < nr;
      const float* row = qkv + (r0 + (ok ? src : 0)) * (3 * D) + head * HD + t;
      kv[c] = ok ? __ldg(row + D) : 0.f;
      vv[c] = ok ? __ldg(row + 2 * D) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < PL; ++r) rv[r] = __ldg(relk + r * D + head * HD + t);
#pragma unroll
    for (int qi = 0; qi < CH; ++qi)
      qv[qi] = qi < nq ? __ldg(qkv + (r0 + blk * CH + qi) * (3 * D) + head * HD + t) : 0.f;
#pragma unroll
    for (int c = 0; c < CTX; ++c) {
      ks[c][t] = kv[c] * kscale;
      vs[c][t] = vv[c];
    }
#pragma unroll
    for (int r = 0; r < PL; ++r) rk[r][t] = rv[r];
#pragma unroll
    for (int qi = 0; qi < CH; ++qi) qs[qi][t] = qv[qi] * qm;
  }
  __syncthreads();
  // dot products: items [0, 288) query-key, [288, 444) query-relative
  for (int it = t; it < CH * CTX + CH * PL; it += 128) {
    const bool isk = it < CH * CTX;
    const int qi = isk ? it / CTX : (it - CH * CTX) / PL;
    const int c = isk ? it % CTX : (it - CH * CTX) % PL;
    if (qi >= nq) continue;
    const float4* a = reinterpret_cast<const float4*>(qs[qi]);
    const float4* b = reinterpret_cast<const float4*>(isk ? ks[c] : rk[c]);
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;  // four independent chains
#pragma unroll 8
    for (int j = 0; j < HD / 4; ++j) {
      const float4 x = a[j], y = b[j];
      s0 = fmaf(x.x, y.x, s0);
      s1 = fmaf(x.y, y.y, s1);
      s2 = fmaf(x.z, y.z, s2);
      s3 = fmaf(x.w, y.w, s3);
    }
    const float s = (s0 + s1) + (s2 + s3);
    if (isk) dk[qi][c] = s;
    else dr[qi][c] = s;
  }
  for (int i = t; i < CH * CTX; i += 128) wt[i / CTX][i % CTX] = 0.f;
  __syncthreads();
  const int lane = t & 31, warp = t >> 5;
  for (int qi = warp; qi < nq; qi += 4) {
    const int src = blk * CH + lane - (CTX - CH);
    const bool kv_ok = lane < CTX && src >= 0 && src < nr;
    const int rel = lane - qi;
    const bool rel_ok = lane < CTX && rel >= 0 && rel < PL;
    float sc = -INFINITY;
    if (lane < CTX) {
      const float p = (kv_ok ? dk[qi][lane] : 0.f) + (rel_ok ? dr[qi][rel] : 0.f);
      sc = tanhf(p / softcap) * softcap;
    }
    const float mx = warp_max_a(sc);
    const float e = lane < CTX ? expf(sc - mx) : 0.f;
    const float den = warp_sum_a(e);
    if (lane < CTX) wt[qi][lane] = kv_ok ? e / den : 0.f;  // out-of-clip slots add no value
  }
  __syncthreads();
  const float inv_code = s_code != 0.0f ? 1.0f / s_code : 0.0f;
  float acc[CH];  // the 12 rows' sums as independent chains (rows >= nq have zero weights)
#pragma unroll
  for (int qi = 0; qi < CH; ++qi) acc[qi] = 0.f;
#pragma unroll
  for (int c = 0; c < CTX; ++c) {
    const float v = vs[c][t];
#pragma unroll
    for (int qi = 0; qi < CH; ++qi) acc[qi] = fmaf(wt[qi][c], v, acc[qi]);
  }
#pragma unroll
  for (int qi = 0; qi < CH; ++qi) {
    if (qi >= nq) break;
    const float o = acc[qi];
    const long oi = (r0 + blk * CH + qi) * D + head * HD + t;
    if (s_code != 0.0f) {  // integer codes for the post projection's input scale
      o_hi[oi] = __float2half_rn(srq_code(o, s_code, inv_code));
    } else {
      __half h, l;
      split_f16(o, h, l);
      o_hi[oi] = h;
      o_lo[oi] = l;
    }
  }
}

cudaError_t audio_attention_blocks(const float* qkv, const float* relk, const float* qmul, const int* blk_clip,
                                   const int* blk_index, int nblocks, const int* row0, const int* rows, float kscale,
                                   float softcap, __half* o_hi, __half* o_lo, float s_code, cudaStream_t st) {
  if (nblocks <= 0) return cudaSuccess;
  dim3 grid(nblocks, 8);
  audio_attn_kernel<<<grid, 128, 0, st>>>(qkv, relk, qmul, blk_clip, blk_index, row0, rows, kscale, softcap, o_hi,
                                          o_lo, s_code);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Light-conv middle: causal depthwise conv (kernel 5, left pad 4) within the
// clip (runAudioDepthwiseCausalConv1dCpu, src/audio/kernels.ts:855-884),
// conv_norm RMSNorm, SiLU (runSiluActivationCpu) -> fp16 hi/lo operand of
// linear_end (integer codes when s_code, linear_end's input scale, is non-zero).
// One warp per row, d = 1024.  dw: [5][1024] (tap-major).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) lconv_kernel(const float* __restrict__ g, const float* __restrict__ dw,
                                                    const float* __restrict__ nw, const int* __restrict__ row_clip,
                                                    const int* __restrict__ row0, long nrows, float eps,
                                                    __half* __restrict__ a_hi, __half* __restrict__ a_lo,
                                                    float s_code) {
  constexpr int D = 1024, V = D / 128, KS = 5;
  const int lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= nrows) return;
  const long local = row - row0[row_clip[row]];
  float4 acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int k = 0; k < KS; ++k) {
    const long src = local + k - (KS - 1);
    if (src < 0) continue;
    const float4* x = reinterpret_cast<const float4*>(g + (row + k - (KS - 1)) * D);
    const float4* wk = reinterpret_cast<const float4*>(dw + k * D);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 v = x[lane + 32 * i];
      const float4 w = __ldg(wk + lane + 32 * i);
      acc[i].x = fmaf(v.x, w.x, acc[i].x);
      acc[i].y = fmaf(v.y, w.y, acc[i].y);
      acc[i].z = fmaf(v.z, w.z, acc[i].z);
      acc[i].w = fmaf(v.w, w.w, acc[i].w);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) ss += acc[i].x * acc[i].x + acc[i].y * acc[i].y + acc[i].z * acc[i].z + acc[i].w * acc[i].w;
  const float inv = 1.0f / sqrtf(warp_sum_a(ss) / (float)D + eps);
  const float inv_code = s_code != 0.0f ? 1.0f / s_code : 0.0f;
  const float4* w = reinterpret_cast<const float4*>(nw);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float4 wv = w[lane + 32 * i];
    float v[4] = {(acc[i].x * inv) * wv.x, (acc[i].y * inv) * wv.y, (acc[i].z * inv) * wv.z, (acc[i].w * inv) * wv.w};
    __align__(8) __half hh[4], ll[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float s = v[u] / (1.0f + expf(-v[u]));
      if (s_code != 0.0f) hh[u] = __float2half_rn(srq_code(s, s_code, inv_code));
      else split_f16(s, hh[u], ll[u]);
    }
    const int c = 4 * (lane + 32 * i);
    *reinterpret_cast<uint2*>(a_hi + row * D + c) = *reinterpret_cast<uint2*>(hh);
    if (s_code == 0.0f) *reinterpret_cast<uint2*>(a_lo + row * D + c) = *reinterpret_cast<uint2*>(ll);
  }
}

cudaError_t audio_lconv_rows(const float* g, const float* dw, const float* nw, const int* row_clip, const int* row0,
                             long rows, float eps, __half* a_hi, __half* a_lo, float s_code, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  lconv_kernel<<<(int)((rows + 7) / 8), 256, 0, st>>>(g, dw, nw, row_clip, row0, rows, eps, a_hi, a_lo, s_code);
  return cudaGetLastError();
}

}  // namespace g4m
