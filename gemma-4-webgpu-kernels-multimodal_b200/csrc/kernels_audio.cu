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
// One CTA per (run of up to kAudioAttnRun consecutive 12-row blocks of one
// clip, head), 128 threads.  The 13 relative keys are staged once; a block's
// 12 query / key / value rows are prefetched into registers (thread = head
// dim) while the previous block computes, and after each block its key and
// value rows shift down to become the next block's past window:
//   dots     the 12 x 40 products of the queries with [24 keys | 13 relative
//            keys | 3 zero rows] as a register-blocked tile product: warp w
//            takes dims [32w, 32w + 32), lane (qg, cg) = (lane & 3, lane >> 2)
//            a 3 x 5 block of rows 3qg.. and slots 5cg..; each float4 step
//            loads 8 vectors (broadcast, bank-conflict free with the 132-float
//            row pitch) for 60 FMAs; the 4 warps' partial sums meet in the
//            softmax
//   softmax  one warp per query row, lane = context slot: tanh softcap, max,
//            exp, sum; weights of out-of-clip slots kept in the denominator
//   P*V      thread = output dim, 24-term sums for each of the 12 rows
// qkv: [rows][3 * 1024] f32 (q | k | v); relk: [13][1024]; qmul: [128]
// (= 128^-0.5 / ln 2 * softplus(per_dim_scale)); kscale = ln(1 + e) / ln 2.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128, 4) audio_attn_kernel(const float* __restrict__ qkv,
                                                            const float* __restrict__ relk,
                                                            const float* __restrict__ qmul,
                                                            const int* __restrict__ run_clip,
                                                            const int* __restrict__ run_blk0,
                                                            const int* __restrict__ row0, const int* __restrict__ rows,
                                                            float kscale, float softcap, __half* __restrict__ o_hi,
                                                            __half* __restrict__ o_lo, float s_code) {
  constexpr int HD = 128, CH = 12, CTX = 24, PL = 13, NB = 40, D = 1024, PP = HD + 4;  // PP: padded row pitch
  constexpr int NW = 4;  // warps, one 32-dim slice each in the dot phase
  // qr: the block's queries [12][PP] in the dot phase, then the warps'
  // partial sums red[NW][12][NB] until the softmax is done
  __shared__ __align__(16) float qr[NW * CH * NB];
  // ks rows [0, 12) the previous block's keys, [12, 24) this block's,
  // [24, 37) relative keys, [37, 40) zero
  __shared__ __align__(16) float ks[NB * PP];
  __shared__ __align__(16) float vs[CTX][HD];
  __shared__ __align__(16) float wt[CH][CTX];
  static_assert(NW * CH * NB >= CH * PP, "partial sums alias the queries");
  const int head = blockIdx.y;
  const int clip = run_clip[blockIdx.x], b0 = run_blk0[blockIdx.x];
  const long r0 = row0[clip];
  const int nr = rows[clip];
  const int b1 = min(b0 + kAudioAttnRun, (nr + CH - 1) / CH);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float qm = qmul[t];
  const float* col = qkv + r0 * (3 * D) + head * HD + t;  // this thread's dim of row 0's q
#pragma unroll
  for (int r = 0; r < PL; ++r) ks[(CTX + r) * PP + t] = __ldg(relk + r * D + head * HD + t);
#pragma unroll
  for (int r = CTX + PL; r < NB; ++r) ks[r * PP + t] = 0.f;
#pragma unroll
  for (int c = 0; c < CH; ++c) {  // the past window of block b0 (rows of block b0 - 1; none before row 0)
    const int src = b0 * CH - CH + c;
    const bool ok = src >= 0;
    ks[c * PP + t] = ok ? __ldg(col + (long)src * (3 * D) + D) * kscale : 0.f;
    vs[c][t] = ok ? __ldg(col + (long)src * (3 * D) + 2 * D) : 0.f;
  }
  float pq[CH], pk[CH], pv[CH];  // the next block's rows, in flight while the current one computes
  auto prefetch = [&](int b) {
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int src = b * CH + i;
      const bool ok = src < nr;
      const float* p = col + (long)(ok ? src : 0) * (3 * D);
      pq[i] = ok ? __ldg(p) : 0.f;
      pk[i] = ok ? __ldg(p + D) : 0.f;
      pv[i] = ok ? __ldg(p + 2 * D) : 0.f;
    }
  };
  prefetch(b0);
  const float inv_code = s_code != 0.0f ? 1.0f / s_code : 0.0f;
  for (int b = b0; b < b1; ++b) {
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      qr[i * PP + t] = pq[i] * qm;
      ks[(CH + i) * PP + t] = pk[i] * kscale;
      vs[CH + i][t] = pv[i];
    }
    for (int i = t; i < CH * CTX; i += 128) wt[i / CTX][i % CTX] = 0.f;
    __syncthreads();
    if (b + 1 < b1) prefetch(b + 1);
    const int nq = min(CH, nr - b * CH);  // query rows of this block
    {
      const int qg = lane & 3, cg = lane >> 2;
      float acc[3][5];
#pragma unroll
      for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int c = 0; c < 5; ++c) acc[i][c] = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int d = warp * 32 + 4 * j;
        float4 x[3], y[5];
#pragma unroll
        for (int i = 0; i < 3; ++i) x[i] = *reinterpret_cast<const float4*>(&qr[(3 * qg + i) * PP + d]);
#pragma unroll
        for (int c = 0; c < 5; ++c) y[c] = *reinterpret_cast<const float4*>(&ks[(5 * cg + c) * PP + d]);
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
          for (int c = 0; c < 5; ++c) {
            acc[i][c] = fmaf(x[i].x, y[c].x, acc[i][c]);
            acc[i][c] = fmaf(x[i].y, y[c].y, acc[i][c]);
            acc[i][c] = fmaf(x[i].z, y[c].z, acc[i][c]);
            acc[i][c] = fmaf(x[i].w, y[c].w, acc[i][c]);
          }
      }
      __syncthreads();  // every warp is done reading the queries before they turn into red
      float* red = qr + warp * (CH * NB);
#pragma unroll
      for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int c = 0; c < 5; ++c) red[(3 * qg + i) * NB + 5 * cg + c] = acc[i][c];
    }
    __syncthreads();
    for (int qi = warp; qi < nq; qi += NW) {
      const int src = b * CH + lane - (CTX - CH);
      const bool kv_ok = lane < CTX && src >= 0 && src < nr;
      const int rel = lane - qi;
      const bool rel_ok = lane < CTX && rel >= 0 && rel < PL;
      float sc = -INFINITY;
      if (lane < CTX) {
        float p = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const float* red = qr + w * (CH * NB) + qi * NB;
          p += (kv_ok ? red[lane] : 0.f) + (rel_ok ? red[CTX + rel] : 0.f);
        }
        sc = tanhf(p / softcap) * softcap;
      }
      const float mx = warp_max_a(sc);
      const float e = lane < CTX ? expf(sc - mx) : 0.f;
      const float den = warp_sum_a(e);
      if (lane < CTX) wt[qi][lane] = kv_ok ? e / den : 0.f;  // out-of-clip slots add no value
    }
    __syncthreads();
    float acc[CH];  // the 12 rows' sums as independent chains (rows >= nq have zero weights)
#pragma unroll
    for (int qi = 0; qi < CH; ++qi) acc[qi] = 0.f;
#pragma unroll
    for (int c4 = 0; c4 < CTX / 4; ++c4) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = vs[4 * c4 + u][t];
#pragma unroll
      for (int qi = 0; qi < CH; ++qi) {
        const float4 w = *reinterpret_cast<const float4*>(&wt[qi][4 * c4]);
        acc[qi] = fmaf(w.x, v[0], acc[qi]);
        acc[qi] = fmaf(w.y, v[1], acc[qi]);
        acc[qi] = fmaf(w.z, v[2], acc[qi]);
        acc[qi] = fmaf(w.w, v[3], acc[qi]);
      }
    }
#pragma unroll
    for (int qi = 0; qi < CH; ++qi) {
      if (qi >= nq) break;
      const float o = acc[qi];
      const long oi = (r0 + b * CH + qi) * D + head * HD + t;
      if (s_code != 0.0f) {  // integer codes for the post projection's input scale
        o_hi[oi] = __float2half_rn(srq_code(o, s_code, inv_code));
      } else {
        __half h, l;
        split_f16(o, h, l);
        o_hi[oi] = h;
        o_lo[oi] = l;
      }
    }
    __syncthreads();  // every read of this block's window is done
#pragma unroll
    for (int i = 0; i < CH; ++i) {  // this block's keys and values become the next block's past (own column)
      ks[i * PP + t] = ks[(CH + i) * PP + t];
      vs[i][t] = vs[CH + i][t];
    }
  }
}

cudaError_t audio_attention_blocks(const float* qkv, const float* relk, const float* qmul, const int* run_clip,
                                   const int* run_blk0, int nruns, const int* row0, const int* rows, float kscale,
                                   float softcap, __half* o_hi, __half* o_lo, float s_code, cudaStream_t st) {
  if (nruns <= 0) return cudaSuccess;
  dim3 grid(nruns, 8);
  audio_attn_kernel<<<grid, 128, 0, st>>>(qkv, relk, qmul, run_clip, run_blk0, row0, rows, kscale, softcap, o_hi,
                                          o_lo, s_code);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Light-conv middle: causal depthwise conv (kernel 5, left pad 4) within the
// clip (runAudioDepthwiseCausalConv1dCpu, src/audio/kernels.ts:855-884),
// conv_norm RMSNorm, SiLU (runSiluActivationCpu) -> fp16 hi/lo operand of
// linear_end (integer codes when s_code, linear_end's input scale, is non-zero).
// Persistent blocks (two per SM, 256 threads) walk chunks of 8 packed rows.
// A chunk and its 4-row causal halo are 12 consecutive input rows, fetched by
// one thread as bulk copies into a double-buffered shared-memory ring, so the
// next chunk streams in while this one is computed:
//   conv     thread t owns channels [4t, 4t + 4): a 5-row register window
//            slides down the chunk; row i's result overwrites its own slot,
//            which no later row reads; per-row sums of squares meet in `red`
//   output   warp w takes row w: conv_norm, SiLU, operand planes
// Every wait is bounded; all threads agree on the outcome before going on.
// dw: [5][1024] (tap-major).
// ---------------------------------------------------------------------------
constexpr int kLcRows = 8, kLcHalo = 4, kLcWin = kLcRows + kLcHalo, kLcD = 1024;
constexpr int kLcStage = kLcWin * kLcD * 4;  // 48 KB
constexpr int kLcSmem = 2 * kLcStage;

__global__ void __launch_bounds__(256, 2) lconv_kernel(const float* __restrict__ g, const float* __restrict__ dw,
                                                       const float* __restrict__ nw, const int* __restrict__ row_clip,
                                                       const int* __restrict__ row0, long nrows, float eps,
                                                       __half* __restrict__ a_hi, __half* __restrict__ a_lo,
                                                       float s_code, int* err) {
  constexpr int D = kLcD, KS = kLcHalo + 1, R = kLcRows;
  extern __shared__ __align__(128) float lc_buf[];  // [2][12][1024]
  __shared__ __align__(8) uint64_t bar_full[2];
  __shared__ int first_tap[R];  // first tap whose source row lies inside the row's clip
  __shared__ __align__(16) float red[R][8];
  __shared__ int abort_flag, skip;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const long nchunks = (nrows + R - 1) / R;
  if (t == 0) {
    skip = *reinterpret_cast<volatile int*>(err) != 0;
    abort_flag = 0;
    mbar_init(&bar_full[0], 1);
    mbar_init(&bar_full[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (skip) return;  // an earlier kernel on this device already failed
  auto issue = [&](long chunk, int s) {
    const long first = chunk * R - kLcHalo;
    const long lo = first > 0 ? first : 0, hi = chunk * R + R < nrows ? chunk * R + R : nrows;
    float* dst = lc_buf + (long)s * kLcWin * D + (lo - first) * D;
    mbar_expect_tx(&bar_full[s], (uint32_t)((hi - lo) * D * 4));
    for (long r = lo; r < hi; ++r) bulk_load(dst + (r - lo) * D, g + r * D, D * 4, &bar_full[s]);
  };
  long issued = 0;
  if (t == 0) {
    for (int j = 0; j < 2; ++j) {
      const long c = blockIdx.x + (long)j * gridDim.x;
      if (c < nchunks) {
        issue(c, j);
        ++issued;
      }
    }
  }
  float4 w[KS], nv[8];
#pragma unroll
  for (int k = 0; k < KS; ++k) w[k] = __ldg(reinterpret_cast<const float4*>(dw + k * D) + t);
#pragma unroll
  for (int v = 0; v < 8; ++v) nv[v] = __ldg(reinterpret_cast<const float4*>(nw) + lane + 32 * v);
  const float inv_code = s_code != 0.0f ? 1.0f / s_code : 0.0f;
  long j = 0;
  for (long chunk = blockIdx.x; chunk < nchunks; chunk += gridDim.x, ++j) {
    const int s = (int)(j & 1);
    const long base = chunk * R;
    if (t < R) {
      const long r = base + t;
      const long local = r < nrows ? r - row0[row_clip[r]] : kLcHalo;
      first_tap[t] = local >= kLcHalo ? 0 : (int)(kLcHalo - local);
    }
    const bool got = mbar_wait(&bar_full[s], (uint32_t)((j >> 1) & 1), err, kErrWaitFull, &abort_flag);
    if (!__syncthreads_and(got)) break;
    float* B = lc_buf + (long)s * kLcWin * D;
    {
      float4 win[KS];
#pragma unroll
      for (int k = 0; k < KS - 1; ++k) win[k] = reinterpret_cast<const float4*>(B + k * D)[t];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        win[KS - 1] = reinterpret_cast<const float4*>(B + (i + KS - 1) * D)[t];
        const int k0 = first_tap[i];
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < KS; ++k) {
          if (k < k0) continue;
          acc.x = fmaf(win[k].x, w[k].x, acc.x);
          acc.y = fmaf(win[k].y, w[k].y, acc.y);
          acc.z = fmaf(win[k].z, w[k].z, acc.z);
          acc.w = fmaf(win[k].w, w[k].w, acc.w);
        }
        reinterpret_cast<float4*>(B + i * D)[t] = acc;
        const float ss = warp_sum_a(acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w);
        if (lane == 0) red[i][warp] = ss;
#pragma unroll
        for (int k = 0; k < KS - 1; ++k) win[k] = win[k + 1];
      }
    }
    __syncthreads();
    {
      const long row = base + warp;
      if (row < nrows) {
        const float4 p0 = *reinterpret_cast<const float4*>(&red[warp][0]);
        const float4 p1 = *reinterpret_cast<const float4*>(&red[warp][4]);
        const float tot = ((p0.x + p0.y) + (p0.z + p0.w)) + ((p1.x + p1.y) + (p1.z + p1.w));
        const float inv = 1.0f / sqrtf(tot / (float)D + eps);
        const float4* xr = reinterpret_cast<const float4*>(B + warp * D);
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float4 x = xr[lane + 32 * v];
          float u4[4] = {(x.x * inv) * nv[v].x, (x.y * inv) * nv[v].y, (x.z * inv) * nv[v].z, (x.w * inv) * nv[v].w};
          __align__(8) __half hh[4], ll[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float sv = u4[u] * sigmoid_f(u4[u]);
            if (s_code != 0.0f) hh[u] = __float2half_rn(srq_code(sv, s_code, inv_code));
            else split_f16(sv, hh[u], ll[u]);
          }
          const int c = 4 * (lane + 32 * v);
          *reinterpret_cast<uint2*>(a_hi + row * D + c) = *reinterpret_cast<uint2*>(hh);
          if (s_code == 0.0f) *reinterpret_cast<uint2*>(a_lo + row * D + c) = *reinterpret_cast<uint2*>(ll);
        }
      }
    }
    __syncthreads();  // the stage and `red` are free again
    if (t == 0) {
      const long nxt = chunk + 2L * gridDim.x;
      if (nxt < nchunks) {
        fence_proxy_async_smem();  // this CTA's generic writes to the stage come before the copy's
        issue(nxt, s);
        ++issued;
      }
    }
  }
  if (t == 0) {  // after an abort: wait (bounded) for copies still in flight before the CTA exits
    for (long q = j; q < issued; ++q) {
      const uint32_t b = smem_u32(&bar_full[q & 1]);
      const long long t0 = clock64();
      while (!mbar_try_wait(b, (uint32_t)((q >> 1) & 1))) {
        if (clock64() - t0 > kWaitCycles) {
          atomicCAS(err, 0, kErrWaitDrain);
          break;
        }
      }
    }
  }
}

cudaError_t audio_lconv_rows(const float* g, const float* dw, const float* nw, const int* row_clip, const int* row0,
                             long rows, float eps, __half* a_hi, __half* a_lo, float s_code, int* err,
                             cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  static bool attr_set[64] = {false};
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(lconv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kLcSmem);
    if (e != cudaSuccess) return e;
    cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (sms[dev] <= 0) sms[dev] = 148;
    attr_set[dev] = true;
  }
  const long chunks = (rows + kLcRows - 1) / kLcRows;
  const int grid = (int)(chunks < 2L * sms[dev] ? chunks : 2L * sms[dev]);
  lconv_kernel<<<grid, 256, kLcSmem, st>>>(g, dw, nw, row_clip, row0, rows, eps, a_hi, a_lo, s_code, err);
  return cudaGetLastError();
}

}  // namespace g4m
