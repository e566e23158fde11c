// Audio tower kernels: log-mel front end, chunked local self-attention and
// the light-conv depthwise block (the subsample convs are in
// subsample_sm100.cu).
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
// (512), magnitude, HTK mel filters (257 x 128), log(mel + 1e-3).  Frame f
// of a clip reads waveform samples [f*160 - 160, f*160 + 160) (160 leading
// zeros, frameLength / 2).
//
// One warp per frame, 8 frames per 256-thread CTA.  The 512 points live in
// registers, 16 per lane: butterfly stages of half-size 1..8 run inside a
// lane in the blocked layout (element 16 lane + j), half-size 16 pairs lanes
// lane ^ 1 through shuffles, a padded shared-memory transpose moves to the
// cyclic layout (element lane + 32 j), where half-sizes 32..256 again run
// inside a lane.  Every butterfly is fftRadix2's (src/preprocess/audio.ts:
// 191-212): double arithmetic from float inputs, without contraction, stored
// to float as its Float32Array is.
// ---------------------------------------------------------------------------
namespace {
__device__ __forceinline__ void fft_bfly(float& er, float& ei, float& odr, float& odi, double wr, double wi) {
  const double xr = odr, xi = odi;
  const double tr = __dsub_rn(__dmul_rn(xr, wr), __dmul_rn(xi, wi));
  const double ti = __dadd_rn(__dmul_rn(xr, wi), __dmul_rn(xi, wr));
  const double a = er, b = ei;
  odr = (float)__dsub_rn(a, tr);
  odi = (float)__dsub_rn(b, ti);
  er = (float)__dadd_rn(a, tr);
  ei = (float)__dadd_rn(b, ti);
}
}  // namespace

__global__ void __launch_bounds__(256) logmel_kernel(const float* __restrict__ samples, const long* __restrict__ soff,
                                                     const long* __restrict__ slen, const int* __restrict__ foff,
                                                     const int* __restrict__ fcount, int clips, int total_frames,
                                                     const float* __restrict__ window, const float* __restrict__ mel,
                                                     const int* __restrict__ mel_rng, const double2* __restrict__ tw,
                                                     float* __restrict__ feats) {
  constexpr int PADN = 512 + 32;  // one float2 of padding after every 16 elements
  __shared__ float2 xb[8][PADN];
  __shared__ float mg[8][260];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gf = blockIdx.x * 8 + warp;
  if (gf >= total_frames) return;  // warp-uniform: the kernel only synchronises within a warp
  int lo = 0, hi = clips - 1;      // clip of this frame: binary search over frame offsets
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (foff[mid] <= gf) lo = mid;
    else hi = mid - 1;
  }
  const int clip = lo, f = gf - foff[clip];
  if (f >= fcount[clip]) return;
  const float* x = samples + soff[clip];
  const long L = slen[clip];
  float re[16], im[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {  // element 16 lane + j holds input sample brev9(16 lane + j)
    const int n = __brev(16 * lane + j) >> 23;
    float v = 0.f;
    if (n < 320) {
      const long idx = (long)f * 160 + n - 160;
      if (idx >= 0 && idx < L) v = x[idx] * __ldg(window + n);
    }
    re[j] = v;
    im[j] = 0.f;
  }
#pragma unroll
  for (int st = 0; st < 4; ++st) {  // half-sizes 1, 2, 4, 8: partners in the same lane
    const int half = 1 << st, size = 2 << st;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j & half) continue;
      const double2 w = __ldg(tw + (j & (half - 1)) * (512 / size));  // offset in the group = j mod half
      fft_bfly(re[j], im[j], re[j + half], im[j + half], w.x, w.y);
    }
  }
  {  // half-size 16: element 16 lane + j pairs with lane ^ 1; odd lanes hold the upper members
    const bool upper = lane & 1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float pr = __shfl_xor_sync(0xffffffffu, re[j], 1), pim = __shfl_xor_sync(0xffffffffu, im[j], 1);
      const double2 w = __ldg(tw + j * 16);
      float er = upper ? pr : re[j], ei = upper ? pim : im[j];
      float odr = upper ? re[j] : pr, odi = upper ? im[j] : pim;
      fft_bfly(er, ei, odr, odi, w.x, w.y);
      re[j] = upper ? odr : er;
      im[j] = upper ? odi : ei;
    }
  }
  float2* xw = xb[warp];
#pragma unroll
  for (int j = 0; j < 16; ++j) xw[17 * lane + j] = make_float2(re[j], im[j]);  // p + p / 16, p = 16 lane + j
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 16; ++j) {  // element p = lane + 32 j
    const float2 v = xw[lane + 34 * j + (lane >> 4)];
    re[j] = v.x;
    im[j] = v.y;
  }
#pragma unroll
  for (int st = 5; st < 9; ++st) {  // half-sizes 32 .. 256: partners j and j + half / 32 in the same lane
    const int hj = 1 << (st - 5), half = 32 << (st - 5), size = 2 * half;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j & hj) continue;
      const int k = lane + 32 * (j & (hj - 1));  // (lane + 32 j) mod half
      const double2 w = __ldg(tw + k * (512 / size));
      fft_bfly(re[j], im[j], re[j + hj], im[j + hj], w.x, w.y);
    }
  }
  float* mw = mg[warp];
#pragma unroll
  for (int j = 0; j < 8; ++j) mw[lane + 32 * j] = (float)hypot((double)re[j], (double)im[j]);
  if (lane == 0) mw[256] = (float)hypot((double)re[8], (double)im[8]);
  __syncwarp();
  for (int m = lane; m < 128; m += 32) {
    double e = 0.0;  // mel energy in double (JS number), in bin order, over the non-zero bins
    const int b1 = mel_rng[2 * m + 1];
    for (int b = mel_rng[2 * m]; b <= b1; ++b) e = __dadd_rn(e, __dmul_rn((double)mw[b], (double)mel[b * 128 + m]));
    feats[(long)gf * 128 + m] = (float)log(e + 0.001);
  }
}

cudaError_t audio_logmel(const float* samples, const long* sample_off, const long* sample_len, const int* frame_off,
                         const int* frames, int clips, int total_frames, const float* window, const float* mel,
                         const int* mel_rng, const double2* twiddle, float* features, cudaStream_t st) {
  if (total_frames <= 0) return cudaSuccess;
  logmel_kernel<<<(total_frames + 7) / 8, 256, 0, st>>>(samples, sample_off, sample_len, frame_off, frames, clips,
                                                        total_frames, window, mel, mel_rng, twiddle, features);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Chunked local self-attention (runAudioSelfAttentionBodyCpu and
// audioSelfAttentionScore, src/audio/kernels.ts:432-512): chunk 12, context
// 24 (12 past-horizon rows), 13 relative positions, per-dim softplus query
// scale, tanh softcap.  Out-of-clip context rows add no key term and no
// value, but their slot stays in the softmax with the relative-only score.
// One CTA per (run of up to kAudioAttnRun consecutive 12-row blocks of one
// clip, head), 128 threads.  Both products run on the tensor cores as
// mma.sync m16n8k16 (f16 in, f32 accumulate) over split operands: every
// f32 value x is stored as hi = f16(x) and lo = f16((x - hi) 2^11), and
// x y = hi_x hi_y + 2^-11 (hi_x lo_y + lo_x hi_y) to ~22 bits, the scaled
// residual never entering the f16 subnormal range.
//   stage    the block's 12 query / key / value rows are prefetched into
//            registers (thread = head dim) while the previous block computes;
//            keys and values go to a two-slot ring (the previous block's rows
//            stay in the other slot), values transposed [dim][slot row]; the
//            13 relative keys are staged once per CTA
//   scores   [12 (16) queries] x [24 keys | 13 relative keys | 3 zero] over
//            128 dims: warp w takes dims [32w, 32w + 32); partial sums meet in
//            the softmax
//   softmax  one warp per query row, lane = context slot: tanh softcap, max,
//            exp, sum; weights of out-of-clip slots kept in the denominator;
//            P written as hi / lo planes in ring order
//   P*V      [16 x 32 ring slots] x [32 x 128]: warp w takes dims [32w, +32);
//            its output rows pass through a staging block in the (by then
//            free) query region and leave as 64 contiguous bytes per row
// qkv: [rows][3 * 1024] f32 (q | k | v); relk: [13][1024]; qmul: [128]
// (= 128^-0.5 / ln 2 * softplus(per_dim_scale)); kscale = ln(1 + e) / ln 2.
// ---------------------------------------------------------------------------
namespace {
constexpr int kAtQP = 136;  // halves per query / key row (68 words: fragment loads hit 32 distinct banks)
constexpr int kAtVP = 40;   // halves per transposed value row and per P row (20 words)
constexpr int kAtQBytes = 2 * 16 * kAtQP * 2;       // Qh, Ql [16][136]
constexpr int kAtRedBytes = 4 * 12 * 40 * 4;        // red [4 warps][12][40] f32, aliases the queries
constexpr int kAtKBytes = 2 * 40 * kAtQP * 2;       // Kh, Kl [40][136]
constexpr int kAtVBytes = 2 * 128 * kAtVP * 2;      // Vth, Vtl [128][40]
constexpr int kAtPBytes = 2 * 16 * kAtVP * 2;       // Ph, Pl [16][40]
constexpr int kAtSmem = (kAtQBytes > kAtRedBytes ? kAtQBytes : kAtRedBytes) + kAtKBytes + kAtVBytes + kAtPBytes;
constexpr float kLoScale = 2048.0f, kLoInv = 1.0f / 2048.0f;

__device__ __forceinline__ void split_scaled(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn((x - __half2float(hi)) * kLoScale);
}

// tanh(x) = sign(x) (1 - 2 / (2^(2 |x| log2 e) + 1)), absolute error ~1e-7;
// saturates to +-1 without overflow.
__device__ __forceinline__ float tanh_f(float x) {
  const float e = ex2_approx(2.0f * kLog2eF * fabsf(x));
  return copysignf(1.0f - 2.0f * rcp_approx(e + 1.0f), x);
}

__device__ __forceinline__ uint32_t ld_h2(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }

__device__ __forceinline__ void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
}  // namespace

__global__ void __launch_bounds__(128, 4) audio_attn_kernel(const float* __restrict__ qkv,
                                                            const float* __restrict__ relk,
                                                            const float* __restrict__ qmul,
                                                            const int* __restrict__ run_clip,
                                                            const int* __restrict__ run_blk0,
                                                            const int* __restrict__ row0, const int* __restrict__ rows,
                                                            float kscale, float softcap, __half* __restrict__ o_hi,
                                                            __half* __restrict__ o_lo, float s_code) {
  constexpr int HD = 128, CH = 12, CTX = 24, PL = 13, NB = 40, D = 1024, NW = 4;
  extern __shared__ __align__(16) uint8_t at_smem[];
  __half* Qh = reinterpret_cast<__half*>(at_smem);
  __half* Ql = Qh + 16 * kAtQP;
  float* red = reinterpret_cast<float*>(at_smem);  // [NW][CH][NB], after the score MMAs
  uint8_t* p8 = at_smem + (kAtQBytes > kAtRedBytes ? kAtQBytes : kAtRedBytes);
  __half* Kh = reinterpret_cast<__half*>(p8);  // rows: ring slots [0, 24), relative keys [24, 37), zero [37, 40)
  __half* Kl = Kh + 40 * kAtQP;
  __half* Vth = Kl + 40 * kAtQP;  // [dim][ring slot], slots [24, 40) zero
  __half* Vtl = Vth + 128 * kAtVP;
  __half* Ph = Vtl + 128 * kAtVP;  // [query][ring slot]
  __half* Pl = Ph + 16 * kAtVP;

  const int head = blockIdx.y;
  const int clip = run_clip[blockIdx.x], b0 = run_blk0[blockIdx.x];
  const long r0 = row0[clip];
  const int nr = rows[clip];
  const int b1 = min(b0 + kAudioAttnRun, (nr + CH - 1) / CH);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const __half hz = __float2half_rn(0.f);
  // zero what no block writes: query rows 12..15, key rows 37..39, P, the value slots 24..39
  for (int i = t; i < 2 * 4 * kAtQP; i += 128) (i < 4 * kAtQP ? Qh : Ql)[12 * kAtQP + (i % (4 * kAtQP))] = hz;
  for (int i = t; i < 2 * 3 * kAtQP; i += 128) (i < 3 * kAtQP ? Kh : Kl)[37 * kAtQP + (i % (3 * kAtQP))] = hz;
  for (int i = t; i < 2 * 16 * kAtVP; i += 128) Ph[i] = hz;  // Ph and Pl are contiguous
  for (int i = t; i < 2 * 128 * kAtVP; i += 128) Vth[i] = hz;  // Vth and Vtl are contiguous
  __syncthreads();
  const float qm = qmul[t];
  const float* col = qkv + r0 * (3 * D) + head * HD + t;  // this thread's dim of row 0's q
#pragma unroll
  for (int r = 0; r < PL; ++r) {
    __half h, l;
    split_scaled(__ldg(relk + r * D + head * HD + t), h, l);
    Kh[(CTX + r) * kAtQP + t] = h;
    Kl[(CTX + r) * kAtQP + t] = l;
  }
  {  // the past window of block b0 (rows of block b0 - 1; none before row 0) in the slot block b0 does not use
    const int slot = 12 * (1 - (b0 & 1));
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int src = b0 * CH - CH + c;
      const bool ok = src >= 0;
      __half h, l;
      split_scaled(ok ? __ldg(col + (long)src * (3 * D) + D) * kscale : 0.f, h, l);
      Kh[(slot + c) * kAtQP + t] = h;
      Kl[(slot + c) * kAtQP + t] = l;
      split_scaled(ok ? __ldg(col + (long)src * (3 * D) + 2 * D) : 0.f, h, l);
      Vth[t * kAtVP + slot + c] = h;
      Vtl[t * kAtVP + slot + c] = l;
    }
  }
  float pq[CH], pk[CH], pv[CH];  // the next block's rows, in flight while the current one computes
  auto prefetch = [&](int b) {
    const float* p = col + (long)(b * CH) * (3 * D);  // row b * 12; rows i at constant offsets
    const int n = nr - b * CH;                        // rows of block b inside the clip
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      pq[i] = pk[i] = pv[i] = 0.f;
      if (i < n) {
        pq[i] = __ldg(p + i * (3 * D));
        pk[i] = __ldg(p + i * (3 * D) + D);
        pv[i] = __ldg(p + i * (3 * D) + 2 * D);
      }
    }
  };
  prefetch(b0);
  const float inv_code = s_code != 0.0f ? 1.0f / s_code : 0.0f;
  const float inv_cap = 1.0f / softcap;
  for (int b = b0; b < b1; ++b) {
    const int cur = 12 * (b & 1), prev = 12 - cur;  // ring slots of this block's rows and of the past window
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      __half h, l;
      split_scaled(pq[i] * qm, h, l);
      Qh[i * kAtQP + t] = h;
      Ql[i * kAtQP + t] = l;
      split_scaled(pk[i] * kscale, h, l);
      Kh[(cur + i) * kAtQP + t] = h;
      Kl[(cur + i) * kAtQP + t] = l;
    }
#pragma unroll
    for (int i = 0; i < CH; i += 2) {
      const __half2 h2 = __floats2half2_rn(pv[i], pv[i + 1]);
      const float2 back = __half22float2(h2);
      *reinterpret_cast<__half2*>(Vth + t * kAtVP + cur + i) = h2;
      *reinterpret_cast<__half2*>(Vtl + t * kAtVP + cur + i) =
          __floats2half2_rn((pv[i] - back.x) * kLoScale, (pv[i + 1] - back.y) * kLoScale);
    }
    __syncthreads();
    if (b + 1 < b1) prefetch(b + 1);
    const int nq = min(CH, nr - b * CH);  // query rows of this block
    {
      // scores: context slot c -> key row (c < 12: past window, c < 24: this block, else relative / zero)
      int krow[5];
#pragma unroll
      for (int nt = 0; nt < 5; ++nt) {
        const int c = nt * 8 + g;
        krow[nt] = c < CH ? prev + c : (c < CTX ? cur + c - CH : c);
      }
      float hh[5][4], xx[5][4];
#pragma unroll
      for (int nt = 0; nt < 5; ++nt)
#pragma unroll
        for (int u = 0; u < 4; ++u) hh[nt][u] = xx[nt][u] = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kb = warp * 32 + 16 * j + 2 * tig;
        uint32_t ah[4], al[4];
        ah[0] = ld_h2(Qh + g * kAtQP + kb);
        ah[1] = ld_h2(Qh + (g + 8) * kAtQP + kb);
        ah[2] = ld_h2(Qh + g * kAtQP + kb + 8);
        ah[3] = ld_h2(Qh + (g + 8) * kAtQP + kb + 8);
        al[0] = ld_h2(Ql + g * kAtQP + kb);
        al[1] = ld_h2(Ql + (g + 8) * kAtQP + kb);
        al[2] = ld_h2(Ql + g * kAtQP + kb + 8);
        al[3] = ld_h2(Ql + (g + 8) * kAtQP + kb + 8);
#pragma unroll
        for (int nt = 0; nt < 5; ++nt) {
          const __half* kh = Kh + krow[nt] * kAtQP + kb;
          const __half* kl = Kl + krow[nt] * kAtQP + kb;
          const uint32_t bh0 = ld_h2(kh), bh1 = ld_h2(kh + 8), bl0 = ld_h2(kl), bl1 = ld_h2(kl + 8);
          mma_16816(hh[nt], ah, bh0, bh1);
          mma_16816(xx[nt], ah, bl0, bl1);
          mma_16816(xx[nt], al, bh0, bh1);
        }
      }
      __syncthreads();  // every warp is done reading the queries before they turn into red
      float* rw = red + warp * (CH * NB);
#pragma unroll
      for (int nt = 0; nt < 5; ++nt) {
        const int cc = nt * 8 + 2 * tig;
        *reinterpret_cast<float2*>(rw + g * NB + cc) =
            make_float2(fmaf(xx[nt][0], kLoInv, hh[nt][0]), fmaf(xx[nt][1], kLoInv, hh[nt][1]));
        if (g + 8 < CH)
          *reinterpret_cast<float2*>(rw + (g + 8) * NB + cc) =
              make_float2(fmaf(xx[nt][2], kLoInv, hh[nt][2]), fmaf(xx[nt][3], kLoInv, hh[nt][3]));
      }
    }
    __syncthreads();
    for (int qi = warp; qi < CH; qi += NW) {
      const int src = b * CH + lane - (CTX - CH);
      const bool kv_ok = lane < CTX && src >= 0 && src < nr;
      const int rel = lane - qi;
      const bool rel_ok = lane < CTX && rel >= 0 && rel < PL;
      float sc = -INFINITY;
      if (lane < CTX && qi < nq) {
        float p = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
          const float* rr = red + w * (CH * NB) + qi * NB;
          p += (kv_ok ? rr[lane] : 0.f) + (rel_ok ? rr[CTX + rel] : 0.f);
        }
        sc = tanh_f(p * inv_cap) * softcap;
      }
      const float mx = warp_max_a(sc);
      const float e = (lane < CTX && qi < nq) ? ex2_approx((sc - mx) * kLog2eF) : 0.f;
      const float inv_den = rcp_approx(warp_sum_a(e));
      if (lane < CTX) {
        // out-of-clip slots add no value; rows past the clip end get zero weights
        const float wgt = (kv_ok && qi < nq) ? e * inv_den : 0.f;
        const int slot = lane < CH ? prev + lane : cur + lane - CH;
        __half h, l;
        split_scaled(wgt, h, l);
        Ph[qi * kAtVP + slot] = h;
        Pl[qi * kAtVP + slot] = l;
      }
    }
    __syncthreads();
    {
      float oh[4][4], ox[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n)
#pragma unroll
        for (int u = 0; u < 4; ++u) oh[n][u] = ox[n][u] = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kb = 16 * j + 2 * tig;
        uint32_t ah[4], al[4];
        ah[0] = ld_h2(Ph + g * kAtVP + kb);
        ah[1] = ld_h2(Ph + (g + 8) * kAtVP + kb);
        ah[2] = ld_h2(Ph + g * kAtVP + kb + 8);
        ah[3] = ld_h2(Ph + (g + 8) * kAtVP + kb + 8);
        al[0] = ld_h2(Pl + g * kAtVP + kb);
        al[1] = ld_h2(Pl + (g + 8) * kAtVP + kb);
        al[2] = ld_h2(Pl + g * kAtVP + kb + 8);
        al[3] = ld_h2(Pl + (g + 8) * kAtVP + kb + 8);
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int dim = warp * 32 + n * 8 + g;
          const __half* vh = Vth + dim * kAtVP + kb;
          const __half* vl = Vtl + dim * kAtVP + kb;
          const uint32_t bh0 = ld_h2(vh), bh1 = ld_h2(vh + 8), bl0 = ld_h2(vl), bl1 = ld_h2(vl + 8);
          mma_16816(oh[n], ah, bh0, bh1);
          mma_16816(ox[n], ah, bl0, bl1);
          mma_16816(ox[n], al, bh0, bh1);
        }
      }
      // The fragments (16 bytes of each of 8 rows per store) go through the
      // warp's 2 KB of the query region (free until the next block's
      // install) as [16 rows][64 B] hi and lo planes, 16-byte chunks
      // XOR-swizzled by row pair, and leave as 64 contiguous bytes per row.
      uint32_t* sth = reinterpret_cast<uint32_t*>(at_smem + warp * 2048);
      uint32_t* stl = sth + 256;
#pragma unroll
      for (int n = 0; n < 4; ++n) {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int qi = g + 8 * half;
          const float o0 = fmaf(ox[n][2 * half], kLoInv, oh[n][2 * half]);
          const float o1 = fmaf(ox[n][2 * half + 1], kLoInv, oh[n][2 * half + 1]);
          const int wd = qi * 16 + 4 * (n ^ ((qi >> 1) & 3)) + tig;
          if (s_code != 0.0f) {  // integer codes for the post projection's input scale
            union {
              __half2 h2;
              uint32_t w;
            } cv;
            cv.h2 = __halves2half2(__float2half_rn(srq_code(o0, s_code, inv_code)),
                                   __float2half_rn(srq_code(o1, s_code, inv_code)));
            sth[wd] = cv.w;
          } else {
            uint32_t hv, lv;
            split2_f16(o0, o1, hv, lv);
            sth[wd] = hv;
            stl[wd] = lv;
          }
        }
      }
      __syncwarp();
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int qi = 8 * k + (lane >> 2), c = lane & 3;
        if (qi < nq) {
          const int wd = qi * 16 + 4 * (c ^ ((qi >> 1) & 3));
          const long oi = (r0 + b * CH + qi) * D + head * HD + warp * 32 + c * 8;
          if (s_code != 0.0f) {
            // the staged codes (small integers, exact in fp16) leave as signed
            // bytes: 8 per lane, D bytes per row
            const uint4 hw = *reinterpret_cast<const uint4*>(sth + wd);
            const uint32_t src[4] = {hw.x, hw.y, hw.z, hw.w};
            uint32_t by[2] = {0, 0};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const __half hv = __ushort_as_half((unsigned short)(src[e >> 1] >> (16 * (e & 1))));
              by[e >> 2] |= ((uint32_t)(int)__half2float(hv) & 0xFFu) << (8 * (e & 3));
            }
            *reinterpret_cast<uint2*>(reinterpret_cast<char*>(o_hi) + oi) = make_uint2(by[0], by[1]);
          } else {
            *reinterpret_cast<uint4*>(o_hi + oi) = *reinterpret_cast<const uint4*>(sth + wd);
            *reinterpret_cast<uint4*>(o_lo + oi) = *reinterpret_cast<const uint4*>(stl + wd);
          }
        }
      }
    }
    __syncthreads();  // P and the value ring are free for the next block
  }
}

cudaError_t audio_attention_blocks(const float* qkv, const float* relk, const float* qmul, const int* run_clip,
                                   const int* run_blk0, int nruns, const int* row0, const int* rows, float kscale,
                                   float softcap, __half* o_hi, __half* o_lo, float s_code, cudaStream_t st) {
  if (nruns <= 0) return cudaSuccess;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(audio_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmem);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  dim3 grid(nruns, 8);
  audio_attn_kernel<<<grid, 128, kAtSmem, st>>>(qkv, relk, qmul, run_clip, run_blk0, row0, rows, kscale, softcap, o_hi,
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
          uint32_t codes = 0;  // signed-byte codes for linear_end's input scale (D bytes per row)
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float sv = u4[u] * sigmoid_f(u4[u]);
            if (s_code != 0.0f) codes |= ((uint32_t)(int)srq_code(sv, s_code, inv_code) & 0xFFu) << (8 * u);
            else split_f16(sv, hh[u], ll[u]);
          }
          const int c = 4 * (lane + 32 * v);
          if (s_code != 0.0f) {
            *reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(a_hi) + row * D + c) = codes;
          } else {
            *reinterpret_cast<uint2*>(a_hi + row * D + c) = *reinterpret_cast<uint2*>(hh);
            *reinterpret_cast<uint2*>(a_lo + row * D + c) = *reinterpret_cast<uint2*>(ll);
          }
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
