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
//            registers as float4 (warp w: rows w, w + 4, w + 8; lane: 4
//            dims) while the previous block computes, then split into 8-byte
//            hi / lo pieces; keys and values go to a two-slot ring (the
//            previous block's rows stay in the other slot), both row-major;
//            the 13 relative keys are staged once per CTA
//   scores   [12 (16) queries] x [24 keys | 13 relative keys | 3 zero] over
//            128 dims: warp w takes dims [32w, 32w + 32), fragments by
//            ldmatrix; partial sums meet in the softmax
//   softmax  warp w takes query rows w, w + 4, w + 8 together (three
//            interleaved reduction chains), lane = context slot: tanh
//            softcap, max, exp, sum; weights of out-of-clip slots kept in the
//            denominator; P written as hi / lo planes in ring order
//   P*V      [16 x 32 ring slots] x [32 x 128]: warp w takes dims [32w, +32),
//            value fragments by ldmatrix.trans from the row-major ring; its
//            output rows pass through a staging block in the (by then free)
//            query region and leave as 64 contiguous bytes per row
// qkv: [rows][3 * 1024] f32 (q | k | v); relk: [13][1024]; qmul: [128]
// (= 128^-0.5 / ln 2 * softplus(per_dim_scale)); kscale = ln(1 + e) / ln 2.
// ---------------------------------------------------------------------------
namespace {
constexpr int kAtQP = 136;  // halves per query / key / value row (68 words: ldmatrix rows hit distinct banks)
constexpr int kAtPP = 40;   // halves per P row (20 words)
constexpr int kAtQBytes = 2 * 16 * kAtQP * 2;       // Qh, Ql [16][136]
constexpr int kAtRedBytes = 4 * 12 * 40 * 4;        // red [4 warps][12][40] f32, aliases the queries
constexpr int kAtKBytes = 2 * 40 * kAtQP * 2;       // Kh, Kl [40][136]
constexpr int kAtVBytes = 2 * 32 * kAtQP * 2;       // Vh, Vl [32 ring slots][136]
constexpr int kAtPBytes = 2 * 16 * kAtPP * 2;       // Ph, Pl [16][40]
constexpr int kAtSmem = (kAtQBytes > kAtRedBytes ? kAtQBytes : kAtRedBytes) + kAtKBytes + kAtVBytes + kAtPBytes;
constexpr float kLoScale = 2048.0f, kLoInv = 1.0f / 2048.0f;

__device__ __forceinline__ void split_scaled(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn((x - __half2float(hi)) * kLoScale);
}

// four values as 8-byte hi and scaled-lo pieces (split_scaled per element)
__device__ __forceinline__ void split4_scaled(float4 v, uint2& hi, uint2& lo) {
  union {
    __half2 h2;
    uint32_t w;
  } h01, h23, l01, l23;
  h01.h2 = __floats2half2_rn(v.x, v.y);
  h23.h2 = __floats2half2_rn(v.z, v.w);
  const float2 b01 = __half22float2(h01.h2), b23 = __half22float2(h23.h2);
  l01.h2 = __floats2half2_rn((v.x - b01.x) * kLoScale, (v.y - b01.y) * kLoScale);
  l23.h2 = __floats2half2_rn((v.z - b23.x) * kLoScale, (v.w - b23.y) * kLoScale);
  hi = make_uint2(h01.w, h23.w);
  lo = make_uint2(l01.w, l23.w);
}

// tanh(x) = sign(x) (1 - 2 / (2^(2 |x| log2 e) + 1)), absolute error ~1e-7;
// saturates to +-1 without overflow.
__device__ __forceinline__ float tanh_f(float x) {
  const float e = ex2_approx(2.0f * kLog2eF * fabsf(x));
  return copysignf(1.0f - 2.0f * rcp_approx(e + 1.0f), x);
}

__device__ __forceinline__ void ldsm_x4(const __half* p, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p))
               : "memory");
}
__device__ __forceinline__ void ldsm_x2(const __half* p, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p))
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(const __half* p, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p))
               : "memory");
}

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
  __half* Vh = Kl + 40 * kAtQP;  // [ring slot][dim], slots [24, 32) zero
  __half* Vl = Vh + 32 * kAtQP;
  __half* Ph = Vl + 32 * kAtQP;  // [query][ring slot]
  __half* Pl = Ph + 16 * kAtPP;

  const int head = blockIdx.y;
  const int clip = run_clip[blockIdx.x], b0 = run_blk0[blockIdx.x];
  const long r0 = row0[clip];
  const int nr = rows[clip];
  const int b1 = min(b0 + kAudioAttnRun, (nr + CH - 1) / CH);
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int g = lane >> 2, tig = lane & 3;
  const __half hz = __float2half_rn(0.f);
  // zero what no block writes: query rows 12..15, key rows 37..39, P, the value slots 24..31
  for (int i = t; i < 2 * 4 * kAtQP; i += 128) (i < 4 * kAtQP ? Qh : Ql)[12 * kAtQP + (i % (4 * kAtQP))] = hz;
  for (int i = t; i < 2 * 3 * kAtQP; i += 128) (i < 3 * kAtQP ? Kh : Kl)[37 * kAtQP + (i % (3 * kAtQP))] = hz;
  for (int i = t; i < 2 * 16 * kAtPP; i += 128) Ph[i] = hz;  // Ph and Pl are contiguous
  for (int i = t; i < 2 * 8 * kAtQP; i += 128) (i < 8 * kAtQP ? Vh : Vl)[24 * kAtQP + (i % (8 * kAtQP))] = hz;
  const float4 qm = __ldg(reinterpret_cast<const float4*>(qmul) + lane);
  // this lane's 4 dims of row 0's q; rows at constant offsets
  const float* col = qkv + r0 * (3 * D) + head * HD + 4 * lane;
  auto put = [&](__half* hi_plane, __half* lo_plane, int row, float4 v) {
    uint2 h, l;
    split4_scaled(v, h, l);
    *reinterpret_cast<uint2*>(hi_plane + row * kAtQP + 4 * lane) = h;
    *reinterpret_cast<uint2*>(lo_plane + row * kAtQP + 4 * lane) = l;
  };
  for (int r = warp; r < PL; r += NW)
    put(Kh, Kl, CTX + r, __ldg(reinterpret_cast<const float4*>(relk + r * D + head * HD) + lane));
  {  // the past window of block b0 (rows of block b0 - 1; none before row 0) in the slot block b0 does not use
    const int slot = 12 * (1 - (b0 & 1));
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int c = warp + NW * u;
      const int src = b0 * CH - CH + c;
      const bool ok = src >= 0;
      float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
      if (ok) {
        k = __ldg(reinterpret_cast<const float4*>(col + (long)src * (3 * D) + D));
        v = __ldg(reinterpret_cast<const float4*>(col + (long)src * (3 * D) + 2 * D));
      }
      put(Kh, Kl, slot + c, make_float4(k.x * kscale, k.y * kscale, k.z * kscale, k.w * kscale));
      put(Vh, Vl, slot + c, v);
    }
  }
  float4 pq[3], pk[3], pv[3];  // the next block's rows, in flight while the current one computes
  auto prefetch = [&](int b) {
    const float* p = col + (long)(b * CH) * (3 * D);  // row b * 12
    const int n = nr - b * CH;                        // rows of block b inside the clip
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int i = warp + NW * u;
      pq[u] = pk[u] = pv[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < n) {
        pq[u] = __ldg(reinterpret_cast<const float4*>(p + i * (3 * D)));
        pk[u] = __ldg(reinterpret_cast<const float4*>(p + i * (3 * D) + D));
        pv[u] = __ldg(reinterpret_cast<const float4*>(p + i * (3 * D) + 2 * D));
      }
    }
  };
  prefetch(b0);
  const float inv_code = s_code != 0.0f ? 1.0f / s_code : 0.0f;
  const float inv_cap = 1.0f / softcap;
  // ldmatrix row / column of this lane within a 16 x 16 fragment
  const int lr = (lane & 7) + 8 * ((lane >> 3) & 1), lc = 8 * (lane >> 4);
  for (int b = b0; b < b1; ++b) {
    const int cur = 12 * (b & 1), prev = 12 - cur;  // ring slots of this block's rows and of the past window
    __syncthreads();  // the previous block is done with the query region, P and its ring slot
#pragma unroll
    for (int u = 0; u < 3; ++u) {
      const int i = warp + NW * u;
      put(Qh, Ql, i, make_float4(pq[u].x * qm.x, pq[u].y * qm.y, pq[u].z * qm.z, pq[u].w * qm.w));
      put(Kh, Kl, cur + i, make_float4(pk[u].x * kscale, pk[u].y * kscale, pk[u].z * kscale, pk[u].w * kscale));
      put(Vh, Vl, cur + i, pv[u]);
    }
    __syncthreads();
    if (b + 1 < b1) prefetch(b + 1);
    const int nq = min(CH, nr - b * CH);  // query rows of this block
    {
      // scores: context slot c -> key row (c < 12: past window, c < 24: this block, else relative / zero).
      // ldmatrix row addresses: key tiles {0, 1} and {2, 3} as x4 (lanes 16..31 the second tile), tile 4 as x2
      auto krow = [&](int c) { return c < CH ? prev + c : (c < CTX ? cur + c - CH : c); };
      const int kr01 = krow((lane >> 4) * 8 + (lane & 7)), kr23 = krow(16 + (lane >> 4) * 8 + (lane & 7));
      const int kr4 = krow(32 + (lane & 7));
      const int kc = 8 * ((lane >> 3) & 1);  // b0 / b1 half of the 16 dims
      float hh[5][4], xx[5][4];
#pragma unroll
      for (int nt = 0; nt < 5; ++nt)
#pragma unroll
        for (int u = 0; u < 4; ++u) hh[nt][u] = xx[nt][u] = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int kb = warp * 32 + 16 * j;
        uint32_t ah[4], al[4], bh[5][2], bl[5][2];
        ldsm_x4(Qh + lr * kAtQP + kb + lc, ah);
        ldsm_x4(Ql + lr * kAtQP + kb + lc, al);
        {
          uint32_t r[4];
          ldsm_x4(Kh + kr01 * kAtQP + kb + kc, r);
          bh[0][0] = r[0], bh[0][1] = r[1], bh[1][0] = r[2], bh[1][1] = r[3];
          ldsm_x4(Kl + kr01 * kAtQP + kb + kc, r);
          bl[0][0] = r[0], bl[0][1] = r[1], bl[1][0] = r[2], bl[1][1] = r[3];
          ldsm_x4(Kh + kr23 * kAtQP + kb + kc, r);
          bh[2][0] = r[0], bh[2][1] = r[1], bh[3][0] = r[2], bh[3][1] = r[3];
          ldsm_x4(Kl + kr23 * kAtQP + kb + kc, r);
          bl[2][0] = r[0], bl[2][1] = r[1], bl[3][0] = r[2], bl[3][1] = r[3];
          ldsm_x2(Kh + kr4 * kAtQP + kb + kc, bh[4]);
          ldsm_x2(Kl + kr4 * kAtQP + kb + kc, bl[4]);
        }
#pragma unroll
        for (int nt = 0; nt < 5; ++nt) {
          mma_16816(hh[nt], ah, bh[nt][0], bh[nt][1]);
          mma_16816(xx[nt], ah, bl[nt][0], bl[nt][1]);
          mma_16816(xx[nt], al, bh[nt][0], bh[nt][1]);
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
    {
      // query rows warp, warp + 4, warp + 8 side by side
      const int src = b * CH + lane - (CTX - CH);
      const bool kv_ok = lane < CTX && src >= 0 && src < nr;
      float sc[3], mx[3], e[3], den[3];
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        const int qi = warp + NW * u;
        const int rel = lane - qi;
        const bool rel_ok = lane < CTX && rel >= 0 && rel < PL;
        sc[u] = -INFINITY;
        if (lane < CTX && qi < nq) {
          float p = 0.f;
#pragma unroll
          for (int w = 0; w < NW; ++w) {
            const float* rr = red + w * (CH * NB) + qi * NB;
            p += (kv_ok ? rr[lane] : 0.f) + (rel_ok ? rr[CTX + rel] : 0.f);
          }
          sc[u] = tanh_f(p * inv_cap) * softcap;
        }
        mx[u] = sc[u];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < 3; ++u) mx[u] = fmaxf(mx[u], __shfl_xor_sync(0xffffffffu, mx[u], o));
#pragma unroll
      for (int u = 0; u < 3; ++u) {
        e[u] = (lane < CTX && warp + NW * u < nq) ? ex2_approx((sc[u] - mx[u]) * kLog2eF) : 0.f;
        den[u] = e[u];
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int u = 0; u < 3; ++u) den[u] += __shfl_xor_sync(0xffffffffu, den[u], o);
      if (lane < CTX) {
        const int slot = lane < CH ? prev + lane : cur + lane - CH;
#pragma unroll
        for (int u = 0; u < 3; ++u) {
          const int qi = warp + NW * u;
          // out-of-clip slots add no value; rows past the clip end get zero weights
          const float wgt = (kv_ok && qi < nq) ? e[u] * rcp_approx(den[u]) : 0.f;
          __half h, l;
          split_scaled(wgt, h, l);
          Ph[qi * kAtPP + slot] = h;
          Pl[qi * kAtPP + slot] = l;
        }
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
        uint32_t ah[4], al[4];
        ldsm_x4(Ph + lr * kAtPP + 16 * j + lc, ah);
        ldsm_x4(Pl + lr * kAtPP + 16 * j + lc, al);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          // value tiles: slots [16 j, +16) x dims [32 warp + 16 p, +16); lanes 16..31 the second dim tile
          const int vr = 16 * j + lr, vc = warp * 32 + 16 * p + lc;
          uint32_t vh[4], vl[4];
          ldsm_x4_t(Vh + vr * kAtQP + vc, vh);
          ldsm_x4_t(Vl + vr * kAtQP + vc, vl);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int n = 2 * p + h;
            mma_16816(oh[n], ah, vh[2 * h], vh[2 * h + 1]);
            mma_16816(ox[n], ah, vl[2 * h], vl[2 * h + 1]);
            mma_16816(ox[n], al, vh[2 * h], vh[2 * h + 1]);
          }
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
            const uint32_t srcw[4] = {hw.x, hw.y, hw.z, hw.w};
            uint32_t by[2] = {0, 0};
#pragma unroll
            for (int e2 = 0; e2 < 8; ++e2) {
              const __half hv = __ushort_as_half((unsigned short)(srcw[e2 >> 1] >> (16 * (e2 & 1))));
              by[e2 >> 2] |= ((uint32_t)(int)__half2float(hv) & 0xFFu) << (8 * (e2 & 3));
            }
            *reinterpret_cast<uint2*>(reinterpret_cast<char*>(o_hi) + oi) = make_uint2(by[0], by[1]);
          } else {
            *reinterpret_cast<uint4*>(o_hi + oi) = *reinterpret_cast<const uint4*>(sth + wd);
            *reinterpret_cast<uint4*>(o_lo + oi) = *reinterpret_cast<const uint4*>(stl + wd);
          }
        }
      }
    }
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
// Each CTA (256 threads, two per SM) streams one contiguous range of packed
// rows.  Thread t owns channels [4t, 4t + 4) for the whole range:
//   ring     one thread keeps kLcSlots groups of kLcG rows in flight as bulk
//            copies (no multicast) into a shared-memory ring
//   conv     the 4 rows before the current one stay in registers (a sliding
//            window), so every input row is read from HBM once; a tap whose
//            source row lies in another clip (clip ids slide with the window)
//            contributes zero
//   norm     per-row sums of squares: a reduce-scatter over the warp's lanes
//            (6 shuffles for the group's kLcG rows), then one CTA barrier per
//            group through a double-buffered [kLcG][8 warps] table; the same
//            barrier releases the group's ring slot
//   output   conv_norm, SiLU and the operand planes from the thread's own
//            registers: every row leaves as 8 contiguous bytes per thread
// Every wait is bounded; all threads agree on the outcome before going on.
// dw: [5][1024] (tap-major).
// ---------------------------------------------------------------------------
constexpr int kLcG = 8, kLcSlots = 3, kLcHalo = 4, kLcD = 1024;  // 32 KB slots, 96 KB per CTA
constexpr int kLcSlotBytes = kLcG * kLcD * 4;

// Reduce-scatter of G per-lane values over the warp: each halving step keeps
// half of the values and sends the other half to the partner lane (xor 16,
// 8, ...), then plain butterflies finish; lane l returns the warp total of
// value l / (32 / G), with the same pairings as a butterfly all-reduce of
// each value.
template <int G>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[G], int lane) {
  static_assert(G == 2 || G == 4 || G == 8 || G == 16, "G: a power of two up to 16");
#pragma unroll
  for (int h = G / 2, m = 16; h >= 1; h /= 2, m /= 2) {
    const bool up = (lane & m) != 0;
#pragma unroll
    for (int j = 0; j < h; ++j) {
      const float keep = up ? v[j + h] : v[j], send = up ? v[j] : v[j + h];
      v[j] = keep + __shfl_xor_sync(0xffffffffu, send, m);
    }
  }
  float q = v[0];
#pragma unroll
  for (int m = 16 / G; m >= 1; m /= 2) q += __shfl_xor_sync(0xffffffffu, q, m);
  return q;
}  // 16 KB
constexpr int kLcSmem = kLcSlots * kLcSlotBytes;

__global__ void __launch_bounds__(256, 2) lconv_kernel(const float* __restrict__ g, const float* __restrict__ dw,
                                                       const float* __restrict__ nw, const int* __restrict__ row_clip,
                                                       long nrows, long rows_per_cta, float eps,
                                                       __half* __restrict__ a_hi, __half* __restrict__ a_lo,
                                                       float s_code, int* err) {
  constexpr int D = kLcD, G = kLcG, S = kLcSlots, KS = kLcHalo + 1;
  extern __shared__ __align__(128) float lc_ring[];  // [S][G][1024]
  __shared__ __align__(8) uint64_t bar_full[S];
  __shared__ __align__(16) float red[2][G][8];
  __shared__ int abort_flag, skip;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const long rs = (long)blockIdx.x * rows_per_cta;
  const long re = rs + rows_per_cta < nrows ? rs + rows_per_cta : nrows;
  if (rs >= re) return;  // the whole CTA: nothing below has started
  const int ngroups = (int)((re - rs + G - 1) / G);
  if (t == 0) {
    skip = *reinterpret_cast<volatile int*>(err) != 0;
    abort_flag = 0;
    for (int k = 0; k < S; ++k) mbar_init(&bar_full[k], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (skip) return;  // an earlier kernel on this device already failed
  auto issue = [&](int gi) {
    const long r = rs + (long)gi * G;
    const long n = re - r < G ? re - r : G;
    const int k = gi % S;
    mbar_expect_tx(&bar_full[k], (uint32_t)(n * D * 4));
    bulk_load(lc_ring + (long)k * G * D, g + r * D, (uint32_t)(n * D * 4), &bar_full[k]);
  };
  int issued = 0;
  if (t == 0)
    for (; issued < S && issued < ngroups; ++issued) issue(issued);
  float4 w[KS];
#pragma unroll
  for (int k = 0; k < KS; ++k) w[k] = __ldg(reinterpret_cast<const float4*>(dw + k * D) + t);
  const float4 nv = __ldg(reinterpret_cast<const float4*>(nw) + t);
  // the window: rows rs - 4 .. rs - 1 (raw values; clip id -1 before row 0)
  float4 win[KS - 1];
  int cw[KS - 1];
#pragma unroll
  for (int k = 0; k < KS - 1; ++k) {
    const long r = rs - (KS - 1) + k;
    win[k] = r >= 0 ? __ldg(reinterpret_cast<const float4*>(g + r * D) + t) : make_float4(0.f, 0.f, 0.f, 0.f);
    cw[k] = r >= 0 ? __ldg(row_clip + r) : -1;
  }
  // clip ids of the next group: lane i < G holds row i's
  int cnext = (lane < G && rs + lane < re) ? __ldg(row_clip + rs + lane) : -2;
  const float inv_code = s_code != 0.0f ? 1.0f / s_code : 0.0f;
  int gi = 0;
  for (; gi < ngroups; ++gi) {
    const long r0 = rs + (long)gi * G;
    int cg[G];
#pragma unroll
    for (int i = 0; i < G; ++i) cg[i] = __shfl_sync(0xffffffffu, cnext, i);
    if (gi + 1 < ngroups) cnext = (lane < G && r0 + G + lane < re) ? __ldg(row_clip + r0 + G + lane) : -2;
    const bool got = mbar_wait(&bar_full[gi % S], (uint32_t)((gi / S) & 1), err, kErrWaitFull, &abort_flag);
    const float* B = lc_ring + (long)(gi % S) * G * D;
    float4 y[G];
    float ps[G];
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const float4 x = got ? reinterpret_cast<const float4*>(B + i * D)[t] : make_float4(0.f, 0.f, 0.f, 0.f);
      const int c = cg[i];
      // taps in ascending order from zero; a window row of another clip adds nothing
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int k = 0; k < KS - 1; ++k) {
        if (cw[k] == c) {
          acc.x = fmaf(win[k].x, w[k].x, acc.x);
          acc.y = fmaf(win[k].y, w[k].y, acc.y);
          acc.z = fmaf(win[k].z, w[k].z, acc.z);
          acc.w = fmaf(win[k].w, w[k].w, acc.w);
        }
      }
      acc.x = fmaf(x.x, w[KS - 1].x, acc.x);
      acc.y = fmaf(x.y, w[KS - 1].y, acc.y);
      acc.z = fmaf(x.z, w[KS - 1].z, acc.z);
      acc.w = fmaf(x.w, w[KS - 1].w, acc.w);
      y[i] = acc;
      ps[i] = acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
#pragma unroll
      for (int k = 0; k < KS - 2; ++k) {
        win[k] = win[k + 1];
        cw[k] = cw[k + 1];
      }
      win[KS - 2] = x;
      cw[KS - 2] = c;
    }
    const float q = warp_reduce_scatter<G>(ps, lane);
    if ((lane & (32 / G - 1)) == 0) red[gi & 1][lane / (32 / G)][warp] = q;
    if (!__syncthreads_and(got)) break;  // the slot is free and the group's partial sums are in
    if (t == 0 && issued < ngroups) {
      fence_proxy_async_smem();
      issue(issued);  // into the slot this group just released
      ++issued;
    }
    // lane i < G finishes row i's norm factor; the other lanes take it by shuffle
    float inv_l = 0.f;
    if (lane < G) {
      const float4 p0 = *reinterpret_cast<const float4*>(&red[gi & 1][lane][0]);
      const float4 p1 = *reinterpret_cast<const float4*>(&red[gi & 1][lane][4]);
      const float tot = ((p0.x + p0.y) + (p0.z + p0.w)) + ((p1.x + p1.y) + (p1.z + p1.w));
      inv_l = 1.0f / sqrtf(tot / (float)D + eps);
    }
#pragma unroll
    for (int i = 0; i < G; ++i) {
      const long row = r0 + i;
      const float inv = __shfl_sync(0xffffffffu, inv_l, i);
      if (row < re) {
        const float u4[4] = {(y[i].x * inv) * nv.x, (y[i].y * inv) * nv.y, (y[i].z * inv) * nv.z,
                             (y[i].w * inv) * nv.w};
        if (s_code != 0.0f) {
          uint32_t codes = 0;  // signed-byte codes for linear_end's input scale (D bytes per row)
#pragma unroll
          for (int u = 0; u < 4; ++u)
            codes |= ((uint32_t)(int)srq_code(u4[u] * sigmoid_f(u4[u]), s_code, inv_code) & 0xFFu) << (8 * u);
          *reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(a_hi) + row * D + 4 * t) = codes;
        } else {
          uint32_t h01, l01, h23, l23;
          split2_f16(u4[0] * sigmoid_f(u4[0]), u4[1] * sigmoid_f(u4[1]), h01, l01);
          split2_f16(u4[2] * sigmoid_f(u4[2]), u4[3] * sigmoid_f(u4[3]), h23, l23);
          *reinterpret_cast<uint2*>(a_hi + row * D + 4 * t) = make_uint2(h01, h23);
          *reinterpret_cast<uint2*>(a_lo + row * D + 4 * t) = make_uint2(l01, l23);
        }
      }
    }
  }
  if (t == 0) {  // after an abort: wait (bounded) for copies still in flight before the CTA exits
    for (int q = gi; q < issued; ++q) {
      const uint32_t b = smem_u32(&bar_full[q % S]);
      const long long t0 = clock64();
      while (!mbar_try_wait(b, (uint32_t)((q / S) & 1))) {
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
  (void)row0;  // clip boundaries follow from row_clip alone (rows of a clip are contiguous)
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
  // contiguous ranges of whole groups, two CTAs per SM at most
  const long groups = (rows + kLcG - 1) / kLcG;
  const long ctas = groups < 2L * sms[dev] ? groups : 2L * sms[dev];
  const long per = ((groups + ctas - 1) / ctas) * kLcG;
  const int grid = (int)((rows + per - 1) / per);
  lconv_kernel<<<grid, 256, kLcSmem, st>>>(g, dw, nw, row_clip, rows, per, eps, a_hi, a_lo, s_code, err);
  return cudaGetLastError();
}

}  // namespace g4m
