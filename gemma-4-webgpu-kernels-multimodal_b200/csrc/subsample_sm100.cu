// Audio subsample convs on sm_100a (runAudioSubsampleConvLayerCpu twice,
// src/audio/kernels.ts:112-183, and the flatten of runAudioSubsampleProjectionCpu,
// 22-62).  Source rows outside the clip are skipped, as masked or out-of-range
// source times are in the reference.
//
// Layer 0 (1 -> 128 channels, 3x3 stride 2, channel LayerNorm with weight,
// ReLU): statistics in double from the nine taps and precomputed weight
// moments, the 128 channel values of 16 positions as mma.sync products of the
// taps and the filters (split fp16 operands), the statistics applied in f32.
// The result is stored as fp16 hi / lo planes [rows][64 freq][128 ch] in which every
// clip's rows are preceded and followed by a zero row, so a layer-1 tap that
// leaves the clip reads zeros.
//
// Layer 1 (128 -> 32 channels, 3x3 stride 2, LayerNorm, ReLU) is an implicit
// GEMM on tcgen05: M = 128 output positions (4 rows x 32 frequencies), N = 32
// channels, K = 9 taps x 128 channels.  The layer-0 planes are described to
// TMA as 5-D tensors (channel, frequency parity, frequency / 2, row parity,
// row / 2), so for each tap (kt, kf) and 64-channel half the stride-2 im2col
// tile L0[2 t1 + kt - 1][2 f1 + kf - 1][c] is one dense box (64 channels x 32
// frequencies x 4 rows at fixed parities) landing in the 128-byte swizzled
// K-major layout the MMA reads (frequency -1 is an out-of-range, zero-filled
// coordinate).  Operands are fp16 hi / lo planes; the three terms
// Ah Bh + Ah Bl + Al Bh accumulate in f32 in TMEM as two MMAs per k-step,
// Ah [Bh | Bl] (N = 64) and Al Bh (N = 32).  The epilogue thread of
// position (t1, f1) holds its 32 channels, so the LayerNorm is thread-local
// (double statistics, as the reference's JS numbers).
//   warp 0  TMA producer (2-stage ring; two CTAs per SM)   warp 1  TMEM owner + MMA issuer
//   warps 2..5  epilogue (warp % 4 = output row of the tile, lane = f1)
#include "g4m_kernels.h"
#include "g4m_sm100.cuh"

namespace g4m {

namespace {
constexpr int SA_BYTES = 128 * 128;  // A tile: 128 positions x 64 channels fp16
constexpr int SB_BYTES = 32 * 128;   // B tile: 32 output channels x 64 channels fp16
constexpr int SSTAGE = 2 * SA_BYTES + 2 * SB_BYTES;
constexpr int SSTAGES = 2;  // 2 stages: two CTAs per SM, one's epilogue overlapping the other's mainloop
constexpr int SKB = 18;              // k-blocks: 9 taps x 2 channel halves
constexpr int SUB_SMEM = SSTAGES * SSTAGE + 1024;
constexpr int SUB_THREADS = 192;
constexpr int L0_ROW = 64 * 128;     // elements of one layer-0 row

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// 1 / sqrt(a) for a normal positive double: the float hardware estimate
// refined by two Newton-Raphson steps r <- r (3 - a r^2) / 2 in double
// (relative error ~2^-22 -> ~2^-43 -> below double rounding).
__device__ __forceinline__ double rsqrt_nr(double a) {
  double r = (double)rsqrtf((float)a);
  r = r * (1.5 - 0.5 * a * r * r);
  r = r * (1.5 - 0.5 * a * r * r);
  return r;
}

__device__ __forceinline__ void mma_16816_s(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void drain_wait_s(uint64_t* bar, uint32_t parity, int* err) {
  const uint32_t b = smem_u32(bar);
  const long long t0 = clock64();
  while (!mbar_try_wait(b, parity)) {
    if (clock64() - t0 > kWaitCycles) {
      atomicCAS(err, 0, kErrWaitDrain);
      return;
    }
  }
}
}  // namespace

// Layer 0 for 4 layer-0 rows x 64 frequencies per CTA (256 positions).  The
// LayerNorm statistics of a position follow from its nine taps x_k: with
// v_c = sum_k x_k w[c][k], mean = sum_k x_k wbar_k and
// E[v^2] = sum_{k<=l} x_k x_l G_kl, where wbar_k = (1/128) sum_c w[c][k] and
// G_kl = (1 or 2)/128 sum_c w[c][k] w[c][l] (w0stat: 9 + 45 doubles), so
// one thread per position computes them in double (54 FMAs).  The 128
// channel values v_c of 16 positions are one mma.sync m16n8k16 product per
// 8 channels: A = the positions' taps (K = 9, padded to 16), B = the filters,
// both split as hi = f16(x), lo = f16((x - hi) 2^11), three products
// (hi hi into one accumulator, hi lo + lo hi into another, scaled back by
// 2^-11), i.e. the f32-grade 9-term sum.  Warp w takes row w / 2 and 32
// frequencies (two 16-position tiles), four 8-channel tiles at a time; the
// epilogue applies the statistics in f32, (v - mean) (inv n_c), then ReLU
// and the hi / lo planes; each 32-channel chunk passes through the warp's
// 2 KB staging block (16-byte pieces XOR-swizzled by position pair, both
// phases free of bank conflicts) and leaves as 64 contiguous bytes per
// position and plane.
__global__ void __launch_bounds__(256) subsample_l0_kernel(const float* __restrict__ feats, const int* __restrict__ foff,
                                                           const int* __restrict__ fcount, const int* __restrict__ t0off,
                                                           const float* __restrict__ w0,
                                                           const double* __restrict__ w0stat,
                                                           const float* __restrict__ n0, float eps,
                                                           __half* __restrict__ l0h, __half* __restrict__ l0l) {
  constexpr int XP = 130;  // frames: column 0 is frequency -1 (zero), column f + 1 frequency f
  constexpr int KP = 24;   // halves per filter row (taps 9..23 zero; 48-byte rows: B loads hit distinct banks)
  constexpr float kS = 2048.0f;
  __shared__ __align__(16) float xs[9][XP];  // input frames 2 rb - 1 .. 2 rb + 7
  __shared__ __align__(16) __half wsh[128 * KP], wsl[128 * KP];
  __shared__ __align__(16) float nsm[128];
  __shared__ double stat_s[54];
  __shared__ __align__(16) float2 mi[256];  // (mean, 1 / sqrt(var + eps)) per position, f32
  __shared__ __align__(16) uint32_t stage[8 * 512];  // per warp: [16 positions][32 channels] hi, then lo
  const int clip = blockIdx.y, rb = blockIdx.x * 4;  // first layer-0 row of this CTA
  const int F = fcount[clip];
  const int T0 = (F - 1) / 2 + 1;
  if (rb > T0) return;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* fx = feats + (long)foff[clip] * 128;
  for (int i = t; i < 9 * 128; i += 256) {
    const int fr = 2 * rb - 1 + i / 128;
    xs[i / 128][1 + i % 128] = (fr >= 0 && fr < F) ? fx[(long)fr * 128 + (i % 128)] : 0.f;
  }
  if (t < 9) xs[t][0] = 0.f;
  for (int i = t; i < 128 * 16; i += 256) {
    const int c = i >> 4, k = i & 15;
    const float v = k < 9 ? __ldg(w0 + c * 9 + k) : 0.f;
    const __half h = __float2half_rn(v);
    wsh[c * KP + k] = h;
    wsl[c * KP + k] = __float2half_rn((v - __half2float(h)) * kS);
  }
  if (t < 128) nsm[t] = __ldg(n0 + t);
  if (t < 54) stat_s[t] = w0stat[t];
  __syncthreads();
  {  // statistics of position t = (row rb + t / 64, frequency t % 64)
    const int rr = t >> 6, f0 = t & 63;
    double x[9];
#pragma unroll
    for (int kt = 0; kt < 3; ++kt)
#pragma unroll
      for (int kf = 0; kf < 3; ++kf) x[kt * 3 + kf] = (double)xs[2 * rr + kt][2 * f0 + kf];
    double mean = 0.0, e2 = 0.0;
    int q = 9;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      mean = fma(x[k], stat_s[k], mean);
#pragma unroll
      for (int l = k; l < 9; ++l) e2 = fma(x[k] * x[l], stat_s[q++], e2);
    }
    const double var = fmax(e2 - mean * mean, 0.0);
    mi[t] = make_float2((float)mean, (float)rsqrt_nr(var + (double)eps));
  }
  __syncthreads();
  const int rr = warp >> 1, r = rb + rr, fw = 32 * (warp & 1);  // this warp's row and first frequency
  if (r > T0) return;
  const long row_c = (long)t0off[clip];
  if (r == T0) {  // the zero row after the clip (and, for clip 0, the one before it)
    const uint4 z = make_uint4(0u, 0u, 0u, 0u);
    for (int k = 0; k < (clip == 0 ? 2 : 1); ++k) {
      const long row = k == 0 ? row_c + T0 : row_c - 1;
      uint4* zh = reinterpret_cast<uint4*>(l0h + row * L0_ROW + fw * 128);
      uint4* zl = reinterpret_cast<uint4*>(l0l + row * L0_ROW + fw * 128);
      for (int i = lane; i < 32 * 128 / 8; i += 32) zh[i] = z, zl[i] = z;
    }
    return;
  }
  const int g = lane >> 2, tq = lane & 3;
  // taps 2 tq and 2 tq + 1 of this lane's A columns (all < 9), and tap 8 (columns 8..15: tq == 0 only)
  const int k0 = 2 * tq, k1 = 2 * tq + 1;
  const int o0 = (k0 / 3) * XP + k0 % 3, o1 = (k1 / 3) * XP + k1 % 3, o8 = 2 * XP + 2;
  const float* xrow = &xs[2 * rr][0];
  const long rowbase = (row_c + r) * L0_ROW;
  uint32_t* sth = stage + warp * 512;  // this warp's 2 KB: hi words [0, 256), lo words [256, 512)
  uint32_t* stl = sth + 256;
#pragma unroll 1
  for (int m = 0; m < 2; ++m) {
    const int fa = fw + 16 * m + g, fb = fa + 8;  // this lane's two positions (frequencies)
    uint32_t ah[4], al[4];
    {
      const float xa0 = xrow[o0 + 2 * fa], xa1 = xrow[o1 + 2 * fa];
      const float xb0 = xrow[o0 + 2 * fb], xb1 = xrow[o1 + 2 * fb];
      const float xa8 = tq == 0 ? xrow[o8 + 2 * fa] : 0.f, xb8 = tq == 0 ? xrow[o8 + 2 * fb] : 0.f;
      const float v[4][2] = {{xa0, xa1}, {xb0, xb1}, {xa8, 0.f}, {xb8, 0.f}};
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        union {
          __half2 h2;
          uint32_t w;
        } H, L;
        H.h2 = __floats2half2_rn(v[u][0], v[u][1]);
        const float2 b = __half22float2(H.h2);
        L.h2 = __floats2half2_rn((v[u][0] - b.x) * kS, (v[u][1] - b.y) * kS);
        ah[u] = H.w;
        al[u] = L.w;
      }
    }
    const float2 sa = mi[rr * 64 + fa], sb = mi[rr * 64 + fb];
#pragma unroll 1
    for (int nc = 0; nc < 16; nc += 4) {
      float hh[4][4], xx[4][4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int ch = (nc + n) * 8 + g;  // B column of this lane
        const uint32_t bh0 = *reinterpret_cast<const uint32_t*>(wsh + ch * KP + 2 * tq);
        const uint32_t bh1 = *reinterpret_cast<const uint32_t*>(wsh + ch * KP + 2 * tq + 8);
        const uint32_t bl0 = *reinterpret_cast<const uint32_t*>(wsl + ch * KP + 2 * tq);
        const uint32_t bl1 = *reinterpret_cast<const uint32_t*>(wsl + ch * KP + 2 * tq + 8);
#pragma unroll
        for (int u = 0; u < 4; ++u) hh[n][u] = xx[n][u] = 0.f;
        mma_16816_s(hh[n], ah, bh0, bh1);
        mma_16816_s(xx[n], ah, bl0, bl1);
        mma_16816_s(xx[n], al, bh0, bh1);
      }
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        const int c = (nc + n) * 8 + 2 * tq;  // this lane's channel pair
        const float2 nv = *reinterpret_cast<const float2*>(nsm + c);
        float y[4];
        y[0] = fmaxf((fmaf(xx[n][0], 1.0f / kS, hh[n][0]) - sa.x) * (sa.y * nv.x), 0.f);
        y[1] = fmaxf((fmaf(xx[n][1], 1.0f / kS, hh[n][1]) - sa.x) * (sa.y * nv.y), 0.f);
        y[2] = fmaxf((fmaf(xx[n][2], 1.0f / kS, hh[n][2]) - sb.x) * (sb.y * nv.x), 0.f);
        y[3] = fmaxf((fmaf(xx[n][3], 1.0f / kS, hh[n][3]) - sb.x) * (sb.y * nv.y), 0.f);
        uint32_t h01, l01, h23, l23;
        split2_f16(y[0], y[1], h01, l01);
        split2_f16(y[2], y[3], h23, l23);
        // stage [16 positions][32 channels] per plane; 16-byte chunk n of position p at n ^ ((p >> 1) & 3)
        const int wa = g * 16 + 4 * (n ^ ((g >> 1) & 3)) + tq, wb = wa + 8 * 16;  // fb: row g + 8, same swizzle
        sth[wa] = h01;
        stl[wa] = l01;
        sth[wb] = h23;
        stl[wb] = l23;
      }
      __syncwarp();
      // 64 contiguous bytes (32 channels) per position and plane: 8 positions per store
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int p = 8 * k + (lane >> 2), j = lane & 3;
        const int w = p * 16 + 4 * (j ^ ((p >> 1) & 3));
        const long o = rowbase + (long)(fw + 16 * m + p) * 128 + nc * 8 + 8 * j;
        *reinterpret_cast<uint4*>(l0h + o) = *reinterpret_cast<const uint4*>(sth + w);
        *reinterpret_cast<uint4*>(l0l + o) = *reinterpret_cast<const uint4*>(stl + w);
      }
      __syncwarp();
    }
  }
}

__global__ void __launch_bounds__(SUB_THREADS, 2)
    subsample_conv_tc_kernel(const __grid_constant__ CUtensorMap mLh, const __grid_constant__ CUtensorMap mLl,
                             const __grid_constant__ CUtensorMap mWh, const __grid_constant__ CUtensorMap mWl,
                             const int* __restrict__ t0off, const int* __restrict__ row0, const int* __restrict__ rows,
                             const float* __restrict__ n1, float eps, __half* __restrict__ a_hi,
                             __half* __restrict__ a_lo, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[SSTAGES], bar_empty[SSTAGES], bar_acc;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag, skip;
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int clip = blockIdx.y;
  const int R = rows[clip];
  const int t1_0 = blockIdx.x * 4;
  if (t1_0 >= R) return;  // whole CTA: nothing of this clip here
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    skip = *reinterpret_cast<volatile int*>(err) != 0;
    abort_flag = 0;
    for (int s = 0; s < SSTAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    mbar_init(&bar_acc, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (skip) return;  // an earlier kernel on this device already failed
  if (warp == 1) tmem_alloc(&tmem_slot, 64);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  auto sA = [&](int s, int plane) { return sm + s * SSTAGE + plane * SA_BYTES; };
  auto sB = [&](int s, int plane) { return sm + s * SSTAGE + 2 * SA_BYTES + plane * SB_BYTES; };

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&mLh);
      prefetch_tmap(&mWh);
      const int zbase = t0off[clip] + 2 * t1_0 - 1;  // layer-0 row of tap kt = 0 for the tile's first output row
      int issued = 0;
      for (int kb = 0; kb < SKB; ++kb) {
        const int s = kb % SSTAGES, tap = kb >> 1, half = kb & 1, kt = tap / 3, kf = tap % 3;
        // frequency 2 f1 + kf - 1: parity 0 for kf = 1, else 1; half index f1 - 1 (kf = 0) or f1
        const int fpar = kf == 1 ? 0 : 1, fh = kf == 0 ? -1 : 0;
        const int rr = zbase + kt;  // >= 0: a zero row precedes every clip
        if (!mbar_wait(&bar_empty[s], ((kb / SSTAGES) & 1) ^ 1, err, kErrWaitEmpty, &abort_flag)) break;
        mbar_expect_tx(&bar_full[s], SSTAGE);
        tma_load_5d(sA(s, 0), &mLh, &bar_full[s], 64 * half, fpar, fh, rr & 1, rr >> 1);
        tma_load_5d(sA(s, 1), &mLl, &bar_full[s], 64 * half, fpar, fh, rr & 1, rr >> 1);
        tma_load_2d(sB(s, 0), &mWh, &bar_full[s], 64 * half, 32 * tap);
        tma_load_2d(sB(s, 1), &mWl, &bar_full[s], 64 * half, 32 * tap);
        ++issued;
      }
      for (int j = issued > SSTAGES ? issued - SSTAGES : 0; j < issued; ++j)
        drain_wait_s(&bar_full[j % SSTAGES], (j / SSTAGES) & 1, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // B hi (32 rows) and B lo (32 rows) are adjacent 1024-byte-aligned row
      // groups of one stage, i.e. one N = 64 operand [Bh | Bl]: columns 0..31
      // collect Ah Bh + Al Bh, columns 32..63 Ah Bl.
      constexpr uint32_t idesc64 = idesc_f16_f32(128, 64), idesc32 = idesc_f16_f32(128, 32);
      for (int kb = 0; kb < SKB; ++kb) {
        const int s = kb % SSTAGES;
        if (!mbar_wait(&bar_full[s], (kb / SSTAGES) & 1, err, kErrWaitFull, &abort_flag)) break;
        tc_fence_after();
        const uint32_t ah = smem_u32(sA(s, 0)), al = smem_u32(sA(s, 1));
        const uint32_t bh = smem_u32(sB(s, 0));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint64_t dbh = desc_k_sw128(bh + k * 32);
          mma_f16_ss(tmem, desc_k_sw128(ah + k * 32), dbh, idesc64, (kb > 0 || k > 0) ? 1u : 0u);
          mma_f16_ss(tmem, desc_k_sw128(al + k * 32), dbh, idesc32, 1u);
        }
        mma_commit(&bar_empty[s]);
      }
      mma_commit(&bar_acc);  // every MMA above has completed when this arrives
      drain_wait_s(&bar_acc, 0, err);
    }
  } else {
    const int q = warp & 3;  // TMEM lanes 32 q .. 32 q + 31 = positions of output row t1_0 + q
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&bar_acc, 0, err, kErrWaitAccFull, &abort_flag));
    if (ok) {
      tc_fence_after();
      float acc[32], acc_lo[32];
      tmem_ld32(tmem + ((uint32_t)(32 * q) << 16), acc);
      tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 32, acc_lo);
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] += acc_lo[j];
      const int t1 = t1_0 + q;
      if (t1 < R) {
        double mean = 0.0;  // channelValues is a Float32Array: statistics in double
#pragma unroll
        for (int j = 0; j < 32; ++j) mean += (double)acc[j];
        mean /= 32.0;
        double var = 0.0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const double dv = (double)acc[j] - mean;
          var += dv * dv;
        }
        const double inv = 1.0 / sqrt(var / 32.0 + (double)eps);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const double nv = ((double)acc[j] - mean) * inv * (double)__ldg(n1 + j);
          v[j] = nv > 0.0 ? (float)nv : 0.f;
        }
        const long orow = (long)row0[clip] + t1;
        __half* dh = a_hi + orow * 1024 + lane * 32;
        __half* dl = a_lo + orow * 1024 + lane * 32;
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint32_t hv[4], lv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) split2_f16(v[j + 2 * u], v[j + 2 * u + 1], hv[u], lv[u]);
          *reinterpret_cast<uint4*>(dh + j) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
          *reinterpret_cast<uint4*>(dl + j) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFnS)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFnS encode_fn_s() {
  static EncodeTiledFnS fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFnS>(p);
  }
  return fn;
}

// Layer-0 plane [rows][64][128] fp16 (rows even) as a 5-D map (channel,
// frequency parity, frequency / 2, row parity, row / 2): dense boxes of
// 64 channels x 1 x 32 x 1 x 4 = one tap's 128-position im2col tile (16 KB),
// 128-byte swizzle.
static bool make_l0_map(CUtensorMap* map, const __half* base, long total_rows) {
  EncodeTiledFnS fn = encode_fn_s();
  if (!fn || (reinterpret_cast<uintptr_t>(base) % 16) != 0 || (total_rows % 2) != 0) return false;
  cuuint64_t dims[5] = {128, 2, 32, 2, (cuuint64_t)(total_rows / 2)};
  cuuint64_t strides[4] = {128 * 2, 2 * 128 * 2, 64 * 128 * 2, 2 * 64 * 128 * 2};
  cuuint32_t box[5] = {64, 1, 32, 1, 4};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<__half*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t audio_subsample_tc(const float* feats, const int* frame_off, const int* frames, const int* t0off,
                               long l0_rows, const int* row0, const int* rows, int clips, int max_t0, int max_rows,
                               const float* w0, const double* w0stat, const float* n0, const __half* w1_hi,
                               const __half* w1_lo, const float* n1, float eps, __half* l0h, __half* l0l,
                               __half* a_hi, __half* a_lo, int* err, cudaStream_t st) {
  if (clips <= 0 || max_rows <= 0) return cudaSuccess;
  if (clips > 65535) return cudaErrorInvalidValue;  // grid y = clip
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(subsample_conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SUB_SMEM);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  subsample_l0_kernel<<<dim3((max_t0 + 1 + 3) / 4, clips), 256, 0, st>>>(feats, frame_off, frames, t0off, w0, w0stat,
                                                                        n0, eps, l0h, l0l);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  CUtensorMap mLh, mLl, mWh, mWl;
  if (!make_l0_map(&mLh, l0h, l0_rows) || !make_l0_map(&mLl, l0l, l0_rows) ||
      !make_tmap_f16(&mWh, w1_hi, 9 * 32, 128, 32) || !make_tmap_f16(&mWl, w1_lo, 9 * 32, 128, 32))
    return cudaErrorInvalidValue;
  dim3 grid((max_rows + 3) / 4, clips);
  subsample_conv_tc_kernel<<<grid, SUB_THREADS, SUB_SMEM, st>>>(mLh, mLl, mWh, mWl, t0off, row0, rows, n1, eps, a_hi,
                                                                a_lo, err);
  return cudaGetLastError();
}

}  // namespace g4m
