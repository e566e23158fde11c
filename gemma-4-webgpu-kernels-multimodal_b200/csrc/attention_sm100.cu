// Vision self-attention on tcgen05: flash-style, head_dim 64, scale 1, no
// mask (full bidirectional attention over the image's patches).
//
// Replaces runVisionAttentionBodyWebGpu (src/vision/kernels.ts:500-668), whose
// WGSL recomputes every score three times per output element; CPU twin
// runVisionAttentionBodyCpu (75-131).
//
// Operands are fp16 hi/lo planes, so every product is split into three
// tensor-core terms (hi*hi + hi*lo + lo*hi) for fp32-grade scores and
// outputs:   S = Qh Kh^T + Qh Kl^T + Ql Kh^T,   O += Ph Vh + Ph Vl + Pl Vh.
//
// One CTA per (image*head, 128-query tile), 192 threads:
//   warp 0      TMA: Q once, then K / V^T tiles of 128 keys (2-stage ring)
//   warp 1      TMEM owner + MMA issuer: S into two TMEM buffers (S_{j+1}
//               overlaps the softmax of S_j), P*V into a third region
//   warps 2..9  softmax: warpgroup g runs an independent online softmax over
//               key columns [64g, 64g + 64) of every S tile (its own max, sum,
//               P sub-tile, P*V accumulator and O registers); the two partial
//               results are merged once at the end.  One query row per thread.
// Layouts: Q, K [bh][n][64]; V^T [bh][64][vt_pitch] (keys >= n read as zero);
// O [(img*n + q)][head*64 + d].
#include "g4m_kernels.h"
#include "g4m_sm100.cuh"

namespace g4m {

namespace {

constexpr int kSoftGroups = 2;                        // softmax warpgroups (key-column halves)
constexpr int kThreads = 64 + 128 * kSoftGroups;
constexpr int QT = 128;                // queries per CTA
constexpr int KT = 128;                // keys per tile
constexpr int HD = 64;
constexpr int TILE_BYTES = 128 * 128;  // one [128 rows x 64 fp16] swizzled tile
constexpr int Q_OFF = 0;                         // q hi, q lo
constexpr int KV_OFF = 2 * TILE_BYTES;           // 2 stages x (k hi, k lo, vt hi (2 x 8K), vt lo (2 x 8K))
constexpr int KV_STAGE = 4 * TILE_BYTES;
constexpr int P_OFF = KV_OFF + 2 * KV_STAGE;     // p hi (2 sub-tiles), p lo (2 sub-tiles)
constexpr int SMEM_BYTES = P_OFF + 4 * TILE_BYTES;
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 512;  // S0 [0,128) S1 [128,256) PV0 [256,320) PV1 [320,384)
constexpr float kLog2e = 1.4426950408889634f;
static_assert(SMEM_ALLOC + 512 <= 232448, "dynamic + static shared memory exceeds 227 KB per block");

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Byte offset of element (row, col) of a [rows x 64] fp16 tile in the
// 128-byte swizzle layout (16-byte chunk index XOR row % 8).
__device__ __forceinline__ uint32_t sw128_off(int row, int col) {
  return (uint32_t)row * 128u + ((uint32_t)(((col >> 3) ^ (row & 7)) << 4)) + (uint32_t)((col & 7) << 1);
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap mQh, const __grid_constant__ CUtensorMap mQl,
                   const __grid_constant__ CUtensorMap mKh, const __grid_constant__ CUtensorMap mKl,
                   const __grid_constant__ CUtensorMap mVh, const __grid_constant__ CUtensorMap mVl, int n, int heads,
                   __half* __restrict__ o_hi, __half* __restrict__ o_lo, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t b_q, b_kvf[2], b_kve[2], b_sf[2], b_se[2], b_p, b_pv;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag, skip;

  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, q0 = blockIdx.x * QT;
  const int T = (n + KT - 1) / KT;

  if (threadIdx.x == 0) {
    skip = *reinterpret_cast<volatile int*>(err) != 0;
    abort_flag = 0;
    mbar_init(&b_q, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&b_kvf[s], 1);
      mbar_init(&b_kve[s], 1);
      mbar_init(&b_sf[s], 1);
      mbar_init(&b_se[s], 4 * kSoftGroups);
    }
    mbar_init(&b_p, 4 * kSoftGroups);
    mbar_init(&b_pv, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (skip) return;  // an earlier CTA of this grid already failed
  if (warp == 1) tmem_alloc(&tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&mQh);
      prefetch_tmap(&mKh);
      prefetch_tmap(&mVh);
      mbar_expect_tx(&b_q, 2 * TILE_BYTES);
      tma_load_2d(sm + Q_OFF, &mQh, &b_q, 0, bh * n + q0);
      tma_load_2d(sm + Q_OFF + TILE_BYTES, &mQl, &b_q, 0, bh * n + q0);
      int issued = 0;
      for (int j = 0; j < T; ++j) {
        const int s = j & 1, k = j >> 1;
        if (!mbar_wait(&b_kve[s], (k & 1) ^ 1, err, kErrWaitEmpty, &abort_flag)) break;
        uint8_t* st = sm + KV_OFF + s * KV_STAGE;
        mbar_expect_tx(&b_kvf[s], KV_STAGE);
        tma_load_2d(st, &mKh, &b_kvf[s], 0, bh * n + j * KT);
        tma_load_2d(st + TILE_BYTES, &mKl, &b_kvf[s], 0, bh * n + j * KT);
        // V^T [64 d][128 keys] as two [64 x 64] swizzled sub-tiles per plane
        tma_load_2d(st + 2 * TILE_BYTES, &mVh, &b_kvf[s], j * KT, bh * HD);
        tma_load_2d(st + 2 * TILE_BYTES + TILE_BYTES / 2, &mVh, &b_kvf[s], j * KT + 64, bh * HD);
        tma_load_2d(st + 3 * TILE_BYTES, &mVl, &b_kvf[s], j * KT, bh * HD);
        tma_load_2d(st + 3 * TILE_BYTES + TILE_BYTES / 2, &mVl, &b_kvf[s], j * KT + 64, bh * HD);
        ++issued;
      }
      // drain: Q and the last use of each stage
      const uint32_t qb = smem_u32(&b_q);
      long long t0 = clock64();
      while (!mbar_try_wait(qb, 0) && clock64() - t0 < kWaitCycles) {
      }
      for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j) {
        const uint32_t b = smem_u32(&b_kvf[j & 1]);
        t0 = clock64();
        while (!mbar_try_wait(b, (j >> 1) & 1)) {
          if (clock64() - t0 > kWaitCycles) {
            atomicCAS(err, 0, kErrWaitDrain);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16_f32(128, KT);
      constexpr uint32_t id_pv = idesc_f16_f32(128, HD);
      const uint32_t qh = smem_u32(sm + Q_OFF), ql = qh + TILE_BYTES;
      const uint32_t ph = smem_u32(sm + P_OFF), pl = ph + 2 * TILE_BYTES;
      bool ok = mbar_wait(&b_q, 0, err, kErrWaitFull, &abort_flag);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1, k = j >> 1;
        if (!mbar_wait(&b_kvf[s], k & 1, err, kErrWaitFull, &abort_flag)) return false;
        if (!mbar_wait(&b_se[s], (k & 1) ^ 1, err, kErrWaitAccEmpty, &abort_flag)) return false;
        tc_fence_after();
        const uint32_t kh = smem_u32(sm + KV_OFF + s * KV_STAGE), kl = kh + TILE_BYTES;
        const uint32_t d = tmem + s * KT;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t dq = desc_k_sw128(qh + kk * 32), dk = desc_k_sw128(kh + kk * 32);
          mma_f16_ss(d, dq, dk, id_s, kk > 0 ? 1u : 0u);
          mma_f16_ss(d, dq, desc_k_sw128(kl + kk * 32), id_s, 1u);
          mma_f16_ss(d, desc_k_sw128(ql + kk * 32), dk, id_s, 1u);
        }
        mma_commit(&b_sf[s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < T && ok; ++j) {
        if (j + 1 < T && !issue_s(j + 1)) break;
        if (!mbar_wait(&b_p, j & 1, err, kErrWaitFull, &abort_flag)) break;
        tc_fence_after();
        const int s = j & 1;
        const uint32_t vh = smem_u32(sm + KV_OFF + s * KV_STAGE + 2 * TILE_BYTES), vl = vh + TILE_BYTES;
        // one K=64 P*V chain per key half, each into its own accumulator
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const uint32_t d = tmem + 2 * KT + half * HD;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t off = kk * 32;
            const uint64_t dph = desc_k_sw128(ph + half * TILE_BYTES + off);
            const uint64_t dvh = desc_k_sw128(vh + half * (TILE_BYTES / 2) + off);
            mma_f16_ss(d, dph, dvh, id_pv, kk > 0 ? 1u : 0u);
            mma_f16_ss(d, dph, desc_k_sw128(vl + half * (TILE_BYTES / 2) + off), id_pv, 1u);
            mma_f16_ss(d, desc_k_sw128(pl + half * TILE_BYTES + off), dvh, id_pv, 1u);
          }
        }
        mma_commit(&b_pv);
        mma_commit(&b_kve[s]);
      }
      // Let the last stage-release commits land before the CTA can exit.
      if (ok && !abort_flag) {
        for (int j = T > 2 ? T - 2 : 0; j < T; ++j)
          if (!mbar_wait(&b_kve[j & 1], (j >> 1) & 1, err, kErrWaitDrain, &abort_flag)) break;
      }
    }
  } else {
    // softmax warps: group g = key half g of every tile
    const int q = warp & 3;
    const int g = (warp - 2) >> 2;
    const int r = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    constexpr int KH = KT / kSoftGroups;  // 64 keys per group
    uint8_t* ph = sm + P_OFF + g * TILE_BYTES;  // this group's P sub-tile (hi)
    uint8_t* pl = ph + 2 * TILE_BYTES;          // (lo)
    const uint32_t pv_col = 2 * KT + g * HD;    // this group's P*V accumulator
    float o[HD];
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    bool ok = true;
    for (int j = 0; j < T; ++j) {
      const int b = j & 1, k = j >> 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&b_sf[b], k & 1, err, kErrWaitAccFull, &abort_flag));
      if (!ok) break;
      tc_fence_after();
      const uint32_t sbase = tmem + lane_base + b * KT + g * KH;
      const int kvalid = n - j * KT - g * KH;  // valid keys among this group's 64
      const bool full = kvalid >= KH;
      // pass 1: running max over this group's keys
      float mt = -INFINITY;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t sr[32];
        tmem_ld32_nw(sbase + hb * 32, sr);
        tmem_wait_ld();
        if (full) {
#pragma unroll
          for (int c = 0; c < 32; ++c) mt = fmaxf(mt, __uint_as_float(sr[c]));
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (hb * 32 + c < kvalid) mt = fmaxf(mt, __uint_as_float(sr[c]));
        }
      }
      const float mn = fmaxf(m, mt);  // -inf only while this group has seen no valid key
      const float alpha = (m == -INFINITY) ? 0.f : ex2((m - mn) * kLog2e);
      const float mnl = (mn == -INFINITY) ? 0.f : mn * kLog2e;
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(&b_pv, (j - 1) & 1, err, kErrWaitAccFull, &abort_flag));
        if (!ok) break;
        tc_fence_after();
        uint32_t pv[32];
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          tmem_ld32_nw(tmem + lane_base + pv_col + hb * 32, pv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[hb * 32 + i] = fmaf(o[hb * 32 + i], alpha_prev, __uint_as_float(pv[i]));
        }
      }
      // pass 2: probabilities, row sum, P (hi / lo) into this group's swizzled sub-tile
      float rs = 0.f;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        uint32_t sr[32];
        tmem_ld32_nw(sbase + hb * 32, sr);
        tmem_wait_ld();
        if (full) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float p = ex2(fmaf(__uint_as_float(sr[c]), kLog2e, -mnl));
            sr[c] = __float_as_uint(p);
            rs += p;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float p = (hb * 32 + c < kvalid) ? ex2(fmaf(__uint_as_float(sr[c]), kLog2e, -mnl)) : 0.f;
            sr[c] = __float_as_uint(p);
            rs += p;
          }
        }
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint32_t hv[4], lv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
            split2_f16(__uint_as_float(sr[c + 2 * u]), __uint_as_float(sr[c + 2 * u + 1]), hv[u], lv[u]);
          const uint32_t off = sw128_off(r, hb * 32 + c);
          *reinterpret_cast<uint4*>(ph + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
          *reinterpret_cast<uint4*>(pl + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b_se[b]);  // S buffer b may be overwritten (tile j + 2)
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b_p);
      l = fmaf(l, alpha, rs);
      alpha_prev = alpha;
      m = mn;
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&b_pv, (T - 1) & 1, err, kErrWaitAccFull, &abort_flag));
      if (ok) {
        tc_fence_after();
        uint32_t pv[32];
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          tmem_ld32_nw(tmem + lane_base + pv_col + hb * 32, pv);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[hb * 32 + i] = fmaf(o[hb * 32 + i], alpha_prev, __uint_as_float(pv[i]));
        }
      }
    }
    // Merge the two key halves (flash-decoding style): group g keeps output
    // columns [32g, 32g + 32) and receives the partner's (m, l, O) for them
    // through the P region, idle once the last P*V has completed.
    float* xch = reinterpret_cast<float*>(sm + P_OFF);  // [group][row][34]
    {
      float* mine = xch + ((size_t)g * 128 + r) * 34;
      mine[0] = m;
      mine[1] = l;
      if (g == 0) {  // hand the partner the columns it keeps (constant indices)
#pragma unroll
        for (int i = 0; i < 32; ++i) mine[2 + i] = o[32 + i];
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) mine[2 + i] = o[i];
      }
    }
    asm volatile("bar.sync %0, %1;" ::"r"(1 + q), "r"(32 * kSoftGroups) : "memory");
    if (ok) {
      const float* other = xch + ((size_t)(1 - g) * 128 + r) * 34;
      const float m2 = other[0], l2 = other[1];
      const float mm = fmaxf(m, m2);
      const float a1 = (m == -INFINITY) ? 0.f : ex2((m - mm) * kLog2e);
      const float a2 = (m2 == -INFINITY) ? 0.f : ex2((m2 - mm) * kLog2e);
      const float inv = 1.0f / (l * a1 + l2 * a2);
      float own[32];
      if (g == 0) {
#pragma unroll
        for (int i = 0; i < 32; ++i) own[i] = o[i];
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) own[i] = o[32 + i];
      }
      const int qrow = q0 + r;
      if (qrow < n) {
        const int img = bh / heads, head = bh % heads;
        const size_t orow = (size_t)img * n + qrow;
        __half* dh = o_hi + orow * (size_t)(heads * HD) + head * HD + 32 * g;
        __half* dl = o_lo + orow * (size_t)(heads * HD) + head * HD + 32 * g;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint32_t hv[4], lv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const float v0 = (own[i + 2 * u] * a1 + other[2 + i + 2 * u] * a2) * inv;
            const float v1 = (own[i + 2 * u + 1] * a1 + other[2 + i + 2 * u + 1] * a2) * inv;
            split2_f16(v0, v1, hv[u], lv[u]);
          }
          *reinterpret_cast<uint4*>(dh + i) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
          *reinterpret_cast<uint4*>(dl + i) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
        }
      }
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

cudaError_t vision_attention_tc(const __half* q_hi, const __half* q_lo, const __half* k_hi, const __half* k_lo,
                                const __half* vt_hi, const __half* vt_lo, int bh, int n, int vt_pitch, int heads,
                                __half* o_hi, __half* o_lo, int* err, cudaStream_t st) {
  if (bh <= 0 || n <= 0) return cudaSuccess;
  if (vt_pitch % 64 != 0 || vt_pitch < n) return cudaErrorInvalidValue;
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_ALLOC);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  CUtensorMap mQh, mQl, mKh, mKl, mVh, mVl;
  const uint64_t rows = (uint64_t)bh * n;
  if (!make_tmap_f16(&mQh, q_hi, rows, HD, 128) || !make_tmap_f16(&mQl, q_lo, rows, HD, 128) ||
      !make_tmap_f16(&mKh, k_hi, rows, HD, 128) || !make_tmap_f16(&mKl, k_lo, rows, HD, 128))
    return cudaErrorInvalidValue;
  // V^T viewed as [bh*64 rows][n cols]; boxes of 64 keys x 64 rows
  if (!make_tmap_f16_any(&mVh, vt_hi, (uint64_t)bh * HD, (uint64_t)n, (uint64_t)vt_pitch, 64) ||
      !make_tmap_f16_any(&mVl, vt_lo, (uint64_t)bh * HD, (uint64_t)n, (uint64_t)vt_pitch, 64))
    return cudaErrorInvalidValue;
  dim3 grid((n + QT - 1) / QT, bh);
  attn_tc_kernel<<<grid, kThreads, SMEM_ALLOC, st>>>(mQh, mQl, mKh, mKl, mVh, mVl, n, heads, o_hi, o_lo, err);
  return cudaGetLastError();
}

}  // namespace g4m
