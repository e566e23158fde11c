// Vision self-attention on tcgen05: flash-style, head_dim 64, scale 1, no
// mask (full bidirectional attention over the image's patches).
//
// Replaces runVisionAttentionBodyWebGpu (src/vision/kernels.ts:500-668), whose
// WGSL recomputes every score three times per output element; CPU twin
// runVisionAttentionBodyCpu (75-131).
//
// Operands are fp16 hi/lo planes, so every product is split into three
// tensor-core terms (hi*hi + hi*lo + lo*hi) for fp32-grade scores and
// outputs:   S = Qh Kh^T + Qh Kl^T + Ql Kh^T,   O += Ph (Vh + Vl) + Pl Vh.
// An N = 64 tcgen05.mma takes three quarters of the time of an N = 128 one
// (measured: 48 against 64 cycles), so P*V stacks the V hi and lo planes into
// one N = 128 operand: Ph [Vh | Vl] (N = 128) and Pl Vh (N = 64, the stacked
// operand's first 64 rows) accumulate into 128 TMEM columns whose two halves
// are summed at the end (112 cycles per 16 keys, against 128 for
// Pl [Vh | Vl] and 144 for three N = 64 products).
//
// One CTA per (image*head, 256 queries) = two 128-query tiles A and B that
// share every K / V tile, 320 threads:
//   warp 0      TMA: both Q tiles once, then K / V^T tiles of 128 keys
//               (2-stage ring)
//   warp 1      TMEM owner + MMA issuer, ping-ponging the tiles so that the
//               softmax of one overlaps the tensor-core work of the other:
//                 P*V_A(j), S_A(j+1), P*V_B(j), S_B(j+1), ...
//   warps 2..5  softmax of tile A, warps 6..9 of tile B: one query row per
//               thread, the whole 128-key score row in registers.
// TMEM (512 columns): S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512)
// (O columns [0,64) accumulate P*Vh, [64,128) P*Vl).
// The softmax overwrites its S columns with P: the 32 keys of S columns
// [32c, 32c+32) become fp16 hi in columns [32c, 32c+16) and lo in
// [32c+16, 32c+32), and the P*V MMA reads P straight from TMEM (A operand),
// so P never touches shared memory.  O accumulates in TMEM across key tiles; a
// row's running max is raised (and its O row rescaled in TMEM) only when a
// tile's max exceeds it by more than 2^8, so P <= 2^(8 + kPShift) and the
// rescale is rare.
// The next S of a tile overwrites its P columns, so the MMA warp issues it
// only after that tile's P*V has completed (waits overlap the other tile's
// MMAs).
// Layouts: Q, K [bh][n][64]; V^T [bh][64][vt_pitch] (keys >= n read as zero);
// O [(img*n + q)][head*64 + d].
#include "g4m_kernels.h"
#include "g4m_sm100.cuh"

namespace g4m {

namespace {

constexpr int kThreads = 64 + 256;
constexpr int QT = 128;                // queries per tile (two tiles per CTA)
constexpr int KT = 128;                // keys per tile
constexpr int HD = 64;
constexpr int TILE_BYTES = 128 * 128;  // one [128 rows x 64 fp16] swizzled tile
constexpr int Q_OFF = 0;               // tile t: q hi at 2t, q lo at 2t+1 (x TILE_BYTES)
constexpr int KV_OFF = 4 * TILE_BYTES; // 2 stages x (k hi, k lo, [vt hi | vt lo] keys 0-63, keys 64-127)
constexpr int KV_STAGE = 4 * TILE_BYTES;
constexpr int SMEM_BYTES = KV_OFF + 2 * KV_STAGE;
constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;       // log2 growth of a row's max that triggers a rescale
constexpr float kPShift = 7.0f;        // log2 of P at a row's running max (so P <= 2^15 < fp16 max)
static_assert(SMEM_ALLOC + 512 <= 232448, "dynamic + static shared memory exceeds 227 KB per block");

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// P of two keys as fp16 hi / lo words: hi = fp16(p), lo = fp16(p - hi), the
// same planes as the generic split, with p - hi formed by one
// mixed-precision FMA per key straight from the packed hi (hi * -1 + p, exact)
// instead of unpacking hi to f32 and subtracting: the softmax's exponential
// pass is bound by instruction issue, and this saves two of six instructions
// per key pair.
__device__ __forceinline__ void split2_p(float p0, float p1, uint32_t& hw, uint32_t& lw) {
  asm("{\n"
      " .reg .f16 h0, h1, m1;\n"
      " .reg .f32 l0, l1;\n"
      " cvt.rn.f16x2.f32 %0, %3, %2;\n"
      " mov.b32 {h0, h1}, %0;\n"
      " mov.b16 m1, 0xBC00;\n"
      " fma.rn.f32.f16 l0, h0, m1, %2;\n"
      " fma.rn.f32.f16 l1, h1, m1, %3;\n"
      " cvt.rn.f16x2.f32 %1, l1, l0;\n"
      "}"
      : "=r"(hw), "=r"(lw)
      : "f"(p0), "f"(p1));
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

__device__ __forceinline__ void tmem_ld16_nw(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// Thread i of the warp writes lane (lane_base + i), columns [col, col+16).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16: A is M=128 rows in TMEM lanes,
// two fp16 K-elements per 32-bit column.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <bool ACC>
__device__ __forceinline__ void mma_f16_ts_c(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "n"(ACC ? 1 : 0)
      : "memory");
}

// Bounded wait that ignores the CTA abort flag (exit-path drains).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* err) {
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

__global__ void __launch_bounds__(kThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap mQh, const __grid_constant__ CUtensorMap mQl,
                   const __grid_constant__ CUtensorMap mKh, const __grid_constant__ CUtensorMap mKl,
                   const __grid_constant__ CUtensorMap mVh, const __grid_constant__ CUtensorMap mVl, int n, int heads,
                   __half* __restrict__ o_hi, __half* __restrict__ o_lo, float s_code, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t b_q, b_kvf[2], b_kve[2], b_s[2], b_p[2], b_pv[2], b_done;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag, skip;

  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y, q0 = blockIdx.x * 2 * QT;
  const int T = (n + KT - 1) / KT;

  if (threadIdx.x == 0) {
    skip = *reinterpret_cast<volatile int*>(err) != 0;
    abort_flag = 0;
    mbar_init(&b_q, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&b_kvf[s], 1);
      mbar_init(&b_kve[s], 1);
      mbar_init(&b_s[s], 1);
      mbar_init(&b_p[s], 4);
      mbar_init(&b_pv[s], 1);
    }
    mbar_init(&b_done, 1);
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
      mbar_expect_tx(&b_q, 4 * TILE_BYTES);
      for (int t = 0; t < 2; ++t) {
        tma_load_2d(sm + Q_OFF + 2 * t * TILE_BYTES, &mQh, &b_q, 0, bh * n + q0 + t * QT);
        tma_load_2d(sm + Q_OFF + (2 * t + 1) * TILE_BYTES, &mQl, &b_q, 0, bh * n + q0 + t * QT);
      }
      int issued = 0;
      for (int j = 0; j < T; ++j) {
        const int s = j & 1, k = j >> 1;
        if (!mbar_wait(&b_kve[s], (k & 1) ^ 1, err, kErrWaitEmpty, &abort_flag)) break;
        uint8_t* st = sm + KV_OFF + s * KV_STAGE;
        mbar_expect_tx(&b_kvf[s], KV_STAGE);
        tma_load_2d(st, &mKh, &b_kvf[s], 0, bh * n + j * KT);
        tma_load_2d(st + TILE_BYTES, &mKl, &b_kvf[s], 0, bh * n + j * KT);
        // V^T [64 d][128 keys]: per 64-key half, the hi plane's 64 rows then
        // the lo plane's, one [128 x 64] swizzled N = 128 operand
        for (int h = 0; h < 2; ++h) {
          tma_load_2d(st + (2 + h) * TILE_BYTES, &mVh, &b_kvf[s], j * KT + 64 * h, bh * HD);
          tma_load_2d(st + (2 + h) * TILE_BYTES + TILE_BYTES / 2, &mVl, &b_kvf[s], j * KT + 64 * h, bh * HD);
        }
        ++issued;
      }
      // drain: Q and the last use of each stage
      drain_wait(&b_q, 0, err);
      for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j) drain_wait(&b_kvf[j & 1], (j >> 1) & 1, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16_f32(128, KT);
      constexpr uint32_t id_pv = idesc_f16_f32(128, 2 * HD);
      constexpr uint32_t id_pv_h = idesc_f16_f32(128, HD);  // Pl Vh: the stacked operand's first 64 rows
      bool ok = mbar_wait(&b_q, 0, err, kErrWaitFull, &abort_flag);
      // Descriptor of the tile at byte offset 0 of the aligned region; every
      // operand descriptor below is this plus a constant offset.
      const uint64_t dbase = desc_k_sw128(smem_u32(sm));
      // S_t(j) = Q_t K_j^T into TMEM columns [128 t, 128 t + 128)
      auto issue_s = [&](int t, int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&b_kvf[s], (j >> 1) & 1, err, kErrWaitFull, &abort_flag)) return false;
        tc_fence_after();
        const uint64_t qh = desc_add(dbase, Q_OFF + 2 * t * TILE_BYTES), ql = desc_add(qh, TILE_BYTES);
        const uint64_t kh = desc_add(dbase, KV_OFF + s * KV_STAGE), kl = desc_add(kh, TILE_BYTES);
        const uint32_t d = tmem + t * KT;
        mma_f16_ss_c<false>(d, qh, kh, id_s);
        mma_f16_ss_c<true>(d, qh, kl, id_s);
        mma_f16_ss_c<true>(d, ql, kh, id_s);
#pragma unroll
        for (int kk = 1; kk < HD / 16; ++kk) {
          mma_f16_ss_c<true>(d, desc_add(qh, kk * 32), desc_add(kh, kk * 32), id_s);
          mma_f16_ss_c<true>(d, desc_add(qh, kk * 32), desc_add(kl, kk * 32), id_s);
          mma_f16_ss_c<true>(d, desc_add(ql, kk * 32), desc_add(kh, kk * 32), id_s);
        }
        mma_commit(&b_s[t]);
        return true;
      };
      // O_t += Ph_t(j) [Vh | Vl]_j + Pl_t(j) Vh_j with P_t in TMEM: keys [16 kk, 16 kk + 16)
      // hi at S column 32 (kk / 2) + 8 (kk % 2), lo 16 columns further
      auto issue_pv = [&](int t, int j) -> bool {
        if (!mbar_wait(&b_p[t], j & 1, err, kErrWaitFull, &abort_flag)) return false;
        tc_fence_after();
        const uint64_t v = desc_add(dbase, KV_OFF + (j & 1) * KV_STAGE + 2 * TILE_BYTES);
        const uint32_t d = tmem + O_COL + t * 2 * HD, a = tmem + t * KT;
        mma_f16_ts(d, a, v, id_pv, j > 0 ? 1u : 0u);  // the first product of the tile starts O at j = 0
        mma_f16_ts_c<true>(d, a + 16, v, id_pv_h);
#pragma unroll
        for (int kk = 1; kk < KT / 16; ++kk) {
          const uint64_t dv = desc_add(v, (kk >> 2) * TILE_BYTES + (kk & 3) * 32);
          const uint32_t ah = a + 32 * (kk >> 1) + 8 * (kk & 1);
          mma_f16_ts_c<true>(d, ah, dv, id_pv);
          mma_f16_ts_c<true>(d, ah + 16, dv, id_pv_h);
        }
        mma_commit(&b_pv[t]);
        return true;
      };
      if (ok) ok = issue_s(0, 0) && issue_s(1, 0);
      for (int j = 0; j < T && ok; ++j) {
        if (!(ok = issue_pv(0, j))) break;
        if (j + 1 < T) {
          // S_A(j+1) overwrites P_A(j): wait for P*V_A(j) (P*V_B(j-1) / S_B(j) keep the pipe busy)
          if (!(ok = mbar_wait(&b_pv[0], j & 1, err, kErrWaitAccFull, &abort_flag))) break;
          if (!(ok = issue_s(0, j + 1))) break;
        }
        if (!(ok = issue_pv(1, j))) break;
        mma_commit(&b_kve[j & 1]);  // every MMA reading stage j & 1 has been issued
        if (j + 1 < T) {
          if (!(ok = mbar_wait(&b_pv[1], j & 1, err, kErrWaitAccFull, &abort_flag))) break;
          if (!(ok = issue_s(1, j + 1))) break;
        }
      }
      // Every MMA issued above completes before the CTA can exit.
      mma_commit(&b_done);
      drain_wait(&b_done, 0, err);
    }
  } else {
    // softmax of query tile t: one row per thread, TMEM lane quarter (warp % 4)
    const int t = (warp - 2) >> 2;
    const int qw = warp & 3;
    const uint32_t lane_base = (uint32_t)(32 * qw) << 16;
    const uint32_t s_col = tmem + lane_base + t * KT;
    const uint32_t o_col = tmem + lane_base + O_COL + t * 2 * HD;
    float m = -INFINITY, l = 0.f;  // running max (log2 units) and row sum
    bool ok = true;
    for (int j = 0; j < T; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&b_s[t], j & 1, err, kErrWaitAccFull, &abort_flag));
      if (!ok) break;
      tc_fence_after();
      const int kvalid = n - j * KT;  // < KT only on the last tile
      float mp[8];  // pass 1: eight independent max chains
      // the whole score row; pass 2 reuses chunks 0 and 1 from here and
      // reloads chunks 2 and 3 into registers whose values are dead by then
      uint32_t sr[KT];
      {
#pragma unroll
        for (int c = 0; c < KT / 32; ++c) tmem_ld32_nw(s_col + 32 * c, sr + 32 * c);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 8; ++u) mp[u] = __uint_as_float(sr[u]);  // key 0 is always valid
        if (kvalid >= KT) {
#pragma unroll
          for (int c = 8; c < KT; ++c) mp[c & 7] = fmaxf(mp[c & 7], __uint_as_float(sr[c]));
        } else {
#pragma unroll
          for (int c = 1; c < KT; ++c)
            mp[c & 7] = fmaxf(mp[c & 7], c < kvalid ? __uint_as_float(sr[c]) : -INFINITY);
          for (int u = 1; u < 8; ++u)
            if (u >= kvalid) mp[u] = -INFINITY;
        }
      }
      const float mt = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])),
                             fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7]))) * kLog2e;
      if (j == 0) {
        m = mt;
      } else {
        const bool need = mt > m + kRescale;
        if (__any_sync(0xffffffffu, need)) {
          // O_t holds P*V through tile j-1: wait for it, then rescale the rows that need it
          ok = __all_sync(0xffffffffu, mbar_wait(&b_pv[t], (j - 1) & 1, err, kErrWaitAccFull, &abort_flag));
          if (!ok) break;
          tc_fence_after();
          const float alpha = need ? ex2(m - mt) : 1.0f;
#pragma unroll
          for (int h = 0; h < 2 * HD / 16; ++h) {
            uint32_t ov[16];
            tmem_ld16_nw(o_col + 16 * h, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st16(o_col + 16 * h, ov);
          }
          l *= alpha;
          if (need) m = mt;
        }
      }
      // pass 2: P = 2^(s log2e - m + kPShift) chunk by chunk (32 keys); chunks 0 and 1
      // come from pass 1's registers, chunks 2 and 3 are reloaded while
      // chunks 0 and 1 are converted; P hi / lo go back into the chunk's own
      // columns.
      // P carries a factor 2^kPShift (the row sum carries it too, so it cancels
      // in O / l): keys well below the row's maximum keep their lo plane out of
      // the fp16 subnormal range.
      const float mneg = kPShift - m;
      float rp[4] = {0.f, 0.f, 0.f, 0.f};  // four independent sum chains
      tmem_ld32_nw(s_col + 64, sr + 64);    // chunk 2
#pragma unroll
      for (int c = 0; c < KT / 32; ++c) {
        // chunk c's 32 scores: 0 -> sr[0..32), 1 -> sr[32..64), 2 -> sr[64..96), 3 -> sr[0..32) (reloaded)
        uint32_t* cur = sr + (c == 1 ? 32 : (c == 2 ? 64 : 0));
        if (c == 1) tmem_ld32_nw(s_col + 96, sr);  // chunk 3, over chunk 0's dead values
        if (c == 2) tmem_wait_ld();                // chunks 2 and 3 have landed
        const int lim = kvalid - 32 * c;  // keys of this chunk that are valid (>= 32: all)
        uint32_t hv[16], lv[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          float p0 = ex2(fmaf(__uint_as_float(cur[2 * u]), kLog2e, mneg));
          float p1 = ex2(fmaf(__uint_as_float(cur[2 * u + 1]), kLog2e, mneg));
          if (lim < 32) {
            p0 = 2 * u < lim ? p0 : 0.f;
            p1 = 2 * u + 1 < lim ? p1 : 0.f;
          }
          rp[u & 3] += p0 + p1;
          split2_p(p0, p1, hv[u], lv[u]);
        }
        tmem_st16(s_col + 32 * c, hv);
        tmem_st16(s_col + 32 * c + 16, lv);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b_p[t]);
      l += (rp[0] + rp[1]) + (rp[2] + rp[3]);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&b_pv[t], (T - 1) & 1, err, kErrWaitAccFull, &abort_flag));
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const float inv_code = s_code != 0.0f ? 1.0f / s_code : 0.0f;
      const int img = bh / heads, head = bh % heads;
      // this warp's 32 query rows leave as one block through its 4 KB of the
      // tile's Q region (free: the tile's last S MMA completed before its
      // last softmax), whole sectors per store
      uint4* stage = reinterpret_cast<uint4*>(sm + Q_OFF + 2 * t * TILE_BYTES + qw * 4096);
      const int wq0 = q0 + t * QT + 32 * qw;  // query row of lane 0
      const size_t ostride = (size_t)heads * HD * 2;
      const size_t obase = ((size_t)img * n + wq0) * (size_t)(heads * HD) + head * HD;
      if (s_code != 0.0f) {
        // signed-byte codes for the o_proj input scale: 64 bytes per row
        // (row stride heads * 64 bytes)
        uint4 w[4];
#pragma unroll
        for (int h = 0; h < HD / 16; ++h) {
          uint32_t ov[16], ol[16];
          tmem_ld16_nw(o_col + 16 * h, ov);       // P * Vh
          tmem_ld16_nw(o_col + HD + 16 * h, ol);  // P * Vl
          tmem_wait_ld();
          uint32_t b4[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint32_t x = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float v = (__uint_as_float(ov[4 * u + e]) + __uint_as_float(ol[4 * u + e])) * inv;
              x |= ((uint32_t)(int)srq_code(v, s_code, inv_code) & 0xFFu) << (8 * e);
            }
            b4[u] = x;
          }
          w[h] = make_uint4(b4[0], b4[1], b4[2], b4[3]);
        }
        warp_store_block<64>(stage, w, reinterpret_cast<char*>(o_hi) + obase, (size_t)heads * HD, n - wq0, lane);
      }
      // hi and lo planes one at a time, the O columns re-read from TMEM chunk
      // by chunk so that only the plane's eight words stay live
      const int planes = s_code != 0.0f ? 0 : 2;
#pragma unroll 1
      for (int pl = 0; pl < planes; ++pl) {
        uint4 w[8];
#pragma unroll
        for (int h = 0; h < HD / 16; ++h) {
          uint32_t ov[16], ol[16];
          tmem_ld16_nw(o_col + 16 * h, ov);       // P * Vh
          tmem_ld16_nw(o_col + HD + 16 * h, ol);  // P * Vl
          tmem_wait_ld();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t q4[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i = 8 * half + 2 * u;
              const float x0 = (__uint_as_float(ov[i]) + __uint_as_float(ol[i])) * inv;
              const float x1 = (__uint_as_float(ov[i + 1]) + __uint_as_float(ol[i + 1])) * inv;
              uint32_t hw, lw;
              split2_f16(x0, x1, hw, lw);
              q4[u] = pl ? lw : hw;
            }
            w[2 * h + half] = make_uint4(q4[0], q4[1], q4[2], q4[3]);
          }
        }
        warp_store_block<128>(stage, w, reinterpret_cast<char*>((pl ? o_lo : o_hi) + obase), ostride, n - wq0, lane);
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
                                __half* o_hi, __half* o_lo, float s_code, int* err, cudaStream_t st) {
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
  dim3 grid((n + 2 * QT - 1) / (2 * QT), bh);
  attn_tc_kernel<<<grid, kThreads, SMEM_ALLOC, st>>>(mQh, mQl, mKh, mKl, mVh, mVl, n, heads, o_hi, o_lo, s_code, err);
  return cudaGetLastError();
}

}  // namespace g4m
