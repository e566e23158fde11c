// tcgen05 GEMM for the QAT / F32 / BF16 linears of the Gemma 4 E2B media
// towers, with the reference's per-channel math fused into the epilogue.
//
// Replaces, on the device:
//   runQatI8LinearWebGpu       src/kernels/qat.ts:601-759 (CPU twin 458-487)
//   runPackedQatLinearWebGpu   src/kernels/qat.ts:263-432 (CPU twin 215-247)
//   runF32LinearRowsWebGpu     src/kernels/qat.ts:35-157  (CPU twin 6-33)
//   runVisionPatchEmbeddingWebGpu src/vision/kernels.ts:1021-1194 (matmul part)
//   and, fused into epilogues, runVisionMlpActivationWebGpu, runSiluActivationWebGpu,
//   runGluActivationWebGpu, the q/k/v head RMSNorm and runVisionRopeWebGpu.
//
// D[M,N] = sum over terms of A_t[M,K] * B_t[N,K]^T, fp16 operands, f32
// accumulation in tensor memory.  Activations are carried as two fp16
// planes (hi = fp16(x), lo = fp16(x - hi)), so one QAT linear is
// hi*W + lo*W (int8 / unsigned-code weights are exact in fp16) and an F32
// linear adds hi*W_lo: fp32-grade results from the fp16 tensor path.  The
// tensor core truncates each product to the running accumulator's precision,
// so callers can split K into chunks (GemmArgs::chunk_kb) that are summed
// with round-to-nearest f32 adds.  One-term GEMMs run on statically
// quantised inputs: signed-byte codes x int8 weights, tcgen05 kind::i8,
// exact int32 accumulation.
//
// Kernel structure (one CTA per SM, persistent over output tiles):
//   warp 0       TMA producer (one elected lane), STAGES-deep smem ring
//   warp 1       TMEM owner + MMA issuer (one lane), 2 accumulator buffers
//   warps 2..9   two epilogue warpgroups (column halves of each tile):
//                TMEM -> registers -> fused math -> global
// Every wait is bounded; a timeout records an error word and the CTA
// unwinds, drains its own in-flight copies and frees its TMEM.
#include "g4m_kernels.h"
#include "g4m_sm100.cuh"
#include "runtime_internal.h"

#include <algorithm>
#include <mutex>

namespace g4m {

constexpr int BM = 128;
constexpr int BK = 64;      // k-block of the fp16 GEMMs (128 bytes of a row)
constexpr int BK_I8 = 128;  // k-block of the int8 GEMMs (the same 128 bytes)
constexpr int kEpiGroups = 2;                       // epilogue warpgroups
constexpr int kGemmThreads = 64 + 128 * kEpiGroups;  // producer, MMA, epilogue

template <int BN, int TERMS, int AMODE = 0>
struct GemmCfg {
  static constexpr int NA = (TERMS >= 2 || AMODE == 2) ? 2 : 1;
  static constexpr int NB = TERMS == 3 ? 2 : 1;
  static constexpr int A_BYTES = BM * 128;  // one 128-byte swizzled row per tile row and k-block
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = NA * A_BYTES + NB * B_BYTES;
  static constexpr int STAGES = (196608 / STAGE_BYTES) > 6 ? 6 : (196608 / STAGE_BYTES);
  static constexpr int EPI_STAGE = 4096;  // per epilogue warp: a 32-row x 128-byte store block
  static constexpr int SMEM = STAGES * STAGE_BYTES + 4 * kEpiGroups * EPI_STAGE + 1024;
  static_assert(SMEM + 1024 <= 232448, "pipeline + epilogue stages exceed 227 KB of shared memory");
  static constexpr int TMEM_COLS = 2 * BN;
};

// srqScalar (src/kernels/qat.ts:489-492): clamp(round(v/s), -128, 127) * s.
__device__ __forceinline__ float srq_f(float v, float s) {
  if (s == 0.0f) return v;
  return srq_code(v, s, 1.0f / s) * s;
}

// geluPytorchTanh (src/vision/kernels.ts:155-159):
// 0.5 x (1 + tanh(u)) = x * sigmoid(2u), u = sqrt(2/pi) (x + 0.044715 x^3).
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
  return x * sigmoid_f(2.0f * u);
}

// n values -> fp16 hi/lo planes (16-byte stores; n multiple of 8, 16-byte aligned)
__device__ __forceinline__ void store_f16x2_row(__half* hi, __half* lo, const float* v, int n) {
  for (int j = 0; j < n; j += 8) {
    uint32_t hv[4], lv[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) split2_f16(v[j + 2 * u], v[j + 2 * u + 1], hv[u], lv[u]);
    *reinterpret_cast<uint4*>(hi + j) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
    *reinterpret_cast<uint4*>(lo + j) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
  }
}

// One 64-column head of the vision q | k | v projection: per-channel weight
// scale x row scale, output srq, then the head RMSNorm (weight nw, or none
// for v: runVisionRmsNormCpu, src/vision/kernels.ts:5-32).
__device__ __forceinline__ void load_scales32(const float* p, float* s);
__device__ __forceinline__ void qkv_head_norm(float* v, const float* col_scale, float rsw, float so, float eps,
                                              const float* nw) {
  float sc[32];
  load_scales32(col_scale, sc);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = (v[j] * rsw) * sc[j];
  load_scales32(col_scale + 32, sc);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[32 + j] = (v[32 + j] * rsw) * sc[j];
  if (so != 0.0f) {
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = srq_f(v[j], so);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 64; ++j) ss = fmaf(v[j], v[j], ss);
  const float inv = 1.0f / sqrtf(ss / 64.0f + eps);
  if (nw) {
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = (v[j] * inv) * __ldg(nw + j);
  } else {
#pragma unroll
    for (int j = 0; j < 64; ++j) v[j] = v[j] * inv;
  }
}

// 32 consecutive per-channel scales (broadcast loads, 16-byte aligned)
__device__ __forceinline__ void load_scales32(const float* p, float* s) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 v = __ldg(q + i);
    s[4 * i] = v.x;
    s[4 * i + 1] = v.y;
    s[4 * i + 2] = v.z;
    s[4 * i + 3] = v.w;
  }
}

// 32 floats as 16-byte words: f32, fp16 hi, fp16 lo (x - hi), or srq codes.
__device__ __forceinline__ void pack_f32(const float* v, uint4 (&o)[8]) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    o[c] = make_uint4(__float_as_uint(v[4 * c]), __float_as_uint(v[4 * c + 1]), __float_as_uint(v[4 * c + 2]),
                      __float_as_uint(v[4 * c + 3]));
}
template <bool LO>
__device__ __forceinline__ void pack_f16(const float* v, uint4* o, int nwords16) {
#pragma unroll
  for (int c = 0; c < nwords16; ++c) {
    uint32_t w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint32_t hw, lw;
      split2_f16(v[8 * c + 2 * u], v[8 * c + 2 * u + 1], hw, lw);
      w[u] = LO ? lw : hw;
    }
    o[c] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}
// 32 floats -> srq codes as signed bytes (two 16-byte words).
__device__ __forceinline__ void pack_codes_i8(const float* v, float sc, uint4 (&o)[2]) {
  const float inv = 1.0f / sc;
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    uint32_t x = 0;
#pragma unroll
    for (int u = 0; u < 4; ++u) x |= ((uint32_t)(int)srq_code(v[4 * i + u], sc, inv) & 0xFFu) << (8 * u);
    w[i] = x;
  }
  o[0] = make_uint4(w[0], w[1], w[2], w[3]);
  o[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

// 32 accumulator columns of this warp's lanes as floats: f32 accumulators as
// they are, s32 accumulators (int8 GEMMs) converted.
template <bool I8>
__device__ __forceinline__ void acc_ld32(uint32_t taddr, float* v) {
  tmem_ld32(taddr, v);
  if (I8) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (float)__float_as_int(v[i]);
  }
}

template <int BN, int TERMS, int EPI, int AMODE>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap mA0, const __grid_constant__ CUtensorMap mA1,
                   const __grid_constant__ CUtensorMap mB0, const __grid_constant__ CUtensorMap mB1,
                   const __grid_constant__ CUtensorMap mA2, GemmArgs a) {
  static_assert(AMODE == 0 || TERMS == 1, "per-region A selection runs on integer codes (one term)");
  using C = GemmCfg<BN, TERMS, AMODE>;
  // One term means integer codes (static input quantisation) against int8
  // weights: signed bytes, kind::i8 MMAs and exact int32 accumulation.
  constexpr bool I8 = TERMS == 1;
  constexpr int KBE = I8 ? BK_I8 : BK;  // elements per k-block
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bar_full[C::STAGES], bar_empty[C::STAGES], bar_accf[2], bar_acce[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag, skip;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_n = a.N / BN, tiles_m = (a.M + BM - 1) / BM, tiles = tiles_m * tiles_n;
  const int kblocks = a.K / KBE;

  if (threadIdx.x == 0) skip = *reinterpret_cast<volatile int*>(a.err) != 0;
  __syncthreads();
  if (skip) return;  // an earlier kernel on this device already failed
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bar_full[s], 1);
      mbar_init(&bar_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bar_accf[b], 1);
      mbar_init(&bar_acce[b], 4 * kEpiGroups);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&mA0);
    prefetch_tmap(&mB0);
    if (C::NA == 2 || AMODE == 1) prefetch_tmap(&mA1);
    if (C::NB == 2) prefetch_tmap(&mB1);
    if (AMODE == 1) prefetch_tmap(&mA2);
  }
  if (warp == 1) tmem_alloc(&tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  auto sA = [&](int s, int t) { return smem + s * C::STAGE_BYTES + t * C::A_BYTES; };
  auto sB = [&](int s, int t) { return smem + s * C::STAGE_BYTES + C::NA * C::A_BYTES + t * C::B_BYTES; };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int mb = tile / tiles_n, nb = tile % tiles_n;
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t r = it / C::STAGES;
          if (!mbar_wait(&bar_empty[s], (r & 1) ^ 1, a.err, kErrWaitEmpty, &abort_flag)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bar_full[s], C::STAGE_BYTES);
          if (AMODE == 1) {
            const int region = nb * BN / a.proj_width;
            const CUtensorMap* ma = region == 0 ? &mA0 : (region == 1 ? &mA1 : &mA2);
            tma_load_2d(sA(s, 0), ma, &bar_full[s], kb * KBE, mb * BM);
          } else {
            tma_load_2d(sA(s, 0), &mA0, &bar_full[s], kb * KBE, mb * BM);
          }
          if (C::NA == 2) tma_load_2d(sA(s, 1), &mA1, &bar_full[s], kb * KBE, mb * BM);
          tma_load_2d(sB(s, 0), &mB0, &bar_full[s], kb * KBE, nb * BN);
          if (C::NB == 2) tma_load_2d(sB(s, 1), &mB1, &bar_full[s], kb * KBE, nb * BN);
        }
      }
      // Drain: the last use of every stage must have landed before exit.
      const uint32_t first = it > (uint32_t)C::STAGES ? it - C::STAGES : 0;
      for (uint32_t j = first; j < it; ++j) {
        const uint32_t b = smem_u32(&bar_full[j % C::STAGES]);
        const long long t0 = clock64();
        while (!mbar_try_wait(b, (j / C::STAGES) & 1)) {
          if (clock64() - t0 > kWaitCycles) {
            atomicCAS(a.err, 0, kErrWaitDrain);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = I8 ? idesc_i8_s32(BM, BN) : idesc_f16_f32(BM, BN);
      constexpr uint32_t idesc_half = I8 ? idesc_i8_s32(BM, BN / 2) : idesc_f16_f32(BM, BN / 2);
      // K chunks of every tile go to the two TMEM buffers alternately, in
      // one sequence over all tiles of this CTA: chunk k lands in buffer k & 1
      // (its (k >> 1)-th use).  The epilogue keeps each tile's running total
      // in the buffer of its latest chunk (chunk_kb == 0: one chunk per tile,
      // plain double buffering across tiles).
      uint32_t it = 0, kc = 0;  // k-blocks and chunks issued so far
      bool ok = true;
      const uint64_t dbase = desc_k_sw128(smem_u32(smem));
      const int chunk_len = a.chunk_kb > 0 ? a.chunk_kb : kblocks;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        uint32_t b = 0, d = tmem_base;
        int left = 0;  // k-blocks left in the current chunk
        for (int kb = 0; kb < kblocks; ++kb, ++it) {
          const bool first = left == 0;
          if (first) left = chunk_len;
          const bool last = --left == 0 || kb + 1 == kblocks;
          if (first) {
            b = kc & 1;
            if (!mbar_wait(&bar_acce[b], ((kc >> 1) & 1) ^ 1, a.err, kErrWaitAccEmpty, &abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            d = tmem_base + b * BN;
          }
          const int s = it % C::STAGES;
          const uint32_t r = it / C::STAGES;
          if (!mbar_wait(&bar_full[s], r & 1, a.err, kErrWaitFull, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ga = desc_add(dbase, s * C::STAGE_BYTES);   // A (hi) of stage s
          const uint64_t gb = desc_add(ga, C::NA * C::A_BYTES);       // B (hi) of stage s
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 32 bytes of K per MMA: 16 fp16 or 32 int8 elements
            const uint64_t da0 = desc_add(ga, k * 32), db0 = desc_add(gb, k * 32);
            const uint32_t acc = (!first || k > 0) ? 1u : 0u;
            if (AMODE == 2) {
              // halves of the B tile (rows [0, BN/2) and [BN/2, BN)) against their own codes
              const uint64_t da1 = desc_add(ga, C::A_BYTES + k * 32), db1 = desc_add(gb, (BN / 2) * 128 + k * 32);
              if (I8) {
                mma_i8_ss(d, da0, db0, idesc_half, acc);
                mma_i8_ss(d + BN / 2, da1, db1, idesc_half, acc);
              } else {
                mma_f16_ss(d, da0, db0, idesc_half, acc);
                mma_f16_ss(d + BN / 2, da1, db1, idesc_half, acc);
              }
              continue;
            }
            if (I8) {
              if (k == 0) mma_i8_ss(d, da0, db0, idesc, acc);
              else mma_i8_ss_c<true>(d, da0, db0, idesc);
              continue;
            }
            if (k == 0) mma_f16_ss(d, da0, db0, idesc, acc);
            else mma_f16_ss_c<true>(d, da0, db0, idesc);
            if (TERMS >= 2) mma_f16_ss_c<true>(d, desc_add(ga, C::A_BYTES + k * 32), db0, idesc);
            if (TERMS == 3) mma_f16_ss_c<true>(d, da0, desc_add(gb, C::B_BYTES + k * 32), idesc);
          }
          mma_commit(&bar_empty[s]);
          if (last) {
            mma_commit(&bar_accf[b]);
            ++kc;
            left = 0;
          }
        }
      }
      // Let the last stage-release commits land before the CTA can exit.
      if (ok && !abort_flag) {
        const uint32_t first = it > (uint32_t)C::STAGES ? it - C::STAGES : 0;
        for (uint32_t j = first; j < it; ++j)
          if (!mbar_wait(&bar_empty[j % C::STAGES], (j / C::STAGES) & 1, a.err, kErrWaitDrain, &abort_flag)) break;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // kEpiGroups warpgroups split every tile's columns; warp w reads TMEM
    // lanes 32*(w%4) .. +31 (one accumulator row per thread).
    const int q = warp & 3;
    const int eg = (warp - 2) >> 2;
    const int row_in_tile = 32 * q + lane;
    uint4* stage = reinterpret_cast<uint4*>(smem + C::STAGES * C::STAGE_BYTES + (warp - 2) * C::EPI_STAGE);
    const int nchunks = (!I8 && a.chunk_kb) ? (kblocks + a.chunk_kb - 1) / a.chunk_kb : 1;
    const uint32_t lq = (uint32_t)(32 * q) << 16;
    uint32_t kc = 0;  // chunks consumed so far (the MMA warp's sequence)
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
      // tcgen05.ld is warp-collective: every lane takes the same branch.
      bool ok = __all_sync(0xffffffffu, mbar_wait(&bar_accf[kc & 1], (kc >> 1) & 1, a.err, kErrWaitAccFull, &abort_flag));
      if (!ok) break;
      ++kc;
      // Every later chunk of the tile: total (previous buffer) + chunk (its
      // buffer) with round-to-nearest f32 adds, written into the chunk's
      // buffer; the previous buffer is handed back as soon as it is read.
      for (int c = 1; c < nchunks && ok; ++c, ++kc) {
        const uint32_t cb = kc & 1, tb_ = cb ^ 1;
        ok = __all_sync(0xffffffffu, mbar_wait(&bar_accf[cb], (kc >> 1) & 1, a.err, kErrWaitAccFull, &abort_flag));
        if (!ok) break;
        tc_fence_after();
        constexpr int COLS = BN / kEpiGroups;  // this warpgroup's columns
#pragma unroll
        for (int p = 0; p < COLS / 32; ++p) {
          const int col = eg * COLS + 32 * p;
          uint32_t x[32], y[32];
          tmem_ld32_raw(tmem_base + lq + tb_ * BN + col, x);
          tmem_ld32_raw(tmem_base + lq + cb * BN + col, y);
          tmem_wait_ld_all();
          if (p == COLS / 32 - 1) {  // the previous total is fully read: its buffer may take the next chunk
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar_acce[tb_]);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) y[i] = __float_as_uint(__uint_as_float(x[i]) + __uint_as_float(y[i]));
          tmem_st32(tmem_base + lq + cb * BN + col, y);
        }
        tmem_wait_st_all();
      }
      if (!ok) break;
      const uint32_t buf = (kc - 1) & 1;  // the buffer holding the tile's total
      tc_fence_after();
      const int mb = tile / tiles_n, nb = tile % tiles_n;
      const uint32_t tb = tmem_base + ((uint32_t)(32 * q) << 16) + buf * BN;
      const int row = mb * BM + row_in_tile;
      const bool valid = row < a.M;
      const int wrow0 = mb * BM + 32 * q, wrows = a.M - wrow0;  // this warp's 32-row block
      const float rs = a.row_scale;

      if (EPI == EPI_F32 || EPI == EPI_PATCH || EPI == EPI_SILU) {
        constexpr int NCH = BN / 32 / kEpiGroups;
        const int* pxy = (EPI == EPI_PATCH && valid) ? a.pos_xy + 2 * (size_t)(row % a.rows_per_image) : nullptr;
#pragma unroll 1
        for (int c = eg * NCH; c < (eg + 1) * NCH; ++c) {
          float v[32];
          acc_ld32<I8>(tb + c * 32, v);
          if (valid) {
            const int n0 = nb * BN + c * 32;
            if (EPI == EPI_PATCH) {
              const float* px = a.posx_rows + (size_t)pxy[0] * a.N + n0;
              const float* py = a.posy_rows + (size_t)pxy[1] * a.N + n0;
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = (v[j] + px[j]) + py[j];
            } else {
              // fused projections (proj_width > 0) keep their own output scales
              const int which = a.proj_width > 0 ? n0 / a.proj_width : 0;
              const float so = which == 0 ? a.s_out : (which == 1 ? a.s_out_b : a.s_out_c);
              const float rsw = AMODE == 1 ? (which == 0 ? rs : (which == 1 ? a.row_scale_b : a.row_scale_c)) : rs;
              if (a.col_scale) {
                float sc[32];
                load_scales32(a.col_scale + n0, sc);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = (v[j] * rsw) * sc[j];
              }
              if (so != 0.0f) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = srq_f(v[j], so);
              }
              if (EPI == EPI_SILU) {
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = v[j] * sigmoid_f(v[j]);  // runSiluActivationCpu
              } else if (a.bias) {
                float bs[32];
                load_scales32(a.bias + n0, bs);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = v[j] + bs[j];
              }
            }
          }
          const int n0 = nb * BN + c * 32;
          if (EPI == EPI_SILU) {
            char* bh_ = reinterpret_cast<char*>(a.out_hi + (size_t)wrow0 * a.ldh + n0);
            if (a.s_code != 0.0f) {  // signed-byte codes for the next GEMM (ldh bytes per row)
              uint4 w[2];
              pack_codes_i8(v, a.s_code, w);
              warp_store_block<32>(stage, w, reinterpret_cast<char*>(a.out_hi) + (size_t)wrow0 * a.ldh + n0,
                                   (size_t)a.ldh, wrows, lane);
            } else {
              uint4 w[4];
              pack_f16<false>(v, w, 4);
              warp_store_block<64>(stage, w, bh_, (size_t)a.ldh * 2, wrows, lane);
              pack_f16<true>(v, w, 4);
              warp_store_block<64>(stage, w, reinterpret_cast<char*>(a.out_lo + (size_t)wrow0 * a.ldh + n0),
                                   (size_t)a.ldh * 2, wrows, lane);
            }
          } else {
            uint4 w[8];
            pack_f32(v, w);
            warp_store_block<128>(stage, w, reinterpret_cast<char*>(a.out_f32 + (size_t)wrow0 * a.ldo + n0),
                                  (size_t)a.ldo * 4, wrows, lane);
          }
        }
      } else if (EPI == EPI_GELU_GATE || EPI == EPI_GLU) {
        // Tile columns [0, BN/2) carry the first operand (gate / GLU value),
        // [BN/2, BN) the second (up / GLU gate) for the same output columns.
        constexpr int NP = BN / 64 / kEpiGroups;
#pragma unroll 1
        for (int c = eg * NP; c < (eg + 1) * NP; ++c) {
          float g[32], u[32];
          acc_ld32<I8>(tb + c * 32, g);
          acc_ld32<I8>(tb + BN / 2 + c * 32, u);
          if (valid) {
            const int ng = nb * BN + c * 32, nu = nb * BN + BN / 2 + c * 32;
            float sg[32], su[32];
            load_scales32(a.col_scale + ng, sg);
            load_scales32(a.col_scale + nu, su);
            const float rsu = AMODE == 2 ? a.row_scale_b : rs;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              g[j] = (g[j] * rs) * sg[j];
              u[j] = (u[j] * rsu) * su[j];
            }
            if (a.s_out != 0.0f || a.s_out_b != 0.0f) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                g[j] = srq_f(g[j], a.s_out);
                u[j] = srq_f(u[j], a.s_out_b);
              }
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (EPI == EPI_GELU_GATE) g[j] = gelu_tanh_f(g[j]) * u[j];  // runVisionMlpActivationCpu
              else g[j] = g[j] * sigmoid_f(u[j]);                          // runGluActivationCpu
            }
          }
          const int no = nb * (BN / 2) + c * 32;
          if (EPI == EPI_GELU_GATE) {
            char* bh_ = reinterpret_cast<char*>(a.out_hi + (size_t)wrow0 * a.ldh + no);
            if (a.s_code != 0.0f) {  // signed-byte codes for the next GEMM (ldh bytes per row)
              uint4 w[2];
              pack_codes_i8(g, a.s_code, w);
              warp_store_block<32>(stage, w, reinterpret_cast<char*>(a.out_hi) + (size_t)wrow0 * a.ldh + no,
                                   (size_t)a.ldh, wrows, lane);
            } else {
              uint4 w[4];
              pack_f16<false>(g, w, 4);
              warp_store_block<64>(stage, w, bh_, (size_t)a.ldh * 2, wrows, lane);
              pack_f16<true>(g, w, 4);
              warp_store_block<64>(stage, w, reinterpret_cast<char*>(a.out_lo + (size_t)wrow0 * a.ldh + no),
                                   (size_t)a.ldh * 2, wrows, lane);
            }
          } else {
            uint4 w[8];
            pack_f32(g, w);
            warp_store_block<128>(stage, w, reinterpret_cast<char*>(a.out_f32 + (size_t)wrow0 * a.ldo + no),
                                  (size_t)a.ldo * 4, wrows, lane);
          }
        }
      } else if (EPI == EPI_QKV_VISION) {
        // 64-column head groups: scale (+srq), head RMSNorm, 2-D RoPE (q, k),
        // scatter to the attention layouts.
        constexpr int NH = BN / 64 / kEpiGroups;
        const int n_tile0 = nb * BN;
        const int which = n_tile0 / a.proj_width;  // 0 q, 1 k, 2 v
        const int head0 = (n_tile0 % a.proj_width) / 64;
        const int img = valid ? row / a.rows_per_image : 0;
        const int tok = valid ? row % a.rows_per_image : 0;
        const float so = which == 0 ? a.s_out : (which == 1 ? a.s_out_b : a.s_out_c);
        const float rsw = AMODE == 1 ? (which == 0 ? rs : (which == 1 ? a.row_scale_b : a.row_scale_c)) : rs;
        const float* nw = which == 0 ? a.qn_w : (which == 1 ? a.kn_w : nullptr);
        if (which < 2) {
          // the warp's 32 rows are consecutive tokens of one image when the
          // image's rows are a multiple of 32: then q / k leave as one block
          const bool block = a.rows_per_image % 32 == 0;
#pragma unroll 1
          for (int hh = eg * NH; hh < (eg + 1) * NH; ++hh) {
            float v[64];
            acc_ld32<I8>(tb + hh * 64, v);
            acc_ld32<I8>(tb + hh * 64 + 32, v + 32);
            if (valid) {
              qkv_head_norm(v, a.col_scale + n_tile0 + hh * 64, rsw, so, a.eps, nw);
              const float4* cs = reinterpret_cast<const float4*>(a.rope_cs) + (size_t)tok * 16;
#pragma unroll
              for (int p = 0; p < 2; ++p) {  // rotate-half pairs (f, f + 16) in place
#pragma unroll
                for (int f = 0; f < 16; f += 2) {
                  const float4 c2 = __ldg(cs + (p * 16 + f) / 2);  // (cos, sin) of f and f + 1
                  const float x1 = v[p * 32 + f], x2 = v[p * 32 + 16 + f];
                  const float y1 = v[p * 32 + f + 1], y2 = v[p * 32 + 16 + f + 1];
                  v[p * 32 + f] = x1 * c2.x - x2 * c2.y;
                  v[p * 32 + 16 + f] = x2 * c2.x + x1 * c2.y;
                  v[p * 32 + f + 1] = y1 * c2.z - y2 * c2.w;
                  v[p * 32 + 16 + f + 1] = y2 * c2.z + y1 * c2.w;
                }
              }
            }
            if (block) {
              const size_t bh0 = (size_t)(wrow0 / a.rows_per_image) * a.heads + head0 + hh;
              const size_t r0 = bh0 * a.rows_per_image + wrow0 % a.rows_per_image;
              uint4 w[8];
              pack_f16<false>(v, w, 8);
              warp_store_block<128>(stage, w, reinterpret_cast<char*>((which == 0 ? a.q_hi : a.k_hi) + r0 * 64), 128,
                                    wrows, lane);
              pack_f16<true>(v, w, 8);
              warp_store_block<128>(stage, w, reinterpret_cast<char*>((which == 0 ? a.q_lo : a.k_lo) + r0 * 64), 128,
                                    wrows, lane);
            } else if (valid) {
              const size_t bh = (size_t)img * a.heads + head0 + hh;
              __half* dh = (which == 0 ? a.q_hi : a.k_hi) + (bh * a.rows_per_image + tok) * 64;
              __half* dl = (which == 0 ? a.q_lo : a.k_lo) + (bh * a.rows_per_image + tok) * 64;
              store_f16x2_row(dh, dl, v, 64);
            }
          }
        } else {
          // V^T: lanes of consecutive tokens pair up (one 32-bit store per
          // dimension and lane: even lanes the hi plane, odd lanes the lo
          // plane) when no pair can straddle two images; rows at or past M
          // then come in whole pairs, and every lane computes so that the
          // shuffles are full.
          const bool pair_v = (a.rows_per_image & 1) == 0;
#pragma unroll 1
          for (int hh = eg * NH; hh < (eg + 1) * NH; ++hh) {
            float v[64];
            acc_ld32<I8>(tb + hh * 64, v);
            acc_ld32<I8>(tb + hh * 64 + 32, v + 32);
            if (!valid && !pair_v) continue;
            qkv_head_norm(v, a.col_scale + n_tile0 + hh * 64, rsw, so, a.eps, nullptr);
            const size_t bh = (size_t)img * a.heads + head0 + hh;
            if (pair_v) {
              const bool odd = lane & 1;  // tok has the parity of the lane (tiles start at even rows)
              __half* dst = (odd ? a.vt_lo : a.vt_hi) + bh * 64 * (size_t)a.vt_pitch + (tok & ~1);
#pragma unroll
              for (int j = 0; j < 64; j += 2) {
                // hi / lo of dims j and j + 1 as half2 words; even lanes send their lo
                // word and keep the hi one, odd lanes the reverse
                uint32_t hw, lw;
                split2_f16(v[j], v[j + 1], hw, lw);
                const uint32_t other = __shfl_xor_sync(0xffffffffu, odd ? hw : lw, 1);
                const uint32_t own = odd ? lw : hw;
                // (even token, odd token) for dim j, then for dim j + 1
                const uint32_t w0 = odd ? __byte_perm(other, own, 0x5410) : __byte_perm(own, other, 0x5410);
                const uint32_t w1 = odd ? __byte_perm(other, own, 0x7632) : __byte_perm(own, other, 0x7632);
                if (valid) {
                  *reinterpret_cast<uint32_t*>(dst + (size_t)j * a.vt_pitch) = w0;
                  *reinterpret_cast<uint32_t*>(dst + (size_t)(j + 1) * a.vt_pitch) = w1;
                }
              }
            } else {
              __half* dh = a.vt_hi + bh * 64 * (size_t)a.vt_pitch + tok;
              __half* dl = a.vt_lo + bh * 64 * (size_t)a.vt_pitch + tok;
#pragma unroll
              for (int j = 0; j < 64; ++j) {
                __half h, l;
                split_f16(v[j], h, l);
                dh[(size_t)j * a.vt_pitch] = h;
                dl[(size_t)j * a.vt_pitch] = l;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_acce[buf]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// fp16 matrix [rows, cols] (row-major), box 64 columns x box_rows rows, 128B swizzle.
bool make_tmap_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || (cols % 64) != 0 || (reinterpret_cast<uintptr_t>(base) % 16) != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// int8 matrix [rows, cols] (row-major), box 128 columns x box_rows rows, 128B swizzle.
bool make_tmap_i8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || (cols % 128) != 0 || (reinterpret_cast<uintptr_t>(base) % 16) != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_f16_any(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                       uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || !base || (pitch_elems * 2) % 16 != 0 || pitch_elems < cols ||
      (reinterpret_cast<uintptr_t>(base) % 16) != 0)
    return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {pitch_elems * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

static int g_num_sms(int dev) {
  static int cache[64] = {0};
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = v > 0 ? v : 148;
  }
  return cache[dev];
}

template <int BN, int TERMS, int EPI, int AMODE>
static cudaError_t launch_t(const GemmOperands& op, const GemmArgs& args, cudaStream_t st, int max_ctas) {
  using C = GemmCfg<BN, TERMS, AMODE>;
  auto kern = gemm_tc_kernel<BN, TERMS, EPI, AMODE>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  if (AMODE == 1 && (args.proj_width <= 0 || args.proj_width % BN != 0 || args.N > 3 * args.proj_width))
    return cudaErrorInvalidValue;  // every tile must sit inside one region
  // one-term GEMMs read signed-byte codes and int8 weights; the rest fp16 planes
  auto tmap = [](CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    return TERMS == 1 ? make_tmap_i8(m, base, rows, cols, box_rows) : make_tmap_f16(m, base, rows, cols, box_rows);
  };
  CUtensorMap mA0, mA1, mA2, mB0, mB1;
  if (!tmap(&mA0, op.a_hi, args.M, args.K, BM)) return cudaErrorInvalidValue;
  if (!tmap(&mB0, op.b_hi, args.N, args.K, BN)) return cudaErrorInvalidValue;
  mA1 = mA0;
  mA2 = mA0;
  mB1 = mB0;
  if ((C::NA == 2 || AMODE == 1) && !tmap(&mA1, op.a_lo, args.M, args.K, BM)) return cudaErrorInvalidValue;
  if (AMODE == 1 && args.N > 2 * args.proj_width && !tmap(&mA2, op.a_c, args.M, args.K, BM))
    return cudaErrorInvalidValue;
  if (C::NB == 2 && !tmap(&mB1, op.b_lo, args.N, args.K, BN)) return cudaErrorInvalidValue;
  const int tiles = ((args.M + BM - 1) / BM) * (args.N / BN);
  int grid = std::min(tiles, g_num_sms(dev));
  if (max_ctas > 0) grid = std::min(grid, max_ctas);
  if (grid <= 0) return cudaSuccess;
  kern<<<grid, kGemmThreads, C::SMEM, st>>>(mA0, mA1, mB0, mB1, mA2, args);
  return cudaGetLastError();
}

cudaError_t gemm_launch(int bn, int terms, int epi, const GemmOperands& op, const GemmArgs& args_in, cudaStream_t st,
                        int max_ctas, int amode) {
  if (args_in.K % (terms == 1 ? BK_I8 : BK) != 0 || args_in.N % bn != 0 || args_in.M <= 0) return cudaErrorInvalidValue;
  GemmArgs args = args_in;
  if (terms == 1) args.chunk_kb = 0;  // integer codes: the products and their sums are exact integers
#define G4M_CASE(BN_, T_, E_, A_) \
  if (bn == BN_ && terms == T_ && epi == E_ && amode == A_) return launch_t<BN_, T_, E_, A_>(op, args, st, max_ctas);
  G4M_CASE(256, 1, EPI_F32, 0)
  G4M_CASE(256, 2, EPI_F32, 0)
  G4M_CASE(128, 3, EPI_F32, 0)
  G4M_CASE(256, 2, EPI_GELU_GATE, 0)
  G4M_CASE(256, 2, EPI_GLU, 0)
  G4M_CASE(256, 2, EPI_SILU, 0)
  G4M_CASE(256, 2, EPI_QKV_VISION, 0)
  G4M_CASE(256, 2, EPI_PATCH, 0)
  // integer-code operands (static input quantisation)
  G4M_CASE(256, 1, EPI_F32, 1)
  G4M_CASE(256, 1, EPI_QKV_VISION, 1)
  G4M_CASE(256, 1, EPI_GELU_GATE, 2)
  G4M_CASE(256, 1, EPI_SILU, 0)
  G4M_CASE(256, 1, EPI_GLU, 0)
#undef G4M_CASE
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// Operand preparation kernels
// ---------------------------------------------------------------------------

// x f32 [rows, cols] -> hi/lo fp16 planes.  s_in != 0 quantises instead
// (srqScalar) and stores the integer code as a signed byte in `hi` (row
// stride cols bytes) for the int8 GEMM, whose epilogue scales by s_in.
// row_scale (optional, [rows]) multiplies x first (the embedder's inverse RMS).
__global__ void prep_a_kernel(const float* __restrict__ x, long rows, int cols, float s_in, const float* row_scale,
                              __half* __restrict__ hi, __half* __restrict__ lo) {
  const long n = rows * (long)cols;
  const float inv_s = s_in != 0.0f ? 1.0f / s_in : 0.0f;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float v = x[i];
    if (row_scale) v = v * row_scale[i / cols];
    if (s_in != 0.0f) {
      reinterpret_cast<int8_t*>(hi)[i] = (int8_t)srq_code(v, s_in, inv_s);
    } else {
      __half h, l;
      split_f16(v, h, l);
      hi[i] = h;
      lo[i] = l;
    }
  }
}

cudaError_t prep_a(const float* x, long rows, int cols, float s_in, const float* row_scale, __half* hi, __half* lo,
                   cudaStream_t st) {
  const long n = rows * (long)cols;
  int grid = (int)std::min<long>((n + 255) / 256, 148L * 16);
  if (grid <= 0) return cudaSuccess;
  prep_a_kernel<<<grid, 256, 0, st>>>(x, rows, cols, s_in, row_scale, hi, lo);
  return cudaGetLastError();
}

// Weight conversion to fp16 rows.  dst_row = map ? map[r] : r.
//   kind 0: int8 [rows, cols]                      value = w
//   kind 1: unsigned codes packed `bits` per lane   value = code - 2^(bits-1)
//   kind 2: f32 -> hi (and lo if lo != nullptr)
//   kind 3: bf16 bits -> fp16
__global__ void prep_w_kernel(const void* __restrict__ src, int kind, int bits, int rows, int cols, const int* map,
                              __half* __restrict__ hi, __half* __restrict__ lo) {
  const long n = (long)rows * cols;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    const long dst = (long)(map ? map[r] : r) * cols + c;
    float v;
    if (kind == 0) {
      v = (float)reinterpret_cast<const int8_t*>(src)[i];
    } else if (kind == 1) {
      const uint8_t* w = reinterpret_cast<const uint8_t*>(src);
      const int vpb = 8 / bits;
      const long bpr = (long)cols * bits / 8;
      const uint8_t byte = w[(long)r * bpr + c / vpb];
      const int code = (byte >> ((c % vpb) * bits)) & ((1 << bits) - 1);
      v = (float)(code - (1 << (bits - 1)));
    } else if (kind == 2) {
      v = reinterpret_cast<const float*>(src)[i];
    } else {
      const uint16_t b = reinterpret_cast<const uint16_t*>(src)[i];
      v = __uint_as_float((uint32_t)b << 16);
    }
    if (kind == 2 && lo) {
      __half h, l;
      split_f16(v, h, l);
      hi[dst] = h;
      lo[dst] = l;
    } else {
      hi[dst] = __float2half_rn(v);
    }
  }
}

cudaError_t prep_w(const void* src, int kind, int bits, int rows, int cols, const int* map, __half* hi, __half* lo,
                   cudaStream_t st) {
  const long n = (long)rows * cols;
  int grid = (int)std::min<long>((n + 255) / 256, 148L * 16);
  if (grid <= 0) return cudaSuccess;
  prep_w_kernel<<<grid, 256, 0, st>>>(src, kind, bits, rows, cols, map, hi, lo);
  return cudaGetLastError();
}

// Weight conversion to signed bytes for the int8 GEMMs (static input
// quantisation).  dst_row = map ? map[r] : r.
//   kind 0: int8 [rows, cols]                      value = w
//   kind 1: unsigned codes packed `bits` per lane   value = code - 2^(bits-1)
__global__ void prep_w_i8_kernel(const void* __restrict__ src, int kind, int bits, int rows, int cols, const int* map,
                                 int8_t* __restrict__ dst) {
  const long n = (long)rows * cols;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    int v;
    if (kind == 0) {
      v = reinterpret_cast<const int8_t*>(src)[i];
    } else {
      const uint8_t* w = reinterpret_cast<const uint8_t*>(src);
      const int vpb = 8 / bits;
      const long bpr = (long)cols * bits / 8;
      const uint8_t byte = w[(long)r * bpr + c / vpb];
      v = ((byte >> ((c % vpb) * bits)) & ((1 << bits) - 1)) - (1 << (bits - 1));
    }
    dst[(long)(map ? map[r] : r) * cols + c] = (int8_t)v;
  }
}

cudaError_t prep_w_i8(const void* src, int kind, int bits, int rows, int cols, const int* map, int8_t* dst,
                      cudaStream_t st) {
  const long n = (long)rows * cols;
  int grid = (int)std::min<long>((n + 255) / 256, 148L * 16);
  if (grid <= 0) return cudaSuccess;
  prep_w_i8_kernel<<<grid, 256, 0, st>>>(src, kind, bits, rows, cols, map, dst);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Exact-semantics SIMT QAT linear for shapes the tensor-core tiles do not
// cover (in % 64 != 0 or out % 256 != 0).  One thread per output, f32
// accumulation in the reference's order with every product and sum rounded
// to f32 (Math.fround), as runQatI8LinearCpu / runPackedQatLinearCpu do
// (src/kernels/qat.ts:458-487, 215-247).
// ---------------------------------------------------------------------------
__global__ void qat_simt_kernel(const float* __restrict__ x, const void* __restrict__ w, int bits,
                                const float* __restrict__ scale, const float* __restrict__ bias, int rows, int in,
                                int out, float s_in, float s_out, float* __restrict__ y) {
  const long total = (long)rows * out;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = (int)(i / out), o = (int)(i % out);
    const float* xr = x + (long)r * in;
    float res;
    if (bits == 0) {
      const int8_t* wr = reinterpret_cast<const int8_t*>(w) + (long)o * in;
      float sum = 0.f;
      for (int c = 0; c < in; ++c) sum = __fadd_rn(sum, __fmul_rn(srq_f(xr[c], s_in), (float)wr[c]));
      res = srq_f(__fmul_rn(sum, scale[o]), s_out);
    } else {
      const uint8_t* wr = reinterpret_cast<const uint8_t*>(w) + (long)o * in * bits / 8;
      const int vpb = 8 / bits, mask = (1 << bits) - 1;
      float sqa = 0.f, sa = 0.f;
      for (int c = 0; c < in; ++c) {
        const float act = srq_f(xr[c], s_in);
        const int code = (wr[c / vpb] >> ((c % vpb) * bits)) & mask;
        sqa = __fadd_rn(sqa, __fmul_rn((float)code, act));
        sa = __fadd_rn(sa, act);
      }
      const float zp = (float)(1 << (bits - 1));
      res = srq_f(__fmul_rn(scale[o], __fsub_rn(sqa, __fmul_rn(zp, sa))), s_out);
    }
    if (bias) res = __fadd_rn(res, bias[o]);
    y[i] = res;
  }
}

cudaError_t qat_linear_simt(const float* x, const void* w, int bits, const float* scale, const float* bias, int rows,
                            int in, int out, float s_in, float s_out, float* y, cudaStream_t st) {
  const long total = (long)rows * out;
  if (total <= 0) return cudaSuccess;
  const int grid = (int)std::min<long>((total + 127) / 128, 148L * 32);
  qat_simt_kernel<<<grid, 128, 0, st>>>(x, w, bits, scale, bias, rows, in, out, s_in, s_out, y);
  return cudaGetLastError();
}

}  // namespace g4m
