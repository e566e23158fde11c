// Blackwell (sm_100a) building blocks: mbarriers with bounded waits, TMA
// tile loads (never with cluster multicast), tcgen05 tensor-memory
// allocation, MMA issue/commit and TMEM loads, and the UMMA descriptors.
//
// Descriptor layouts follow the PTX ISA "tcgen05 instruction descriptor" and
// "shared memory descriptor" tables (bit positions cross-checked against the
// CUTLASS source header cute/arch/mma_sm100_desc.hpp).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace g4m {

// Error words written by device code (first error wins).
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitFull = 1,     // consumer timed out waiting for a TMA stage
  kErrWaitEmpty = 2,    // producer timed out waiting for a free stage
  kErrWaitAccFull = 3,  // epilogue timed out waiting for an accumulator
  kErrWaitAccEmpty = 4, // MMA timed out waiting for the epilogue
  kErrWaitDrain = 5,    // exit path timed out draining in-flight copies
  kErrShape = 6,
};

// ~2 s at 1.9 GHz: far above any legitimate wait in these kernels.
constexpr long long kWaitCycles = 4000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code` in *err) when the phase
// does not complete within `budget` cycles, or when another warp of the CTA
// already aborted (*abort_flag != 0).
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err, int code,
                                              volatile int* abort_flag, long long budget) {
  const uint32_t b = smem_u32(bar);
  if (mbar_try_wait(b, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(b, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > budget) {
      atomicCAS(err, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                                          volatile int* abort_flag) {
  return mbar_wait_for(bar, parity, err, code, abort_flag, kWaitCycles);
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %0;" ::"r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// 2-D tiled TMA load into this CTA's shared memory, completing on `bar`.
// c0 is the innermost (contiguous) coordinate in elements.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2eF = 1.4426950408889634f;

// sigmoid(x) = 1 / (1 + 2^(-x log2 e)); saturates to 0 / 1 without NaN.
__device__ __forceinline__ float sigmoid_f(float x) { return rcp_approx(1.0f + ex2_approx(-x * kLog2eF)); }

// Warp-cooperative store of a 32-row block: block row r belongs to lane r,
// whose RB bytes are vals[0 .. RB/16).  The rows pass through the warp's
// shared-memory stage (16-byte slots XOR-swizzled so that both phases are
// bank-conflict free) and leave row-contiguously, RB/16 lanes per row, so
// every store instruction writes whole 32-byte sectors of 512/RB rows rather
// than a 16-byte piece of each of 32 rows.  Block row r goes to
// base + r * stride (bytes); rows r >= nrows are not written.
template <int RB>
__device__ __forceinline__ void warp_store_block(uint4* stage, const uint4 (&vals)[RB / 16], char* base,
                                                 size_t stride, int nrows, int lane) {
  constexpr int S = RB / 16, RPI = 32 / S, RP128 = 8 / S;  // slots per row, rows per store, rows per 128 B
  const int swz = (lane / RP128) & (S - 1);
#pragma unroll
  for (int c = 0; c < S; ++c) stage[lane * S + (c ^ swz)] = vals[c];
  __syncwarp();
#pragma unroll
  for (int k = 0; k < S; ++k) {
    const int r = k * RPI + lane / S, sl = lane % S;
    const uint4 x = stage[r * S + (sl ^ ((r / RP128) & (S - 1)))];
    if (r < nrows) *reinterpret_cast<uint4*>(base + (size_t)r * stride + sl * 16) = x;
  }
  __syncwarp();
}

// Untiled bulk copy of `bytes` from global memory into this CTA's shared
// memory, completing on `bar`.  Both addresses 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05
// ---------------------------------------------------------------------------

// Whole warp: allocate `ncols` TMEM columns, address written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16/bf16 operands, f32 accumulate).
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with the accumulate flag fixed at compile time.  A single thread
// issues every MMA of a CTA, so the issue path is kept short: descriptors are
// formed once and advanced by constant offsets (desc_add), the flag is an
// immediate, and the issuing loops are unrolled.  With N = 128 operands a
// longer per-MMA issue sequence, not the tensor pipe, sets the pace.
template <bool ACC>
__device__ __forceinline__ void mma_f16_ss_c(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "n"(ACC ? 1 : 0)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8: signed 8-bit A and B (K = 32
// per instruction, the same 32 bytes of a 128-byte swizzled row as K = 16 of
// fp16), exact 32-bit integer accumulation.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
template <bool ACC>
__device__ __forceinline__ void mma_i8_ss_c(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "n"(ACC ? 1 : 0)
      : "memory");
}

// Shared-memory descriptor advanced by `bytes` (a multiple of 16): the start
// address field is the low 14 bits (address >> 4), and every operand tile
// lies below 256 KB of shared memory, so the sum never carries out of it.
__device__ __forceinline__ uint64_t desc_add(uint64_t desc, uint32_t bytes) { return desc + (uint64_t)(bytes >> 4); }

// Arrive on `bar` once every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// lane (lane_base + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// tcgen05.ld of 32 lanes x 32 columns without the wait (pair with tmem_wait_ld).
__device__ __forceinline__ void tmem_ld32_raw(uint32_t taddr, uint32_t* r) {
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

// Thread i of the warp writes lane (lane_base + i), columns [col, col+32).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld_all() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st_all() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand tile stored in the
// 128-byte swizzle layout written by TMA with CU_TENSOR_MAP_SWIZZLE_128B:
// rows of 64 fp16 (128 B), 8-row swizzle atoms 1024 B apart.
//   bits  0-13 start address >> 4
//   bits 16-29 leading byte offset >> 4 (unused for swizzled K-major; 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 61-63 layout (2 = 128-byte swizzle)
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp16 A and B (K-major), f32 D.
//   bits 4-5 D format (1 = f32); 7-9 A format (0 = f16); 10-12 B format;
//   15/16 A/B major (0 = K); 17-22 N >> 3; 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Instruction descriptor, kind::i8: signed 8-bit A and B (K-major), s32 D.
//   bits 4-5 D format (2 = s32); 7-9 A format (1 = signed 8-bit); 10-12 B
//   format; 17-22 N >> 3; 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_i8_s32(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Two floats -> packed fp16x2 hi and lo words (hi = fp16(x), lo = fp16(x - hi)).
__device__ __forceinline__ void split2_f16(float a, float b, uint32_t& hi, uint32_t& lo) {
  union {
    __half2 h;
    uint32_t u;
  } H, L;
  H.h = __floats2half2_rn(a, b);
  const float2 back = __half22float2(H.h);
  L.h = __floats2half2_rn(a - back.x, b - back.y);
  hi = H.u;
  lo = L.u;
}

__device__ __forceinline__ void split_f16(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

}  // namespace g4m
