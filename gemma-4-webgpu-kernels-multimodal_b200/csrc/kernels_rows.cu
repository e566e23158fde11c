// Fused row kernels: RMSNorm / residual / scaled residual chains of the
// vision and audio layers, one warp per row, float4 loads, warp-shuffle
// reductions, writing both the f32 residual stream and the fp16 hi/lo
// operand of the next GEMM in the same pass.
//
// Replaces runVisionRmsNormWebGpu (src/vision/kernels.ts:161-281, one thread
// per row there), runResidualAddWebGpu (283-387) and
// runScaledResidualAddWebGpu (src/audio/kernels.ts:1127-1240), in the orders
// used by src/vision/encoder.ts:228-297 and src/audio/encoder.ts:761-921.
#include "g4m_kernels.h"
#include "g4m_sm100.cuh"

namespace g4m {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int V>
__device__ __forceinline__ float inv_rms(const float4 (&x)[V], int d, float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) ss += x[i].x * x[i].x + x[i].y * x[i].y + x[i].z * x[i].z + x[i].w * x[i].w;
  ss = warp_sum(ss);
  return 1.0f / sqrtf(ss / (float)d + eps);
}

template <int V>
__global__ void __launch_bounds__(256) fused_rows_kernel(RowArgs r) {
  const int lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= r.rows) return;
  const int d = r.d;
  float4 h[V];
  if (r.y) {
    const float4* y = reinterpret_cast<const float4*>(r.y + row * d);
#pragma unroll
    for (int i = 0; i < V; ++i) h[i] = y[lane + 32 * i];
    if (r.w_post) {
      const float inv = inv_rms<V>(h, d, r.eps);
      const float4* w = reinterpret_cast<const float4*>(r.w_post);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float4 wv = w[lane + 32 * i];
        h[i] = make_float4((h[i].x * inv) * wv.x, (h[i].y * inv) * wv.y, (h[i].z * inv) * wv.z, (h[i].w * inv) * wv.w);
      }
    }
    if (r.h_in) {
      const float4* hi = reinterpret_cast<const float4*>(r.h_in + row * d);
      const float s = r.res_scale;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float4 b = hi[lane + 32 * i];
        h[i] = make_float4(b.x + h[i].x * s, b.y + h[i].y * s, b.z + h[i].z * s, b.w + h[i].w * s);
      }
    }
  } else {
    const float4* hi = reinterpret_cast<const float4*>(r.h_in + row * d);
#pragma unroll
    for (int i = 0; i < V; ++i) h[i] = hi[lane + 32 * i];
  }
  if (r.w_out) {
    const float inv = inv_rms<V>(h, d, r.eps);
    const float4* w = reinterpret_cast<const float4*>(r.w_out);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 wv = w[lane + 32 * i];
      h[i] = make_float4((h[i].x * inv) * wv.x, (h[i].y * inv) * wv.y, (h[i].z * inv) * wv.z, (h[i].w * inv) * wv.w);
    }
  }
  if (r.h_out) {
    float4* ho = reinterpret_cast<float4*>(r.h_out + row * d);
#pragma unroll
    for (int i = 0; i < V; ++i) ho[lane + 32 * i] = h[i];
  }
  if (r.w_next) {
    const float inv = inv_rms<V>(h, d, r.eps);
    const float4* w = reinterpret_cast<const float4*>(r.w_next);
    const float inv_a = r.s_in_next != 0.0f ? 1.0f / r.s_in_next : 0.0f;
    const float inv_b = r.s_in_b != 0.0f ? 1.0f / r.s_in_b : 0.0f;
    const float inv_c = r.s_in_c != 0.0f ? 1.0f / r.s_in_c : 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 wv = w[lane + 32 * i];
      float v[4] = {(h[i].x * inv) * wv.x, (h[i].y * inv) * wv.y, (h[i].z * inv) * wv.z, (h[i].w * inv) * wv.w};
      const int c = 4 * (lane + 32 * i);
      if (r.s_in_next != 0.0f) {
        // integer codes per consumer scale as signed bytes (lda bytes per row):
        // a_hi (s_in_next), a_lo (s_in_b), a_c (s_in_c)
        uint32_t ca = 0, cb = 0, cc = 0;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          ca |= ((uint32_t)(int)srq_code(v[u], r.s_in_next, inv_a) & 0xFFu) << (8 * u);
          if (r.s_in_b != 0.0f) cb |= ((uint32_t)(int)srq_code(v[u], r.s_in_b, inv_b) & 0xFFu) << (8 * u);
          if (r.a_c) cc |= ((uint32_t)(int)srq_code(v[u], r.s_in_c, inv_c) & 0xFFu) << (8 * u);
        }
        const long o = row * r.lda + c;
        *reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(r.a_hi) + o) = ca;
        if (r.s_in_b != 0.0f) *reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(r.a_lo) + o) = cb;
        if (r.a_c) *reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(r.a_c) + o) = cc;
      } else {
        __align__(8) __half hh[4], ll[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) split_f16(v[u], hh[u], ll[u]);
        *reinterpret_cast<uint2*>(r.a_hi + row * r.lda + c) = *reinterpret_cast<uint2*>(hh);
        *reinterpret_cast<uint2*>(r.a_lo + row * r.lda + c) = *reinterpret_cast<uint2*>(ll);
      }
    }
  }
}

cudaError_t fused_rows(const RowArgs& r, cudaStream_t st) {
  if (r.rows <= 0) return cudaSuccess;
  const int blocks = (int)((r.rows + 7) / 8);
  switch (r.d) {
    case 768:
      fused_rows_kernel<6><<<blocks, 256, 0, st>>>(r);
      break;
    case 1024:
      fused_rows_kernel<8><<<blocks, 256, 0, st>>>(r);
      break;
    case 1536:
      fused_rows_kernel<12><<<blocks, 256, 0, st>>>(r);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Per-row inverse RMS (weightless) folded into an fp16 hi/lo operand: the
// embedder's normalisation (src/embedder/index.ts:126-140).
template <int V>
__global__ void __launch_bounds__(256) inv_rms_operand_kernel(const float* x, long rows, int d, float eps, __half* hi,
                                                              __half* lo) {
  const int lane = threadIdx.x & 31;
  const long row = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float4 h[V];
  const float4* src = reinterpret_cast<const float4*>(x + row * d);
#pragma unroll
  for (int i = 0; i < V; ++i) h[i] = src[lane + 32 * i];
  const float inv = inv_rms<V>(h, d, eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    float v[4] = {h[i].x * inv, h[i].y * inv, h[i].z * inv, h[i].w * inv};
    __align__(8) __half hh[4], ll[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) split_f16(v[u], hh[u], ll[u]);
    const int c = 4 * (lane + 32 * i);
    *reinterpret_cast<uint2*>(hi + row * d + c) = *reinterpret_cast<uint2*>(hh);
    *reinterpret_cast<uint2*>(lo + row * d + c) = *reinterpret_cast<uint2*>(ll);
  }
}

cudaError_t row_inv_rms_operand(const float* x, long rows, int d, float eps, __half* hi, __half* lo, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const int blocks = (int)((rows + 7) / 8);
  switch (d) {
    case 768:
      inv_rms_operand_kernel<6><<<blocks, 256, 0, st>>>(x, rows, d, eps, hi, lo);
      break;
    case 1024:
      inv_rms_operand_kernel<8><<<blocks, 256, 0, st>>>(x, rows, d, eps, hi, lo);
      break;
    case 1536:
      inv_rms_operand_kernel<12><<<blocks, 256, 0, st>>>(x, rows, d, eps, hi, lo);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

__global__ void add_bias_rows_kernel(float* y, const float* b, long n, int d) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    y[i] = y[i] + b[i % d];
}

cudaError_t add_bias_rows(float* y, const float* b, long rows, int d, cudaStream_t st) {
  const long n = rows * d;
  if (n <= 0) return cudaSuccess;
  const int grid = (int)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
  add_bias_rows_kernel<<<grid, 256, 0, st>>>(y, b, n, d);
  return cudaGetLastError();
}

__global__ void gather_rows_kernel(const float* src, const int* idx, long n, int d, float* dst) {
  const long total = n * d;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long r = i / d;
    dst[i] = src[(long)idx[r] * d + (i % d)];
  }
}

cudaError_t gather_rows(const float* src, const int* rows_idx, long n, int d, float* dst, cudaStream_t st) {
  const long total = n * d;
  if (total <= 0) return cudaSuccess;
  const int grid = (int)((total + 255) / 256 < 148 * 16 ? (total + 255) / 256 : 148 * 16);
  gather_rows_kernel<<<grid, 256, 0, st>>>(src, rows_idx, n, d, dst);
  return cudaGetLastError();
}

// Self-test of the device-side failure detection: one warp waits on a shared
// mbarrier that nothing arrives on, through the same bounded wait the GEMM
// and attention pipelines use, so the wait expires after `budget` cycles,
// records kErrWaitFull in the error word and the kernel returns.
__global__ void wait_timeout_kernel(int* err, long long budget) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)mbar_wait_for(&bar, 0, err, kErrWaitFull, &abort_flag, budget);
}

cudaError_t selftest_wait_timeout(int* err, long long budget, cudaStream_t st) {
  if (budget <= 0) return cudaErrorInvalidValue;
  wait_timeout_kernel<<<1, 32, 0, st>>>(err, budget);
  return cudaGetLastError();
}

}  // namespace g4m
