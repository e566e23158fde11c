// Vision tower helper kernels: patch operand, 3x3 pooler fused with the
// embedder's inverse RMS, and an fp32 SIMT flash attention (the exact
// baseline the tcgen05 attention is checked against on the device).
#include "g4m_kernels.h"
#include "g4m_sm100.cuh"

namespace g4m {

// Patchify (src/preprocess/image.ts:133-148) + the 2*(p - 0.5) scaling of
// runVisionPatchEmbeddingCpu (src/vision/kernels.ts:1008-1012), written as
// the fp16 hi/lo operand of the patch-projection GEMM.  pixels are
// [n_images][height][width][3] float32; rows are (image, patch_y, patch_x),
// columns (dy * patch + dx) * 3 + channel.
__global__ void __launch_bounds__(256) patch_operand_kernel(const float* __restrict__ px, int n_images, int height,
                                                            int width, int patch, __half* __restrict__ hi,
                                                            __half* __restrict__ lo) {
  // one thread per (patch row, dy): the patch's pixel row dy is 3 * patch
  // contiguous floats of the image and 3 * patch contiguous operand columns
  const int gw = width / patch, gh = height / patch;
  const long rows = (long)n_images * gh * gw;
  const long task = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (task >= rows * patch) return;
  const long row = task / patch;
  const int dy = (int)(task - row * patch);
  const int img = (int)(row / (gh * gw)), p = (int)(row - (long)img * gh * gw);
  const int py = p / gw, pxx = p - py * gw;
  const float* src = px + (((long)img * height + py * patch + dy) * width + (long)pxx * patch) * 3;
  const long o = row * (long)(patch * patch * 3) + (long)dy * patch * 3;
  const int n = 3 * patch;
  if (n == 48 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {  // 16-pixel patches: float4 in, 16 B out
#pragma unroll
    for (int q = 0; q < 6; ++q) {  // 8 values per step
      const float4 a = __ldg(reinterpret_cast<const float4*>(src) + 2 * q);
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 2 * q + 1);
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      __align__(16) __half hh[8], ll[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const double sv = 2.0 * ((double)v[u] - 0.5);
        hh[u] = __double2half(sv);
        ll[u] = __double2half(sv - (double)__half2float(hh[u]));
      }
      *reinterpret_cast<uint4*>(hi + o + 8 * q) = *reinterpret_cast<const uint4*>(hh);
      *reinterpret_cast<uint4*>(lo + o + 8 * q) = *reinterpret_cast<const uint4*>(ll);
    }
  } else {
    for (int k = 0; k < n; ++k) {
      const double sv = 2.0 * ((double)src[k] - 0.5);
      const __half h = __double2half(sv);
      hi[o + k] = h;
      lo[o + k] = __double2half(sv - (double)__half2float(h));
    }
  }
}

cudaError_t vision_patch_operand(const float* pixels, int n_images, int height, int width, int patch, __half* hi,
                                 __half* lo, cudaStream_t st) {
  const long tasks = (long)n_images * (height / patch) * (width / patch) * patch;
  if (tasks <= 0) return cudaSuccess;
  patch_operand_kernel<<<(int)((tasks + 255) / 256), 256, 0, st>>>(pixels, n_images, height, width, patch, hi, lo);
  return cudaGetLastError();
}

// runVisionPoolerCpu (src/vision/kernels.ts:815-833) followed by the
// embedder's weightless RMSNorm (src/embedder/index.ts:126-140): one warp
// per soft token, d = 768.
__global__ void __launch_bounds__(256) pool_operand_kernel(const float* __restrict__ h, const int* __restrict__ idx,
                                                           int n_images, int rows_per_image, int tokens, int k2,
                                                           float eps, float* pooled_out, __half* hi, __half* lo) {
  constexpr int D = 768, V = D / 128;
  const int lane = threadIdx.x & 31;
  const long w = (long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (w >= (long)n_images * tokens) return;
  const int img = (int)(w / tokens), t = (int)(w % tokens);
  float4 acc[V];
#pragma unroll
  for (int i = 0; i < V; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < k2; ++j) {
    const int p = idx[t * k2 + j];
    if (p < 0) continue;
    const float4* src = reinterpret_cast<const float4*>(h + ((long)img * rows_per_image + p) * D);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 v = src[lane + 32 * i];
      acc[i].x += v.x;
      acc[i].y += v.y;
      acc[i].z += v.z;
      acc[i].w += v.w;
    }
  }
  const float scale = sqrtf((float)D) / (float)k2;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    acc[i] = make_float4(acc[i].x * scale, acc[i].y * scale, acc[i].z * scale, acc[i].w * scale);
    ss += acc[i].x * acc[i].x + acc[i].y * acc[i].y + acc[i].z * acc[i].z + acc[i].w * acc[i].w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float inv = 1.0f / sqrtf(ss / (float)D + eps);
  const long orow = (long)img * tokens + t;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = 4 * (lane + 32 * i);
    if (pooled_out) *reinterpret_cast<float4*>(pooled_out + orow * D + c) = acc[i];
    float v[4] = {acc[i].x * inv, acc[i].y * inv, acc[i].z * inv, acc[i].w * inv};
    __align__(8) __half hh[4], ll[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) split_f16(v[u], hh[u], ll[u]);
    *reinterpret_cast<uint2*>(hi + orow * D + c) = *reinterpret_cast<uint2*>(hh);
    *reinterpret_cast<uint2*>(lo + orow * D + c) = *reinterpret_cast<uint2*>(ll);
  }
}

cudaError_t vision_pool_operand(const float* h, const int* pool_idx, int n_images, int rows_per_image, int tokens,
                                int k2, int d, float eps, float* pooled_out, __half* hi, __half* lo, cudaStream_t st) {
  if (d != 768) return cudaErrorInvalidValue;
  const long warps = (long)n_images * tokens;
  if (warps <= 0) return cudaSuccess;
  pool_operand_kernel<<<(int)((warps + 7) / 8), 256, 0, st>>>(h, pool_idx, n_images, rows_per_image, tokens, k2, eps,
                                                               pooled_out, hi, lo);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// fp32 SIMT flash attention, head_dim 64, scale 1, no mask
// (runVisionAttentionBodyCpu, src/vision/kernels.ts:75-131).
// One thread per query row, 128 queries per CTA, 64-key tiles in smem.
// Output: o[(img * n + tok)][head * 64 + d] as fp16 hi/lo.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(128) attn_simt_kernel(const __half* __restrict__ qh, const __half* __restrict__ ql,
                                                        const __half* __restrict__ kh, const __half* __restrict__ kl,
                                                        const __half* __restrict__ vth,
                                                        const __half* __restrict__ vtl, int n, int vt_pitch, float s_code,
                                                        int heads, __half* __restrict__ oh,
                                                        __half* __restrict__ ol) {
  __shared__ float Ks[64][65];
  __shared__ float Vs[64][65];
  const int bh = blockIdx.y;
  const int qrow = blockIdx.x * 128 + threadIdx.x;
  const bool valid = qrow < n;
  float q[64], o[64];
  const size_t qbase = ((size_t)bh * n + (valid ? qrow : 0)) * 64;
#pragma unroll
  for (int d = 0; d < 64; ++d) {
    q[d] = __half2float(qh[qbase + d]) + __half2float(ql[qbase + d]);
    o[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int k0 = 0; k0 < n; k0 += 64) {
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 64; i += 128) {
      const int kr = i / 64, d = i % 64;
      const int key = k0 + kr;
      float kv = 0.f, vv = 0.f;
      if (key < n) {
        const size_t ki = ((size_t)bh * n + key) * 64 + d;
        kv = __half2float(kh[ki]) + __half2float(kl[ki]);
        const size_t vi = ((size_t)bh * 64 + d) * vt_pitch + key;
        vv = __half2float(vth[vi]) + __half2float(vtl[vi]);
      }
      Ks[kr][d] = kv;
      Vs[kr][d] = vv;
    }
    __syncthreads();
    const int kn = min(64, n - k0);
    float s[64];
    float mt = -INFINITY;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < 64; ++d) acc = fmaf(q[d], Ks[j][d], acc);
      s[j] = j < kn ? acc : -INFINITY;
      mt = fmaxf(mt, s[j]);
    }
    const float mn = fmaxf(m, mt);
    const float corr = expf(m - mn);
    l *= corr;
#pragma unroll
    for (int d = 0; d < 64; ++d) o[d] *= corr;
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float p = expf(s[j] - mn);
      l += p;
#pragma unroll
      for (int d = 0; d < 64; ++d) o[d] = fmaf(p, Vs[j][d], o[d]);
    }
    m = mn;
  }
  if (!valid) return;
  const int img = bh / heads, head = bh % heads;
  const size_t orow = (size_t)img * n + qrow;
  const float inv = 1.0f / l;
  __half* dh = oh + orow * (size_t)(heads * 64) + head * 64;
  __half* dl = ol + orow * (size_t)(heads * 64) + head * 64;
  int8_t* dc = reinterpret_cast<int8_t*>(oh) + orow * (size_t)(heads * 64) + head * 64;
#pragma unroll
  for (int d = 0; d < 64; ++d) {
    if (s_code != 0.0f) {  // signed-byte codes for the o_proj input scale
      dc[d] = (int8_t)srq_code(o[d] * inv, s_code, 1.0f / s_code);
    } else {
      __half h, lo;
      split_f16(o[d] * inv, h, lo);
      dh[d] = h;
      dl[d] = lo;
    }
  }
}

cudaError_t vision_attention_simt(const __half* q_hi, const __half* q_lo, const __half* k_hi, const __half* k_lo,
                                  const __half* vt_hi, const __half* vt_lo, int bh, int n, int vt_pitch, int heads,
                                  __half* o_hi, __half* o_lo, float s_code, cudaStream_t st) {
  if (bh <= 0 || n <= 0) return cudaSuccess;
  dim3 grid((n + 127) / 128, bh);
  attn_simt_kernel<<<grid, 128, 0, st>>>(q_hi, q_lo, k_hi, k_lo, vt_hi, vt_lo, n, vt_pitch, s_code, heads, o_hi, o_lo);
  return cudaGetLastError();
}

}  // namespace g4m

namespace g4m {

// ---------------------------------------------------------------------------
// Image resize to the token layout's target size (the canvas drawImage step
// of preprocessGemma4ImageSource, src/preprocess/image.ts:121-128).  The
// browser's "high quality" smoothing is not specified, so this is the
// separable antialiased linear (triangle) filter of PIL / torchvision:
// for output index i of an axis scaled by s = in / out, centre (i + 0.5) s,
// radius r = max(s, 1), weights max(0, 1 - |x + 0.5 - centre| / r) over the
// source pixels x in range, normalised.  At s = 1 it is the identity.  The
// result is rounded to 8 bits (the canvas stores RGBA8) and rescaled by 1/255
// as the reference does.  Pass 1 filters rows ([h][w][c] uint8 ->
// [h][tw][3] f32), pass 2 columns (-> [th][tw][3] f32 in [0, 1]).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tri_weight(float x, float centre, float radius) {
  return fmaxf(0.f, 1.f - fabsf(x + 0.5f - centre) / radius);
}

__global__ void resize_rows_kernel(const uint8_t* __restrict__ src, int h, int w, int c, int tw,
                                   float* __restrict__ tmp) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)h * tw) return;
  const int y = (int)(i / tw), ox = (int)(i % tw);
  const float s = (float)w / (float)tw, r = fmaxf(s, 1.f), centre = (ox + 0.5f) * s;
  const int x0 = max(0, (int)floorf(centre - r)), x1 = min(w - 1, (int)ceilf(centre + r));
  float acc[3] = {0.f, 0.f, 0.f}, ws = 0.f;
  for (int x = x0; x <= x1; ++x) {
    const float wt = tri_weight((float)x, centre, r);
    if (wt == 0.f) continue;
    const uint8_t* p = src + ((long)y * w + x) * c;
    acc[0] = fmaf(wt, (float)p[0], acc[0]);
    acc[1] = fmaf(wt, (float)p[1], acc[1]);
    acc[2] = fmaf(wt, (float)p[2], acc[2]);
    ws += wt;
  }
  const float inv = ws > 0.f ? 1.f / ws : 0.f;
  float* o = tmp + i * 3;
  o[0] = acc[0] * inv;
  o[1] = acc[1] * inv;
  o[2] = acc[2] * inv;
}

__global__ void resize_cols_kernel(const float* __restrict__ tmp, int h, int tw, int th, float* __restrict__ dst) {
  const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (long)th * tw) return;
  const int oy = (int)(i / tw), ox = (int)(i % tw);
  const float s = (float)h / (float)th, r = fmaxf(s, 1.f), centre = (oy + 0.5f) * s;
  const int y0 = max(0, (int)floorf(centre - r)), y1 = min(h - 1, (int)ceilf(centre + r));
  float acc[3] = {0.f, 0.f, 0.f}, ws = 0.f;
  for (int y = y0; y <= y1; ++y) {
    const float wt = tri_weight((float)y, centre, r);
    if (wt == 0.f) continue;
    const float* p = tmp + ((long)y * tw + ox) * 3;
    acc[0] = fmaf(wt, p[0], acc[0]);
    acc[1] = fmaf(wt, p[1], acc[1]);
    acc[2] = fmaf(wt, p[2], acc[2]);
    ws += wt;
  }
  const float inv = ws > 0.f ? 1.f / ws : 0.f;
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float q = fminf(fmaxf(floorf(acc[k] * inv + 0.5f), 0.f), 255.f);  // RGBA8 canvas value
    dst[i * 3 + k] = (float)((double)q * (1.0 / 255.0));  // imageData * rescaleFactor, Float32Array store
  }
}

cudaError_t vision_resize(const uint8_t* src, int h, int w, int c, int th, int tw, float* tmp, float* dst,
                          cudaStream_t st) {
  if (h <= 0 || w <= 0 || th <= 0 || tw <= 0 || (c != 3 && c != 4)) return cudaErrorInvalidValue;
  const long n1 = (long)h * tw, n2 = (long)th * tw;
  resize_rows_kernel<<<(unsigned)((n1 + 255) / 256), 256, 0, st>>>(src, h, w, c, tw, tmp);
  resize_cols_kernel<<<(unsigned)((n2 + 255) / 256), 256, 0, st>>>(tmp, h, tw, th, dst);
  return cudaGetLastError();
}

}  // namespace g4m
