// g4m_linear_run_noalloc: the resident QAT linear run without any device
// allocation.  g4m_linear_run keeps its fp16 hi/lo activation operand in a
// per-linear buffer that grows with cudaMalloc the first time a larger row
// count arrives; this entry point stages that operand in a fixed file-scope
// device array instead, so a call never allocates, frees or grows memory.
//
// Scratch: two fp16 planes (hi, lo) of kNoAllocMaxElems elements each,
// 2 x 8 MiB = 16 MiB of static device memory per device.  A call needs
// rows * in <= kNoAllocMaxElems elements; larger calls are rejected with
// G4M_E_SHAPE before anything is launched.  Nothing in the scratch has to
// start at zero: prep_a writes every element a call reads (rows * in per
// plane) before the GEMM reads it, and the GEMM's tensor maps cover exactly
// rows x in, so no stale element is ever read.
//
// Calls share the scratch of their device: two calls in flight at the same
// time on one device (different streams or host threads) race on it.
#include <mutex>
#include <string>
#include "../../include/g4m.h"
#include "g4m_kernels.h"
#include "runtime_internal.h"

namespace g4m {

constexpr long kNoAllocMaxElems = 1L << 22;  // per plane: rows * in

static __device__ __align__(256) __half g_noalloc_scratch[2 * kNoAllocMaxElems];

// Device address of the scratch on the current device, looked up once per
// device ordinal (cudaGetSymbolAddress, with that device current).
static void* noalloc_scratch(int dev) {
  static std::mutex mu;
  static void* addr[256] = {};
  if (dev < 0 || dev >= 256) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) == cudaSuccess) addr[dev] = p;
  }
  return addr[dev];
}

}  // namespace g4m

using namespace g4m;

extern "C" int g4m_linear_run_noalloc(g4m_linear* L, const float* x_dev, int rows, float* y_dev, void* stream) {
  if (!L || !x_dev || !y_dev || rows < 0) return fail(G4M_E_ARG, "bad argument");
  if (rows == 0) return G4M_OK;
  if ((long)rows * L->in > kNoAllocMaxElems)
    return fail(G4M_E_SHAPE, "g4m_linear_run_noalloc: rows * in = " + std::to_string((long)rows * L->in) +
                                 " exceeds the static scratch of " + std::to_string(kNoAllocMaxElems) +
                                 " elements; use g4m_linear_run");
  Device& d = *L->d;
  cudaSetDevice(d.id);
  (void)cudaGetLastError();
  void* base = noalloc_scratch(d.id);
  if (!base) return fail(G4M_E_CUDA, "g4m_linear_run_noalloc: scratch symbol lookup failed");
  // Views of the static planes sized to their full capacity, so the shared
  // operand path finds them large enough and never reallocates.
  DevBuf hi, lo;
  hi.p = base;
  hi.n = (size_t)kNoAllocMaxElems * sizeof(__half);
  lo.p = (__half*)base + kNoAllocMaxElems;
  lo.n = hi.n;
  // The shared operand path grows a buffer that is too small (cudaFree +
  // cudaMalloc); on these views that would free a static symbol.  Refuse
  // here, whatever the limit above says, so that branch is never reached.
  if ((size_t)rows * (size_t)L->in * sizeof(__half) > hi.n)
    return fail(G4M_E_SHAPE, "g4m_linear_run_noalloc: operand does not fit the static scratch views");
  cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamLegacy;  // NULL: the default stream
  return qat_linear_device(d, L->w16, L->scale, L->bias, L->w_raw, L->bits, rows, L->in, L->out, L->s_in, L->s_out,
                           x_dev, y_dev, hi, lo, st);
}
