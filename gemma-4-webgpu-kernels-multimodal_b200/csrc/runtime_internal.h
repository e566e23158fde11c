// Internal state of the g4m runtime shared by runtime.cu and audio.cu.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

namespace g4m {

struct DevBuf {
  void* p = nullptr;
  size_t n = 0;
};

cudaError_t ensure(DevBuf& b, size_t bytes);
void release(DevBuf& b);
int fail(int code, const std::string& msg);
extern thread_local std::string tl_err;

struct VisionLayer {
  __half* wqkv = nullptr;  // [2304, 768]: q rows, k rows, v rows
  float* sqkv = nullptr;
  float sin_qkv[3] = {0, 0, 0}, sout_qkv[3] = {0, 0, 0};
  float* qn = nullptr;
  float* kn = nullptr;
  __half* wo = nullptr;
  float* so = nullptr;
  float sin_o = 0, sout_o = 0;
  __half* wgu = nullptr;  // [6144, 768]: gate / up rows interleaved in 128-row groups
  float* sgu = nullptr;
  float sin_gu[2] = {0, 0}, sout_gu[2] = {0, 0};
  __half* wd = nullptr;
  float* sd = nullptr;
  float sin_d = 0, sout_d = 0;
  float *n_in = nullptr, *n_pa = nullptr, *n_pf = nullptr, *n_po = nullptr;
};

struct VisionWeights {
  int layers = 0;
  std::vector<VisionLayer> L;
  __half* patch_w = nullptr;  // [768, 768] fp16 (from BF16)
  float* pos = nullptr;       // [2][P][768] f32 (from BF16)
  int P = 0;
  __half* emb_hi = nullptr;  // [1536, 768] F32 split into fp16 hi/lo
  __half* emb_lo = nullptr;
};

struct AudioLayer {
  __half* w_ff1[2] = {nullptr, nullptr};  // [4096, 1024] per feed-forward block
  float* s_ff1[2] = {nullptr, nullptr};
  __half* w_ff2[2] = {nullptr, nullptr};  // [1024, 4096]
  float* s_ff2[2] = {nullptr, nullptr};
  float sin_ff[2][2] = {{0, 0}, {0, 0}}, sout_ff[2][2] = {{0, 0}, {0, 0}};
  float* n_ff_pre[2] = {nullptr, nullptr};
  float* n_ff_post[2] = {nullptr, nullptr};
  __half* wqkv = nullptr;  // [3072, 1024]
  float* sqkv = nullptr;
  float sin_qkv[3] = {0, 0, 0}, sout_qkv[3] = {0, 0, 0};
  __half* wpost = nullptr;
  float* spost = nullptr;
  float sin_post = 0, sout_post = 0;
  float* pds = nullptr;   // per_dim_scale [128]
  float* relk = nullptr;  // relative keys [13][1024] (projected once at load)
  __half* wstart = nullptr;  // [2048, 1024] value / gate rows interleaved
  float* sstart = nullptr;
  float sin_start = 0, sout_start[2] = {0, 0};
  __half* wend = nullptr;
  float* send = nullptr;
  float sin_end = 0, sout_end = 0;
  float* n_lpre = nullptr;
  float* n_conv = nullptr;
  float* dw = nullptr;  // [1024][5]
  float *n_pre_attn = nullptr, *n_post_attn = nullptr, *n_out = nullptr;
};

struct AudioWeights {
  int layers = 0;
  std::vector<AudioLayer> L;
  float* c0w = nullptr;  // [128][1][3][3]
  float* c0n = nullptr;  // [128]
  double* c0stat = nullptr;  // layer-0 weight moments: wbar[9], then G[k][l] for k <= l (45)
  __half *c1_hi = nullptr, *c1_lo = nullptr;  // layer-1 conv [9 taps][32 out][128 in], fp16 hi / lo
  float* c1n = nullptr;  // [32]
  __half *in_hi = nullptr, *in_lo = nullptr;    // input projection [1024, 1024]
  __half *out_hi = nullptr, *out_lo = nullptr;  // output projection [1536, 1024]
  float* out_b = nullptr;
  __half *emb_hi = nullptr, *emb_lo = nullptr;  // embedder [1536, 1536]
  float* window = nullptr;   // periodic Hann [320]
  float* mel = nullptr;      // [257][128]
  int* mel_rng = nullptr;    // [128][2] first / last FFT bin with a non-zero weight per mel channel
  double2* twiddle = nullptr;  // [256] exp(-2 pi i k / 512)
};

struct LayoutCache {
  int gh = -1, gw = -1, tokens = -1;
  DevBuf pos_xy, rope, pool;
};

struct VisionBuffers {
  DevBuf h, y, h0, a_hi, a_lo, a_c, o_hi, o_lo, g_hi, g_lo, q_hi, q_lo, k_hi, k_lo, vt_hi, vt_lo, e_hi, e_lo;
};

struct AudioBuffers {
  DevBuf samples, sample_off, sample_len, frame_off, frames, feats, fmask, t0_off, t0_len, l0, l0mask, t1_off, t1_len,
      l1, row_clip, clip_row0, clip_rows, h, y, qkv, g, a_hi, a_lo, a_c, f_hi, f_lo, keep, proj, e_hi, e_lo, out, h0;
};

// Static input quantisation of projections sharing one operand (q / k / v,
// gate / up): 0 all scales zero (hi/lo operand), 1 all non-zero (one code
// plane per scale), -1 mixed (not supported).
inline int quant_group(const float* s, int n) {
  int nz = 0;
  for (int i = 0; i < n; ++i) nz += s[i] != 0.0f;
  return nz == 0 ? 0 : (nz == n ? 1 : -1);
}

// Opt-in per-launch event timing (g4m_profile_begin / g4m_profile_end).
struct ProfRec {
  const char* label;
  cudaEvent_t a, b;
};

extern std::atomic<long long> g_launches;

struct Device {
  int id = 0;
  bool prof_on = false;
  std::vector<ProfRec> prof;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  cudaStream_t st = nullptr;   // compute
  cudaStream_t cst = nullptr;  // host <-> device copies of the batch calls (overlap the compute of other chunks)
  int* err = nullptr;
  VisionWeights vw;
  AudioWeights aw;
  std::vector<void*> allocs;
  VisionBuffers vb;
  AudioBuffers ab;
  LayoutCache vlc;
  DevBuf io_in, io_out, io_src, io_tmp;  // batch staging; io_src / io_tmp: source images and resize rows
  // g4m_qat_linear's per-call operands, grown on demand and reused by later calls
  DevBuf qw_raw, qw16, qscale, qbias, qx, qy, qa_hi, qa_lo;
  long last_vision_rows = 0;
  long last_audio_rows = 0;
  int aw_mel_sr = 0;  // sampling rate the mel filter bank was built for
  std::mutex mu;

  cudaEvent_t next_event() {
    if (ev_used == ev_pool.size()) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      ev_pool.push_back(e);
    }
    return ev_pool[ev_used++];
  }

  void free_all() {
    for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
    ev_pool.clear();
    for (void* p : allocs) cudaFree(p);
    allocs.clear();
    DevBuf* bufs[] = {&vb.h, &vb.y, &vb.h0, &vb.a_hi, &vb.a_lo, &vb.a_c, &vb.o_hi, &vb.o_lo, &vb.g_hi, &vb.g_lo,
                      &vb.q_hi, &vb.q_lo, &vb.k_hi, &vb.k_lo, &vb.vt_hi, &vb.vt_lo, &vb.e_hi, &vb.e_lo,
                      &vlc.pos_xy, &vlc.rope, &vlc.pool, &io_in, &io_out, &io_src, &io_tmp, &qw_raw, &qw16,
                      &qscale, &qbias, &qx, &qy, &qa_hi, &qa_lo};
    for (DevBuf* b : bufs) release(*b);
    DevBuf* abufs[] = {&ab.samples, &ab.sample_off, &ab.sample_len, &ab.frame_off, &ab.frames, &ab.feats,
                       &ab.fmask, &ab.t0_off, &ab.t0_len, &ab.l0, &ab.l0mask, &ab.t1_off, &ab.t1_len, &ab.l1,
                       &ab.row_clip, &ab.clip_row0, &ab.clip_rows, &ab.h, &ab.y, &ab.qkv, &ab.g, &ab.a_hi,
                       &ab.a_lo, &ab.a_c, &ab.f_hi, &ab.f_lo, &ab.keep, &ab.proj, &ab.e_hi, &ab.e_lo, &ab.out, &ab.h0};
    for (DevBuf* b : abufs) release(*b);
    if (err) cudaFree(err);
    err = nullptr;
    if (st) cudaStreamDestroy(st);
    if (cst) cudaStreamDestroy(cst);
    cst = nullptr;
    st = nullptr;
  }
};

int finish(Device& d, cudaStream_t st);

// Small host -> device metadata uploads on a stream.  With `keep` the source
// is copied into storage that lives until the caller's final synchronize, so
// the host need not wait for the copy; without it the caller synchronizes.
struct HostKeep {
  std::vector<std::vector<char>> bufs;
};
inline cudaError_t upload_meta(void* dst, const void* src, size_t bytes, cudaStream_t st, HostKeep* keep) {
  if (!keep) return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, st);
  keep->bufs.emplace_back((const char*)src, (const char*)src + bytes);
  return cudaMemcpyAsync(dst, keep->bufs.back().data(), bytes, cudaMemcpyHostToDevice, st);
}

// Chunks [first, last) of n equal items for a pipelined batch call.  Only
// the first chunk's upload and the last chunk's download are not hidden
// behind compute, so the head and the tail hold `edge` items and the middle
// is cut into chunks of at most `mid` items (each chunk's upload has to fit
// under the previous chunk's compute).  Batches under three edges run as one
// chunk.
inline std::vector<std::pair<int, int>> edge_chunks(int n, int edge, int mid) {
  std::vector<std::pair<int, int>> c;
  if (n < 3 * edge || edge <= 0 || mid <= 0) {
    c.push_back({0, n});
    return c;
  }
  c.push_back({0, edge});
  const int body = n - 2 * edge, k = (body + mid - 1) / mid;
  for (int i = 0; i < k; ++i)
    c.push_back({edge + (int)((long)body * i / k), edge + (int)((long)body * (i + 1) / k)});
  c.push_back({n - edge, n});
  return c;
}

inline void prof_begin(Device& d, cudaStream_t st, const char* label) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (!d.prof_on) return;
  ProfRec r{label, d.next_event(), d.next_event()};
  cudaEventRecord(r.a, st);
  d.prof.push_back(r);
}
inline void prof_end(Device& d, cudaStream_t st) {
  if (d.prof_on && !d.prof.empty()) cudaEventRecord(d.prof.back().b, st);
}

// Launch a kernel through a launcher returning cudaError_t, counting it and,
// when profiling is on, bracketing it with events under `label`.
#define G4M_RUN(label, x)                                                                            \
  do {                                                                                               \
    ::g4m::prof_begin(d, st, label);                                                                 \
    cudaError_t e_ = (x);                                                                            \
    ::g4m::prof_end(d, st);                                                                          \
    if (e_ != cudaSuccess) return ::g4m::fail(G4M_E_CUDA, std::string(label) + ": " + cudaGetErrorString(e_)); \
  } while (0)
void* dalloc(Device& d, size_t bytes);
float* upload_f32(Device& d, const float* host, size_t n);
int load_audio(Device& d, const class SafeTensors& f);
int load_qat(Device& d, const class SafeTensors& f, const std::string& prefix, const std::string& label, int out, int in,
             bool packed, __half* dst, const std::vector<int>& map, std::vector<float>& scale_host, float& s_in,
             float& s_out, DevBuf& staging, DevBuf& map_dev);
std::vector<int> map_interleave(int n, int which);
cudaError_t qat_linear_simt(const float* x, const void* w, int bits, const float* scale, const float* bias, int rows,
                            int in, int out, float s_in, float s_out, float* y, cudaStream_t st);
int qat_linear_device(Device& d, const __half* w16, const float* scale, const float* bias, const void* w_raw, int bits,
                      int rows, int in, int out, float s_in, float s_out, const float* x_dev, float* y_dev, DevBuf& a_hi,
                      DevBuf& a_lo, cudaStream_t st);

}  // namespace g4m

struct g4m_ctx {
  std::vector<g4m::Device*> devs;
  std::atomic<int> cancel{0};
  int debug = 0;
  int attention_impl = 0;  // 0 tensor-core flash attention, 1 fp32 SIMT (G4M_ATTENTION=simt)
};

struct g4m_linear {
  g4m::Device* d = nullptr;
  int out = 0, in = 0, bits = 0;
  void* w_raw = nullptr;
  __half* w16 = nullptr;
  float* scale = nullptr;
  float* bias = nullptr;
  float s_in = 0, s_out = 0;
  g4m::DevBuf a_hi, a_lo;
};
