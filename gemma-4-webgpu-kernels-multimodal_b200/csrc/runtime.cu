// C ABI runtime of the g4m library: context and per-device state, resident
// weights, the vision tower (and, via audio.cu, the audio tower) on one CUDA
// stream per device, the QAT-linear boundary and the host layout helpers.
//
// Orchestration follows the reference's dataflow (src/vision/index.ts:46-112,
// src/vision/encoder.ts:162-298) but keeps every tensor resident on the
// device between kernels: one host round trip per call instead of one per
// kernel, weights converted once at load instead of fetched per layer.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/g4m.h"
#include "g4m_kernels.h"
#include "runtime_internal.h"
#include "safetensors.h"

namespace g4m {

thread_local std::string tl_err;
std::atomic<long long> g_launches{0};

int fail(int code, const std::string& msg) {
  tl_err = msg;
  return code;
}

cudaError_t ensure(DevBuf& b, size_t bytes) {
  if (b.n >= bytes) return cudaSuccess;
  if (b.p) cudaFree(b.p);
  b.p = nullptr;
  b.n = 0;
  if (bytes == 0) return cudaSuccess;
  cudaError_t e = cudaMalloc(&b.p, bytes);
  if (e == cudaSuccess) b.n = bytes;
  return e;
}

void release(DevBuf& b) {
  if (b.p) cudaFree(b.p);
  b.p = nullptr;
  b.n = 0;
}

int finish(Device& d, cudaStream_t st) {
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(G4M_E_CUDA, std::string("stream synchronize: ") + cudaGetErrorString(e));
  int w = 0;
  e = cudaMemcpy(&w, d.err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(G4M_E_CUDA, std::string("error word read: ") + cudaGetErrorString(e));
  if (w != 0) {
    cudaMemset(d.err, 0, sizeof(int));
    return fail(G4M_E_TIMEOUT, "a device-side bounded wait expired (kernel error code " + std::to_string(w) + ")");
  }
  return G4M_OK;
}

void* dalloc(Device& d, size_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
  d.allocs.push_back(p);
  return p;
}

float* upload_f32(Device& d, const float* host, size_t n) {
  float* p = (float*)dalloc(d, n * sizeof(float));
  if (p && cudaMemcpy(p, host, n * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) return nullptr;
  return p;
}

// ---------------------------------------------------------------------------
// Host layout helpers (product implementations)
// ---------------------------------------------------------------------------

// aspectRatioPreservingSize + computeGemma4ImageTokenLayout,
// src/preprocess/image.ts:4-30, 217-252 (doubles, as JS numbers).
int image_layout(double height, double width, double patch, double max_soft, double pool, int64_t* out) {
  const double max_patches = max_soft * pool * pool;
  if (height <= 0 || width <= 0) return fail(G4M_E_LAYOUT, "Image height and width must be positive.");
  const double total = height * width, target_px = max_patches * patch * patch;
  const double factor = sqrt(target_px / total);
  const double side = pool * patch;
  double th = floor(factor * height / side) * side, tw = floor(factor * width / side) * side;
  if (th == 0 && tw == 0)
    return fail(G4M_E_LAYOUT, "Image resize rounded to 0 x 0 for side multiple " + std::to_string((int)side) + ".");
  const double max_side = floor(max_patches / (pool * pool)) * side;
  if (th == 0) {
    th = side;
    tw = fmin(floor(width / height) * side, max_side);
  } else if (tw == 0) {
    tw = side;
    th = fmin(floor(height / width) * side, max_side);
  }
  if (th * tw > target_px)
    return fail(G4M_E_LAYOUT, "Image resize exceeds " + std::to_string((long long)max_patches) + " patches.");
  out[0] = (int64_t)th;
  out[1] = (int64_t)tw;
  out[2] = (int64_t)(th / patch);
  out[3] = (int64_t)(tw / patch);
  out[4] = (int64_t)max_patches;
  out[5] = (int64_t)floor((th / patch) * (tw / patch) / (pool * pool));
  return G4M_OK;
}

// ---------------------------------------------------------------------------
// Weight loading
// ---------------------------------------------------------------------------

namespace {

bool scalar_f32(const SafeTensors& f, const std::string& name, float& v, std::string& err) {
  const TensorInfo* t = f.find(name);
  if (!t) return (err = "Safetensors tensor not found: " + name, false);
  if (t->dtype != "F32" || !t->shape.empty() || f.bytes(*t) != 4)
    return (err = "Expected scalar F32 tensor for " + name + ", got " + shape_str(*t) + ".", false);
  memcpy(&v, f.data(*t), 4);
  return true;
}

const TensorInfo* need(const SafeTensors& f, const std::string& name, const char* dtype, std::vector<int64_t> shape,
                       const std::string& label, std::string& err) {
  const TensorInfo* t = f.find(name);
  if (!t) {
    err = "Safetensors tensor not found: " + name;
    return nullptr;
  }
  if (t->dtype != dtype || t->shape != shape) {
    err = "Unexpected " + label + " tensor: " + shape_str(*t) + ".";
    return nullptr;
  }
  return t;
}

std::vector<float> bf16_to_f32(const void* p, size_t n) {
  std::vector<float> v(n);
  const uint16_t* b = (const uint16_t*)p;
  for (size_t i = 0; i < n; ++i) {
    uint32_t u = (uint32_t)b[i] << 16;
    memcpy(&v[i], &u, 4);
  }
  return v;
}

}  // namespace

// One QAT projection (I8 or U8 packed) into rows `map[r]` of dst [rows_total, in].
int load_qat(Device& d, const SafeTensors& f, const std::string& prefix, const std::string& label, int out, int in,
             bool packed, __half* dst, const std::vector<int>& map, std::vector<float>& scale_host, float& s_in,
             float& s_out, DevBuf& staging, DevBuf& map_dev) {
  std::string err;
  const TensorInfo* w = f.find(prefix + ".weight");
  if (!w) return fail(G4M_E_IO, "Safetensors tensor not found: " + prefix + ".weight");
  int bits = 0;
  if (!packed) {
    if (w->dtype != "I8" || w->shape != std::vector<int64_t>{out, in})
      return fail(G4M_E_DTYPE, "Unexpected " + label + " weight tensor: " + shape_str(*w) + ".");
  } else {
    // derivePackedQatBits, src/kernels/qat.ts:199-213
    const double b = (double)f.bytes(*w) * 8.0 / ((double)in * out);
    if (!(b == 2 || b == 4 || b == 8))
      return fail(G4M_E_DTYPE, label + ": derived unsupported " + std::to_string(b) + "-bit QAT weights from " +
                                   std::to_string(f.bytes(*w)) + " bytes.");
    bits = (int)b;
    if ((in * bits) % 32 != 0) return fail(G4M_E_DTYPE, label + ": packed QAT row is not byte and u32 aligned.");
    if (w->dtype != "U8" || w->shape != std::vector<int64_t>{out, (int64_t)in * bits / 8})
      return fail(G4M_E_DTYPE, "Unexpected " + label + " packed weight tensor: " + shape_str(*w) + ".");
  }
  const TensorInfo* s = f.find(prefix + ".weight_scale");
  if (!s || s->dtype != "F32" || s->shape != std::vector<int64_t>{out, 1})
    return fail(G4M_E_DTYPE, "Unexpected " + label + " weight scale tensor: " + (s ? shape_str(*s) : "missing") + ".");
  if (!scalar_f32(f, prefix + ".input_activation_scale", s_in, err) ||
      !scalar_f32(f, prefix + ".output_activation_scale", s_out, err))
    return fail(G4M_E_DTYPE, err);
  const float* sv = (const float*)f.data(*s);
  for (int r = 0; r < out; ++r) scale_host[map[r]] = sv[r];
  if (ensure(staging, f.bytes(*w)) != cudaSuccess || ensure(map_dev, map.size() * sizeof(int)) != cudaSuccess)
    return fail(G4M_E_CUDA, "staging allocation failed");
  if (cudaMemcpy(staging.p, f.data(*w), f.bytes(*w), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(map_dev.p, map.data(), map.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
    return fail(G4M_E_CUDA, "weight upload failed");
  // statically quantised inputs (s_in != 0) run on the int8 GEMM: the weights
  // are stored as signed bytes (rows of `in` bytes) in the same buffer
  const cudaError_t ce = s_in != 0.0f
                             ? prep_w_i8(staging.p, packed ? 1 : 0, bits, out, in, (const int*)map_dev.p,
                                         reinterpret_cast<int8_t*>(dst), 0)
                             : prep_w(staging.p, packed ? 1 : 0, bits, out, in, (const int*)map_dev.p, dst, nullptr, 0);
  if (ce != cudaSuccess) return fail(G4M_E_CUDA, "weight conversion launch failed");
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(G4M_E_CUDA, "weight conversion failed");
  return G4M_OK;
}

static std::vector<int> map_offset(int n, int off) {
  std::vector<int> m(n);
  for (int i = 0; i < n; ++i) m[i] = off + i;
  return m;
}

// Rows of two [n, in] matrices interleaved in 128-row groups so one 256-wide
// output tile holds matching columns of both (GEMM epilogues GELU_GATE, GLU).
std::vector<int> map_interleave(int n, int which) {
  std::vector<int> m(n);
  for (int r = 0; r < n; ++r) m[r] = (r / 128) * 256 + which * 128 + (r % 128);
  return m;
}

static int load_vision(Device& d, const SafeTensors& f) {
  const int D = 768, FF = 3072, HD = 64;
  std::string err;
  auto lp = [](int i) { return "model.vision_tower.encoder.layers." + std::to_string(i); };
  int layers = 0;
  while (layers < 16 && f.find(lp(layers) + ".self_attn.q_proj.linear.weight")) ++layers;
  if (layers == 0) return G4M_OK;
  VisionWeights& vw = d.vw;
  vw.L.assign(layers, VisionLayer());
  DevBuf staging, map_dev;
  for (int i = 0; i < layers; ++i) {
    VisionLayer& L = vw.L[i];
    const std::string p = lp(i);
    L.wqkv = (__half*)dalloc(d, (size_t)3 * D * D * 2);
    L.wo = (__half*)dalloc(d, (size_t)D * D * 2);
    L.wgu = (__half*)dalloc(d, (size_t)2 * FF * D * 2);
    L.wd = (__half*)dalloc(d, (size_t)D * FF * 2);
    if (!L.wqkv || !L.wo || !L.wgu || !L.wd) return fail(G4M_E_CUDA, "vision weight allocation failed");
    std::vector<float> sqkv(3 * D), so(D), sgu(2 * FF), sd(D);
    const char* qkv[3] = {"q_proj", "k_proj", "v_proj"};
    for (int j = 0; j < 3; ++j) {
      int rc = load_qat(d, f, p + ".self_attn." + qkv[j] + ".linear", qkv[j], D, D, false, L.wqkv, map_offset(D, j * D),
                        sqkv, L.sin_qkv[j], L.sout_qkv[j], staging, map_dev);
      if (rc) return rc;
    }
    int rc = load_qat(d, f, p + ".self_attn.o_proj.linear", "attention o_proj", D, D, false, L.wo, map_offset(D, 0), so,
                      L.sin_o, L.sout_o, staging, map_dev);
    if (rc) return rc;
    rc = load_qat(d, f, p + ".mlp.gate_proj.linear", "gate_proj", FF, D, false, L.wgu, map_interleave(FF, 0), sgu,
                  L.sin_gu[0], L.sout_gu[0], staging, map_dev);
    if (rc) return rc;
    rc = load_qat(d, f, p + ".mlp.up_proj.linear", "up_proj", FF, D, false, L.wgu, map_interleave(FF, 1), sgu,
                  L.sin_gu[1], L.sout_gu[1], staging, map_dev);
    if (rc) return rc;
    rc = load_qat(d, f, p + ".mlp.down_proj.linear", "down_proj", D, FF, false, L.wd, map_offset(D, 0), sd, L.sin_d,
                  L.sout_d, staging, map_dev);
    if (rc) return rc;
    L.sqkv = upload_f32(d, sqkv.data(), sqkv.size());
    L.so = upload_f32(d, so.data(), so.size());
    L.sgu = upload_f32(d, sgu.data(), sgu.size());
    L.sd = upload_f32(d, sd.data(), sd.size());
    const char* qk[2] = {"q_norm", "k_norm"};
    float** qkd[2] = {&L.qn, &L.kn};
    for (int j = 0; j < 2; ++j) {
      const TensorInfo* t = need(f, p + ".self_attn." + qk[j] + ".weight", "BF16", {HD}, std::string(qkv[j]) + " norm", err);
      if (!t) return fail(G4M_E_DTYPE, err);
      std::vector<float> v = bf16_to_f32(f.data(*t), HD);
      *qkd[j] = upload_f32(d, v.data(), HD);
    }
    const char* nn[4] = {"input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                         "post_feedforward_layernorm"};
    const char* nl[4] = {"input layernorm", "post-attention layernorm", "pre-feedforward layernorm",
                         "post-feedforward layernorm"};
    float** nd[4] = {&L.n_in, &L.n_pa, &L.n_pf, &L.n_po};
    for (int j = 0; j < 4; ++j) {
      const TensorInfo* t = need(f, p + "." + nn[j] + ".weight", "BF16", {D},
                                 "vision layer " + std::to_string(i) + " " + nl[j], err);
      if (!t) return fail(G4M_E_DTYPE, err);
      std::vector<float> v = bf16_to_f32(f.data(*t), D);
      *nd[j] = upload_f32(d, v.data(), D);
    }
    if (!L.sqkv || !L.so || !L.sgu || !L.sd || !L.qn || !L.kn || !L.n_in || !L.n_pa || !L.n_pf || !L.n_po)
      return fail(G4M_E_CUDA, "vision weight upload failed");
  }
  // Patch projection (BF16 [768, 768]) and position table (BF16 [2, P, 768]),
  // src/vision/index.ts:54-60, src/vision/encoder.ts:28-35.
  const TensorInfo* pw = need(f, "model.vision_tower.patch_embedder.input_proj.weight", "BF16", {D, 768},
                              "image embedding patch projection", err);
  if (!pw) return fail(G4M_E_DTYPE, err);
  const TensorInfo* pt = f.find("model.vision_tower.patch_embedder.position_embedding_table");
  if (!pt) return fail(G4M_E_IO, "Safetensors tensor not found: model.vision_tower.patch_embedder.position_embedding_table");
  if (pt->dtype != "BF16" || pt->shape.size() != 3 || pt->shape[0] != 2 || pt->shape[2] != D)
    return fail(G4M_E_DTYPE, "Unexpected position table shape: " + shape_str(*pt) + ".");
  const TensorInfo* ew = need(f, "model.embed_vision.embedding_projection.weight", "F32", {1536, D},
                              "vision embedder projection", err);
  if (!ew) return fail(G4M_E_DTYPE, err);
  vw.patch_w = (__half*)dalloc(d, (size_t)D * 768 * 2);
  vw.P = (int)pt->shape[1];
  std::vector<float> pos = bf16_to_f32(f.data(*pt), (size_t)2 * vw.P * D);
  vw.pos = upload_f32(d, pos.data(), pos.size());
  vw.emb_hi = (__half*)dalloc(d, (size_t)1536 * D * 2);
  vw.emb_lo = (__half*)dalloc(d, (size_t)1536 * D * 2);
  if (!vw.patch_w || !vw.pos || !vw.emb_hi || !vw.emb_lo) return fail(G4M_E_CUDA, "vision weight allocation failed");
  if (ensure(staging, (size_t)1536 * D * 4) != cudaSuccess) return fail(G4M_E_CUDA, "staging allocation failed");
  if (cudaMemcpy(staging.p, f.data(*pw), f.bytes(*pw), cudaMemcpyHostToDevice) != cudaSuccess ||
      prep_w(staging.p, 3, 0, D, 768, nullptr, vw.patch_w, nullptr, 0) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess)
    return fail(G4M_E_CUDA, "patch projection upload failed");
  if (cudaMemcpy(staging.p, f.data(*ew), f.bytes(*ew), cudaMemcpyHostToDevice) != cudaSuccess ||
      prep_w(staging.p, 2, 0, 1536, D, nullptr, vw.emb_hi, vw.emb_lo, 0) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess)
    return fail(G4M_E_CUDA, "vision embedder upload failed");
  release(staging);
  release(map_dev);
  vw.layers = layers;
  return G4M_OK;
}

// ---------------------------------------------------------------------------
// Vision tower
// ---------------------------------------------------------------------------

static int ensure_vision_layout(Device& d, int gh, int gw, int tokens) {
  LayoutCache& c = d.vlc;
  if (c.gh == gh && c.gw == gw && c.tokens == tokens) return G4M_OK;
  const int N = gh * gw;
  std::vector<int> pos(2 * N);
  std::vector<float> cs(2 * 32 * (size_t)N);
  for (int p = 0; p < N; ++p) {
    const int x = p % gw, y = p / gw;
    pos[2 * p] = x;
    pos[2 * p + 1] = y;
    // runVisionRopeCpu angles, src/vision/kernels.ts:55-69: part 0 uses x,
    // part 1 uses y, frequency index f in [0, 16), theta 100.
    for (int part = 0; part < 2; ++part) {
      const double P = part == 0 ? x : y;
      for (int fi = 0; fi < 16; ++fi) {
        const double ang = P / pow(100.0, (double)(2 * fi) / 32.0);
        cs[((size_t)p * 32 + part * 16 + fi) * 2] = (float)cos(ang);
        cs[((size_t)p * 32 + part * 16 + fi) * 2 + 1] = (float)sin(ang);
      }
    }
  }
  // visionPoolIndices, src/vision/kernels.ts:955-980
  const int k = 3, cells_x = gw / k, cells_y = gh / k;
  if (cells_x * cells_y != tokens)
    return fail(G4M_E_SHAPE, "Vision pooler output length " + std::to_string(tokens) + " does not match " +
                                 std::to_string(cells_x) + " x " + std::to_string(cells_y) + ".");
  std::vector<int> idx((size_t)tokens * 9, -1);
  for (int p = 0; p < N; ++p) {
    const int x = p % gw, y = p / gw;
    const int tok = x / k + cells_x * (y / k), local = (y % k) * k + (x % k);
    if (tok < 0 || tok >= tokens)
      return fail(G4M_E_SHAPE, "Vision pooler patch position (" + std::to_string(x) + ", " + std::to_string(y) +
                                   ") maps outside output length.");
    idx[(size_t)tok * 9 + local] = p;
  }
  if (ensure(c.pos_xy, pos.size() * 4) || ensure(c.rope, cs.size() * 4) || ensure(c.pool, idx.size() * 4))
    return fail(G4M_E_CUDA, "layout table allocation failed");
  if (cudaMemcpy(c.pos_xy.p, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice) ||
      cudaMemcpy(c.rope.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) ||
      cudaMemcpy(c.pool.p, idx.data(), idx.size() * 4, cudaMemcpyHostToDevice))
    return fail(G4M_E_CUDA, "layout table upload failed");
  c.gh = gh;
  c.gw = gw;
  c.tokens = tokens;
  return G4M_OK;
}

// Keys per V^T row, padded so TMA boxes of 64 keys stay 16-byte aligned.
static int vt_pitch(int n) { return (n + 63) / 64 * 64; }

static int ensure_vision_buffers(Device& d, int B, int N, long E) {
  const long M = (long)B * N;
  const size_t f32 = 4, f16 = 2, VT = (size_t)B * 12 * 64 * vt_pitch(N);
  VisionBuffers& b = d.vb;
  if (ensure(b.h, M * 768 * f32) || ensure(b.y, M * 768 * f32) || ensure(b.a_hi, M * 768 * f16) ||
      ensure(b.a_lo, M * 768 * f16) || ensure(b.o_hi, M * 768 * f16) || ensure(b.o_lo, M * 768 * f16) ||
      ensure(b.g_hi, M * 3072 * f16) || ensure(b.g_lo, M * 3072 * f16) || ensure(b.q_hi, M * 768 * f16) ||
      ensure(b.q_lo, M * 768 * f16) || ensure(b.k_hi, M * 768 * f16) || ensure(b.k_lo, M * 768 * f16) ||
      ensure(b.vt_hi, VT * f16) || ensure(b.vt_lo, VT * f16) || ensure(b.e_hi, E * 768 * f16) ||
      ensure(b.e_lo, E * 768 * f16))
    return fail(G4M_E_CUDA, "vision activation allocation failed (" + std::to_string(M) + " rows)");
  bool codes3 = false;  // a third code plane for layers with quantised q / k / v
  for (int i = 0; i < d.vw.layers; ++i) codes3 = codes3 || d.vw.L[i].sin_qkv[0] != 0.0f;
  if (codes3 && ensure(b.a_c, M * 768 * f16))
    return fail(G4M_E_CUDA, "vision activation allocation failed (" + std::to_string(M) + " rows)");
  return G4M_OK;
}

#define G4M_LAUNCH(x)                                                                            \
  do {                                                                                          \
    cudaError_t e_ = (x);                                                                       \
    if (e_ != cudaSuccess) return fail(G4M_E_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

// K chunk of the vision tower's and the QAT linear's fp16 hi/lo GEMMs, in
// 64-wide k-blocks (GemmArgs::chunk_kb): two chunks per K = 768 linear,
// eight for K = 3072.  Measured on the 768 x 768 image through 16 propagated
// layers, the device's distance to a float64 evaluation drops from 2.4x to
// 1.3x the reference f32 arithmetic's own distance, for ~5 % of the tower's
// time.  GEMMs on integer codes accumulate exact integers and need none.
constexpr int kVisionChunkKb = 6;

static GemmArgs base_args(Device& d, int M, int N, int K) {
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.M = M;
  a.N = N;
  a.K = K;
  a.chunk_kb = kVisionChunkKb;
  a.row_scale = 1.0f;
  a.row_scale_b = 1.0f;
  a.row_scale_c = 1.0f;
  a.eps = 1e-6f;
  a.err = d.err;
  return a;
}

// Next-operand fields of a row pass whose consumers have input scales s[0..n)
// (integer code planes a_hi, a_lo, a_c when they are non-zero).
static void next_scales(RowArgs& r, const float* s, int n, __half* a_c) {
  r.s_in_next = s ? s[0] : 0.0f;
  r.s_in_b = (s && n > 1) ? s[1] : 0.0f;
  r.s_in_c = (s && n > 2) ? s[2] : 0.0f;
  r.a_c = (s && n > 2 && s[0] != 0.0f) ? a_c : nullptr;
}

// Runs vision layers [first, first+count): on entry vb.h holds the residual
// stream and vb.a_* the input-norm operand of layer `first`.
static int vision_layer_range(g4m_ctx* ctx, Device& d, int B, int N, int first, int count, cudaStream_t st) {
  VisionWeights& vw = d.vw;
  VisionBuffers& b = d.vb;
  const int M = B * N, D = 768;
  for (int i = first; i < first + count; ++i) {
    if (ctx->cancel.load()) return fail(G4M_E_CANCELLED, "Aborted");
    const VisionLayer& L = vw.L[i];
    const bool qkv_codes = L.sin_qkv[0] != 0.0f;  // groups are all-zero or all-non-zero (vision_check_quant)
    const bool gu_codes = L.sin_gu[0] != 0.0f;
    // q, k, v projections + head norms + RoPE (src/vision/encoder.ts:681-724)
    GemmArgs a = base_args(d, M, 3 * D, D);
    a.col_scale = L.sqkv;
    if (qkv_codes) {
      a.row_scale = L.sin_qkv[0];
      a.row_scale_b = L.sin_qkv[1];
      a.row_scale_c = L.sin_qkv[2];
    }
    a.s_out = L.sout_qkv[0];
    a.s_out_b = L.sout_qkv[1];
    a.s_out_c = L.sout_qkv[2];
    a.proj_width = D;
    a.heads = 12;
    a.qn_w = L.qn;
    a.kn_w = L.kn;
    a.rope_cs = (const float*)d.vlc.rope.p;
    a.rows_per_image = N;
    a.vt_pitch = vt_pitch(N);
    a.q_hi = (__half*)b.q_hi.p;
    a.q_lo = (__half*)b.q_lo.p;
    a.k_hi = (__half*)b.k_hi.p;
    a.k_lo = (__half*)b.k_lo.p;
    a.vt_hi = (__half*)b.vt_hi.p;
    a.vt_lo = (__half*)b.vt_lo.p;
    GemmOperands op{(const __half*)b.a_hi.p, (const __half*)b.a_lo.p, L.wqkv, nullptr, (const __half*)b.a_c.p};
    if (qkv_codes) G4M_RUN("gemm_qkv", gemm_launch(256, 1, EPI_QKV_VISION, op, a, st, 0, 1));
    else G4M_RUN("gemm_qkv", gemm_launch(256, 2, EPI_QKV_VISION, op, a, st));
    // attention body (src/vision/kernels.ts:75-114), scale 1
    if (ctx->attention_impl == 0) {
      G4M_RUN("attention", vision_attention_tc((const __half*)b.q_hi.p, (const __half*)b.q_lo.p, (const __half*)b.k_hi.p,
                                     (const __half*)b.k_lo.p, (const __half*)b.vt_hi.p, (const __half*)b.vt_lo.p, B * 12,
                                     N, vt_pitch(N), 12, (__half*)b.o_hi.p, (__half*)b.o_lo.p, L.sin_o, d.err, st));
    } else {
      G4M_RUN("attention", vision_attention_simt((const __half*)b.q_hi.p, (const __half*)b.q_lo.p, (const __half*)b.k_hi.p,
                                       (const __half*)b.k_lo.p, (const __half*)b.vt_hi.p, (const __half*)b.vt_lo.p,
                                       B * 12, N, vt_pitch(N), 12, (__half*)b.o_hi.p, (__half*)b.o_lo.p, L.sin_o, st));
    }
    // o_proj
    a = base_args(d, M, D, D);
    a.col_scale = L.so;
    a.s_out = L.sout_o;
    a.out_f32 = (float*)b.y.p;
    a.ldo = D;
    if (L.sin_o != 0.0f) a.row_scale = L.sin_o;
    op = GemmOperands{(const __half*)b.o_hi.p, (const __half*)b.o_lo.p, L.wo, nullptr, nullptr};
    G4M_RUN("gemm_o", gemm_launch(256, L.sin_o != 0.0f ? 1 : 2, EPI_F32, op, a, st));
    // post-attention norm + residual + pre-feedforward norm
    RowArgs r;
    memset(&r, 0, sizeof(r));
    r.rows = M;
    r.d = D;
    r.eps = 1e-6f;
    r.y = (const float*)b.y.p;
    r.w_post = L.n_pa;
    r.res_scale = 1.0f;
    r.h_in = (const float*)b.h.p;
    r.h_out = (float*)b.h.p;
    r.w_next = L.n_pf;
    next_scales(r, L.sin_gu, 2, nullptr);
    r.a_hi = (__half*)b.a_hi.p;
    r.a_lo = (__half*)b.a_lo.p;
    r.lda = D;
    G4M_RUN("rows", fused_rows(r, st));
    // gate | up with gelu_tanh(gate) * up (src/vision/encoder.ts:1040-1079)
    a = base_args(d, M, 2 * 3072, D);
    a.col_scale = L.sgu;
    a.s_out = L.sout_gu[0];
    a.s_out_b = L.sout_gu[1];
    a.out_hi = (__half*)b.g_hi.p;
    a.out_lo = (__half*)b.g_lo.p;
    a.ldh = 3072;
    a.s_code = L.sin_d;  // down_proj's input scale: store codes
    if (gu_codes) {
      a.row_scale = L.sin_gu[0];
      a.row_scale_b = L.sin_gu[1];
    }
    op = GemmOperands{(const __half*)b.a_hi.p, (const __half*)b.a_lo.p, L.wgu, nullptr, nullptr};
    if (gu_codes) G4M_RUN("gemm_gate_up", gemm_launch(256, 1, EPI_GELU_GATE, op, a, st, 0, 2));
    else G4M_RUN("gemm_gate_up", gemm_launch(256, 2, EPI_GELU_GATE, op, a, st));
    // down_proj
    a = base_args(d, M, D, 3072);
    a.col_scale = L.sd;
    a.s_out = L.sout_d;
    a.out_f32 = (float*)b.y.p;
    a.ldo = D;
    if (L.sin_d != 0.0f) a.row_scale = L.sin_d;
    op = GemmOperands{(const __half*)b.g_hi.p, (const __half*)b.g_lo.p, L.wd, nullptr, nullptr};
    G4M_RUN("gemm_down", gemm_launch(256, L.sin_d != 0.0f ? 1 : 2, EPI_F32, op, a, st));
    // post-feedforward norm + residual (+ next layer's input norm)
    r.w_post = L.n_po;
    const bool more = i + 1 < first + count;
    r.w_next = more ? vw.L[i + 1].n_in : nullptr;
    next_scales(r, more ? vw.L[i + 1].sin_qkv : nullptr, 3, (__half*)b.a_c.p);
    G4M_RUN("rows", fused_rows(r, st));
  }
  return G4M_OK;
}

// Projections that share an operand must all use static input quantisation
// or none of them (q / k / v, gate / up); the rest is per linear.
static int vision_check_quant(const VisionWeights& vw, int layers) {
  for (int i = 0; i < layers; ++i) {
    const VisionLayer& L = vw.L[i];
    if (quant_group(L.sin_qkv, 3) < 0 || quant_group(L.sin_gu, 2) < 0)
      return fail(G4M_E_UNSUPPORTED, "vision layer " + std::to_string(i) +
                                         ": q/k/v (or gate/up) projections mix zero and non-zero "
                                         "input_activation_scale; they share one operand");
  }
  return G4M_OK;
}

int vision_forward(g4m_ctx* ctx, Device& d, int B, const float* pix_dev, int H, int W, int max_soft, int layers,
                   float* out_dev, cudaStream_t st) {
  (void)cudaGetLastError();  // a failed earlier call must not leak into this one
  VisionWeights& vw = d.vw;
  if (vw.layers == 0) return fail(G4M_E_NOT_LOADED, "vision tower weights are not loaded");
  if (layers < 1 || layers > 16)
    return fail(G4M_E_ARG, "Vision encoder layer count must be 1-16, got " + std::to_string(layers) + ".");
  if (layers > vw.layers)
    return fail(G4M_E_NOT_LOADED, "checkpoint holds " + std::to_string(vw.layers) + " vision layers, " +
                                      std::to_string(layers) + " requested");
  int rc = vision_check_quant(vw, layers);
  if (rc) return rc;
  int64_t lay[6];
  rc = image_layout(H, W, 16, max_soft, 3, lay);
  if (rc) return rc;
  if (lay[0] != H || lay[1] != W)
    return fail(G4M_E_SHAPE, "pixels must be at the token layout's target size " + std::to_string(lay[0]) + " x " +
                                 std::to_string(lay[1]) + " (got " + std::to_string(H) + " x " + std::to_string(W) + ")");
  const int gh = (int)lay[2], gw = (int)lay[3], tokens = (int)lay[5], N = gh * gw;
  if (gw - 1 >= vw.P || gh - 1 >= vw.P)
    return fail(G4M_E_SHAPE, "Vision patch positions exceed position table length " + std::to_string(vw.P) + ".");
  if (B <= 0) return G4M_OK;
  rc = ensure_vision_layout(d, gh, gw, tokens);
  if (rc) return rc;
  const long M = (long)B * N;
  rc = ensure_vision_buffers(d, B, N, (long)B * tokens);
  if (rc) return rc;
  VisionBuffers& b = d.vb;
  const int D = 768;
  // patch embedding (src/vision/index.ts:69-78)
  G4M_RUN("patch_operand", vision_patch_operand(pix_dev, B, H, W, 16, (__half*)b.a_hi.p, (__half*)b.a_lo.p, st));
  GemmArgs a = base_args(d, (int)M, D, 768);
  a.out_f32 = (float*)b.h.p;
  a.ldo = D;
  a.rows_per_image = N;
  a.pos_xy = (const int*)d.vlc.pos_xy.p;
  a.posx_rows = vw.pos;
  a.posy_rows = vw.pos + (size_t)vw.P * D;
  GemmOperands op{(const __half*)b.a_hi.p, (const __half*)b.a_lo.p, vw.patch_w, nullptr};
  G4M_RUN("gemm_patch", gemm_launch(256, 2, EPI_PATCH, op, a, st));
  if (ctx->debug) {
    if (ensure(b.h0, M * D * 4)) return fail(G4M_E_CUDA, "debug buffer allocation failed");
    G4M_LAUNCH(cudaMemcpyAsync(b.h0.p, b.h.p, M * D * 4, cudaMemcpyDeviceToDevice, st));
  }
  RowArgs r;
  memset(&r, 0, sizeof(r));
  r.rows = M;
  r.d = D;
  r.eps = 1e-6f;
  r.h_in = (const float*)b.h.p;
  r.w_next = vw.L[0].n_in;
  next_scales(r, vw.L[0].sin_qkv, 3, (__half*)b.a_c.p);
  r.a_hi = (__half*)b.a_hi.p;
  r.a_lo = (__half*)b.a_lo.p;
  r.lda = D;
  G4M_RUN("rows", fused_rows(r, st));
  rc = vision_layer_range(ctx, d, B, N, 0, layers, st);
  if (rc) return rc;
  // pooler + embedder (src/vision/index.ts:94-111)
  G4M_RUN("pool_operand", vision_pool_operand((const float*)b.h.p, (const int*)d.vlc.pool.p, B, N, tokens, 9, D, 1e-6f, nullptr,
                                 (__half*)b.e_hi.p, (__half*)b.e_lo.p, st));
  a = base_args(d, B * tokens, 1536, D);
  a.out_f32 = out_dev;
  a.ldo = 1536;
  op = GemmOperands{(const __half*)b.e_hi.p, (const __half*)b.e_lo.p, vw.emb_hi, vw.emb_lo};
  G4M_RUN("gemm_embed", gemm_launch(128, 3, EPI_F32, op, a, st));
  d.last_vision_rows = M;
  return G4M_OK;
}

int vision_tokens_for(int H, int W, int max_soft, int* tokens) {
  int64_t lay[6];
  int rc = image_layout(H, W, 16, max_soft, 3, lay);
  if (rc) return rc;
  *tokens = (int)lay[5];
  return G4M_OK;
}

// ---------------------------------------------------------------------------
// Single QAT linear
// ---------------------------------------------------------------------------

int qat_linear_device(Device& d, const __half* w16, const float* scale, const float* bias, const void* w_raw, int bits,
                      int rows, int in, int out, float s_in, float s_out, const float* x_dev, float* y_dev, DevBuf& a_hi,
                      DevBuf& a_lo, cudaStream_t st) {
  (void)cudaGetLastError();
  if (w16) {
    if (ensure(a_hi, (size_t)rows * in * 2) || ensure(a_lo, (size_t)rows * in * 2))
      return fail(G4M_E_CUDA, "operand allocation failed");
    G4M_RUN("prep_a", prep_a(x_dev, rows, in, s_in, nullptr, (__half*)a_hi.p, (__half*)a_lo.p, st));
    GemmArgs a = base_args(d, rows, out, in);
    a.col_scale = scale;
    a.row_scale = s_in != 0.0f ? s_in : 1.0f;
    a.s_out = s_out;
    a.bias = bias;
    a.out_f32 = y_dev;
    a.ldo = out;
    GemmOperands op{(const __half*)a_hi.p, (const __half*)a_lo.p, w16, nullptr};
    G4M_RUN("gemm_qat", gemm_launch(256, s_in != 0.0f ? 1 : 2, EPI_F32, op, a, st));
  } else {
    G4M_RUN("qat_simt", qat_linear_simt(x_dev, w_raw, bits, scale, bias, rows, in, out, s_in, s_out, y_dev, st));
  }
  return G4M_OK;
}

// The tensor-core GEMMs take K in 64-element (fp16) or 128-element (int8)
// blocks and N in 256-column tiles; other shapes use the SIMT kernel.
bool qat_tensor_core_shape(int in, int out, float s_in) {
  return in % (s_in != 0.0f ? 128 : 64) == 0 && out % 256 == 0;
}

}  // namespace g4m

using namespace g4m;

// ===========================================================================
// C ABI
// ===========================================================================

extern "C" {

const char* g4m_last_error(void) { return tl_err.c_str(); }

const char* g4m_version(void) { return "g4m sm_100a abi 1"; }

g4m_ctx* g4m_create(const int* devices, int n_devices) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count <= 0) {
    fail(G4M_E_CUDA, "no CUDA device is available");
    return nullptr;
  }
  std::vector<int> ids;
  if (!devices || n_devices <= 0) ids.push_back(0);
  else
    for (int i = 0; i < n_devices; ++i) ids.push_back(devices[i]);
  g4m_ctx* ctx = new g4m_ctx();
  const char* att = getenv("G4M_ATTENTION");
  ctx->attention_impl = (att && !strcmp(att, "simt")) ? 1 : 0;
  for (int id : ids) {
    if (id < 0 || id >= count) {
      fail(G4M_E_ARG, "device index out of range: " + std::to_string(id));
      g4m_destroy(ctx);
      return nullptr;
    }
    Device* d = new Device();
    d->id = id;
    cudaSetDevice(id);
    if (cudaStreamCreateWithFlags(&d->st, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&d->cst, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&d->err, sizeof(int)) != cudaSuccess || cudaMemset(d->err, 0, sizeof(int)) != cudaSuccess) {
      fail(G4M_E_CUDA, "device setup failed on device " + std::to_string(id));
      delete d;
      g4m_destroy(ctx);
      return nullptr;
    }
    ctx->devs.push_back(d);
  }
  return ctx;
}

void g4m_destroy(g4m_ctx* ctx) {
  if (!ctx) return;
  for (Device* d : ctx->devs) {
    cudaSetDevice(d->id);
    cudaStreamSynchronize(d->st);
    d->free_all();
    delete d;
  }
  delete ctx;
}

int g4m_device_count(const g4m_ctx* ctx) { return ctx ? (int)ctx->devs.size() : 0; }

void g4m_cancel(g4m_ctx* ctx) {
  if (ctx) ctx->cancel.store(1);
}
void g4m_clear_cancel(g4m_ctx* ctx) {
  if (ctx) ctx->cancel.store(0);
}

int g4m_set_debug(g4m_ctx* ctx, int on) {
  if (!ctx) return fail(G4M_E_ARG, "null context");
  ctx->debug = on;
  return G4M_OK;
}

int g4m_load_weights(g4m_ctx* ctx, const char* path) {
  if (!ctx || !path) return fail(G4M_E_ARG, "null argument");
  SafeTensors f;
  std::string err;
  if (!f.open(path, err)) return fail(G4M_E_IO, err);
  (void)cudaGetLastError();
  for (Device* d : ctx->devs) {
    std::lock_guard<std::mutex> lk(d->mu);
    cudaSetDevice(d->id);
    int rc = load_vision(*d, f);
    if (rc) return rc;
    rc = load_audio(*d, f);
    if (rc) return rc;
  }
  return G4M_OK;
}

int g4m_loaded_towers(const g4m_ctx* ctx) {
  if (!ctx || ctx->devs.empty()) return 0;
  const Device* d = ctx->devs[0];
  return (d->vw.layers > 0 ? 1 : 0) | (d->aw.layers > 0 ? 2 : 0);
}

int g4m_qat_linear(g4m_ctx* ctx, int di, const float* x, int rows, int in, int out, const void* w, int bits,
                   const float* w_scale, float s_in, float s_out, const float* bias, float* y) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size()) return fail(G4M_E_ARG, "bad context or device index");
  if (!x || !w || !w_scale || !y || rows < 0 || in <= 0 || out <= 0) return fail(G4M_E_ARG, "null or negative argument");
  if (!(bits == 0 || bits == 2 || bits == 4 || bits == 8)) return fail(G4M_E_ARG, "bits must be 0 (int8) or 2/4/8");
  if (bits && (in * bits) % 32 != 0) return fail(G4M_E_SHAPE, "packed QAT row is not byte and u32 aligned.");
  if (rows == 0) return G4M_OK;
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  (void)cudaGetLastError();
  // One call of the reference's runner (runQatI8LinearWebGpu) takes its
  // weights with the activations, so they are uploaded and converted here on
  // every call; the device buffers persist across calls (grown on demand),
  // everything runs on the device's stream, and the host waits once.
  const size_t wbytes = bits ? (size_t)out * in * bits / 8 : (size_t)out * in;
  const bool tc = qat_tensor_core_shape(in, out, s_in);
  if (ensure(d.qw_raw, wbytes) || ensure(d.qscale, (size_t)out * 4) || (bias && ensure(d.qbias, (size_t)out * 4)) ||
      ensure(d.qx, (size_t)rows * in * 4) || ensure(d.qy, (size_t)rows * out * 4) ||
      (tc && ensure(d.qw16, (size_t)out * in * 2)))
    return fail(G4M_E_CUDA, "QAT linear buffer allocation failed");
  cudaStream_t st = d.st;
  if (cudaMemcpyAsync(d.qw_raw.p, w, wbytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(d.qscale.p, w_scale, (size_t)out * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      (bias && cudaMemcpyAsync(d.qbias.p, bias, (size_t)out * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) ||
      cudaMemcpyAsync(d.qx.p, x, (size_t)rows * in * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return fail(G4M_E_CUDA, "QAT linear upload failed");
  if (tc && s_in != 0.0f)
    G4M_RUN("prep_w", prep_w_i8(d.qw_raw.p, bits ? 1 : 0, bits, out, in, nullptr, (int8_t*)d.qw16.p, st));
  else if (tc)
    G4M_RUN("prep_w", prep_w(d.qw_raw.p, bits ? 1 : 0, bits, out, in, nullptr, (__half*)d.qw16.p, nullptr, st));
  int rc = qat_linear_device(d, tc ? (const __half*)d.qw16.p : nullptr, (const float*)d.qscale.p,
                             bias ? (const float*)d.qbias.p : nullptr, d.qw_raw.p, bits, rows, in, out, s_in, s_out,
                             (const float*)d.qx.p, (float*)d.qy.p, d.qa_hi, d.qa_lo, st);
  if (rc) return rc;
  if (cudaMemcpyAsync(y, d.qy.p, (size_t)rows * out * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return fail(G4M_E_CUDA, "output download failed");
  return finish(d, st);
}

int g4m_linear_prepare(g4m_ctx* ctx, int di, const void* w, int bits, int out, int in, const float* w_scale, float s_in,
                       float s_out, const float* bias, g4m_linear** out_linear) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || !w || !w_scale || !out_linear || in <= 0 || out <= 0)
    return fail(G4M_E_ARG, "bad argument");
  if (!(bits == 0 || bits == 2 || bits == 4 || bits == 8)) return fail(G4M_E_ARG, "bits must be 0 (int8) or 2/4/8");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  g4m_linear* L = new g4m_linear();
  L->d = &d;
  L->out = out;
  L->in = in;
  L->bits = bits;
  L->s_in = s_in;
  L->s_out = s_out;
  const size_t wbytes = bits ? (size_t)out * in * bits / 8 : (size_t)out * in;
  bool ok = cudaMalloc(&L->w_raw, wbytes) == cudaSuccess && cudaMalloc(&L->scale, (size_t)out * 4) == cudaSuccess &&
            cudaMemcpy(L->w_raw, w, wbytes, cudaMemcpyHostToDevice) == cudaSuccess &&
            cudaMemcpy(L->scale, w_scale, (size_t)out * 4, cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok && bias)
    ok = cudaMalloc(&L->bias, (size_t)out * 4) == cudaSuccess &&
         cudaMemcpy(L->bias, bias, (size_t)out * 4, cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok && qat_tensor_core_shape(in, out, s_in)) {
    // fp16 weights for the split-operand GEMM, or signed bytes for the int8 GEMM (s_in != 0)
    ok = cudaMalloc(&L->w16, (size_t)out * in * 2) == cudaSuccess &&
         (s_in != 0.0f ? prep_w_i8(L->w_raw, bits ? 1 : 0, bits, out, in, nullptr, reinterpret_cast<int8_t*>(L->w16), 0)
                       : prep_w(L->w_raw, bits ? 1 : 0, bits, out, in, nullptr, L->w16, nullptr, 0)) == cudaSuccess &&
         cudaDeviceSynchronize() == cudaSuccess;
  }
  if (!ok) {
    g4m_linear_free(L);
    return fail(G4M_E_CUDA, "linear weight upload failed");
  }
  *out_linear = L;
  return G4M_OK;
}

int g4m_linear_run(g4m_linear* L, const float* x_dev, int rows, float* y_dev, void* stream) {
  if (!L || !x_dev || !y_dev || rows < 0) return fail(G4M_E_ARG, "bad argument");
  if (rows == 0) return G4M_OK;
  Device& d = *L->d;
  cudaSetDevice(d.id);
  cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamLegacy;  // NULL: the default stream
  return qat_linear_device(d, L->w16, L->scale, L->bias, L->w_raw, L->bits, rows, L->in, L->out, L->s_in, L->s_out,
                           x_dev, y_dev, L->a_hi, L->a_lo, st);
}

void g4m_linear_free(g4m_linear* L) {
  if (!L) return;
  cudaSetDevice(L->d->id);
  if (L->w_raw) cudaFree(L->w_raw);
  if (L->w16) cudaFree(L->w16);
  if (L->scale) cudaFree(L->scale);
  if (L->bias) cudaFree(L->bias);
  release(L->a_hi);
  release(L->a_lo);
  delete L;
}

int g4m_vision_embed_device(g4m_ctx* ctx, int di, int n, const float* pixels_dev, int height, int width,
                            int max_soft_tokens, int layer_count, float* out_dev, void* stream) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || n < 0 || (n > 0 && (!pixels_dev || !out_dev)))
    return fail(G4M_E_ARG, "bad argument");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  cudaStream_t st = stream ? (cudaStream_t)stream : cudaStreamLegacy;  // NULL: the default stream
  return vision_forward(ctx, d, n, pixels_dev, height, width, max_soft_tokens, layer_count, out_dev, st);
}

int g4m_vision_embed_batch(g4m_ctx* ctx, int n, const float* const* pixels, int height, int width, int max_soft_tokens,
                           int layer_count, float* const* out, int* rows_out, int* status) {
  if (!ctx || n < 0 || (n > 0 && (!pixels || !out))) return fail(G4M_E_ARG, "bad argument");
  int tokens = 0;
  int rc = vision_tokens_for(height, width, max_soft_tokens, &tokens);
  if (rc) {
    for (int i = 0; i < n; ++i) {
      if (rows_out) rows_out[i] = 0;
      if (status) status[i] = rc;
    }
    return rc;
  }
  const int G = (int)ctx->devs.size();
  std::vector<int> rcs(G, G4M_OK);
  std::vector<std::string> msgs(G);
  auto work = [&](int g) {
    const int lo = (int)((long)n * g / G), hi = (int)((long)n * (g + 1) / G), cnt = hi - lo;
    if (cnt <= 0) return;
    Device& d = *ctx->devs[g];
    std::lock_guard<std::mutex> lk(d.mu);
    cudaSetDevice(d.id);
    const size_t img = (size_t)height * width * 3, ob = (size_t)tokens * 1536;
    int r = G4M_OK;
    if (ensure(d.io_in, cnt * img * 4) || ensure(d.io_out, cnt * ob * 4)) r = fail(G4M_E_CUDA, "io allocation failed");
    // 8-image head and tail chunks around middle chunks of <= 48 images:
    // uploads queue on the copy stream, each chunk's forward waits for its
    // upload, each download for its forward.  Measured at 64 images: 8 | 48 | 8
    // ends 1.2 % sooner than 4 | 28 | 28 | 4 (the exposed first upload grows
    // by 28 MB, but the edge chunks fill their GEMM tile waves)
    const auto chunks = edge_chunks(cnt, 8, 48);
    std::vector<cudaEvent_t> up(chunks.size()), done(chunks.size());
    for (size_t k = 0; k < chunks.size(); ++k) {
      cudaEventCreateWithFlags(&up[k], cudaEventDisableTiming);
      cudaEventCreateWithFlags(&done[k], cudaEventDisableTiming);
    }
    for (size_t k = 0; !r && k < chunks.size(); ++k) {
      for (int i = chunks[k].first; !r && i < chunks[k].second; ++i)
        if (cudaMemcpyAsync((float*)d.io_in.p + i * img, pixels[lo + i], img * 4, cudaMemcpyHostToDevice, d.cst))
          r = fail(G4M_E_CUDA, "pixel upload failed");
      if (!r && cudaEventRecord(up[k], d.cst)) r = fail(G4M_E_CUDA, "event record failed");
    }
    for (size_t k = 0; !r && k < chunks.size(); ++k) {
      const int c0 = chunks[k].first, cn = chunks[k].second - c0;
      if (cudaStreamWaitEvent(d.st, up[k], 0)) r = fail(G4M_E_CUDA, "stream wait failed");
      if (!r)
        r = vision_forward(ctx, d, cn, (const float*)d.io_in.p + c0 * img, height, width, max_soft_tokens,
                           layer_count, (float*)d.io_out.p + c0 * ob, d.st);
      if (!r && (cudaEventRecord(done[k], d.st) || cudaStreamWaitEvent(d.cst, done[k], 0)))
        r = fail(G4M_E_CUDA, "event record failed");
      for (int i = c0; !r && i < c0 + cn; ++i)
        if (cudaMemcpyAsync(out[lo + i], (float*)d.io_out.p + i * ob, ob * 4, cudaMemcpyDeviceToHost, d.cst))
          r = fail(G4M_E_CUDA, "embedding download failed");
    }
    const int rs = finish(d, d.st);
    const cudaError_t ce = cudaStreamSynchronize(d.cst);
    for (size_t k = 0; k < chunks.size(); ++k) {
      cudaEventDestroy(up[k]);
      cudaEventDestroy(done[k]);
    }
    if (!r) r = rs;
    if (!r && ce != cudaSuccess) r = fail(G4M_E_CUDA, std::string("copy stream: ") + cudaGetErrorString(ce));
    rcs[g] = r;
    if (r) msgs[g] = tl_err;
  };
  if (G == 1) work(0);
  else {
    std::vector<std::thread> th;
    for (int g = 0; g < G; ++g) th.emplace_back(work, g);
    for (auto& t : th) t.join();
  }
  int first = G4M_OK;
  for (int g = 0; g < G; ++g) {
    const int lo = (int)((long)n * g / G), hi = (int)((long)n * (g + 1) / G);
    for (int i = lo; i < hi; ++i) {
      if (rows_out) rows_out[i] = rcs[g] ? 0 : tokens;
      if (status) status[i] = rcs[g];
    }
    if (rcs[g] && !first) {
      first = rcs[g];
      tl_err = msgs[g];
    }
  }
  return first;
}

int g4m_resize_rgb(g4m_ctx* ctx, int di, const uint8_t* src, int height, int width, int channels, int target_height,
                   int target_width, float* dst) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || !src || !dst || height <= 0 || width <= 0 ||
      target_height <= 0 || target_width <= 0 || (channels != 3 && channels != 4))
    return fail(G4M_E_ARG, "bad argument");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  (void)cudaGetLastError();
  const size_t nsrc = (size_t)height * width * channels, ntmp = (size_t)height * target_width * 3,
               ndst = (size_t)target_height * target_width * 3;
  if (ensure(d.io_src, nsrc) || ensure(d.io_tmp, ntmp * 4) || ensure(d.io_out, ndst * 4))
    return fail(G4M_E_CUDA, "resize buffer allocation failed");
  G4M_LAUNCH(cudaMemcpyAsync(d.io_src.p, src, nsrc, cudaMemcpyHostToDevice, d.st));
  cudaStream_t st = d.st;
  G4M_RUN("resize", vision_resize((const uint8_t*)d.io_src.p, height, width, channels, target_height, target_width,
                                  (float*)d.io_tmp.p, (float*)d.io_out.p, st));
  G4M_LAUNCH(cudaMemcpyAsync(dst, d.io_out.p, ndst * 4, cudaMemcpyDeviceToHost, d.st));
  return finish(d, d.st);
}

int g4m_vision_embed_images(g4m_ctx* ctx, int n, const uint8_t* const* images, const int* heights, const int* widths,
                            int channels, int max_soft_tokens, int layer_count, float* const* out, int* rows_out,
                            int* status) {
  if (!ctx || n < 0 || (n > 0 && (!images || !heights || !widths || !out))) return fail(G4M_E_ARG, "bad argument");
  if (channels != 3 && channels != 4) return fail(G4M_E_ARG, "channels must be 3 (RGB) or 4 (RGBA)");
  // token layout of every image (computeGemma4ImageTokenLayout), grouped by target size
  std::vector<int64_t> lay((size_t)n * 6);
  std::vector<int> rcs(n, G4M_OK);
  std::vector<std::string> msgs(n);
  std::vector<std::pair<long, int>> keyed;
  for (int i = 0; i < n; ++i) {
    if (rows_out) rows_out[i] = 0;
    rcs[i] = image_layout(heights[i], widths[i], 16, max_soft_tokens, 3, &lay[(size_t)i * 6]);
    if (rcs[i]) msgs[i] = tl_err;
    else keyed.push_back({lay[(size_t)i * 6] * 100000L + lay[(size_t)i * 6 + 1], i});
  }
  std::stable_sort(keyed.begin(), keyed.end());
  const int G = (int)ctx->devs.size();
  for (size_t a = 0; a < keyed.size();) {
    size_t b = a;
    while (b < keyed.size() && keyed[b].first == keyed[a].first) ++b;
    std::vector<int> grp;
    for (size_t k = a; k < b; ++k) grp.push_back(keyed[k].second);
    a = b;
    const int th = (int)lay[(size_t)grp[0] * 6], tw = (int)lay[(size_t)grp[0] * 6 + 1];
    const int tokens = (int)lay[(size_t)grp[0] * 6 + 5];
    const int m = (int)grp.size();
    auto work = [&](int g) {
      const int lo = (int)((long)m * g / G), hi = (int)((long)m * (g + 1) / G), cnt = hi - lo;
      if (cnt <= 0) return;
      Device& d = *ctx->devs[g];
      std::lock_guard<std::mutex> lk(d.mu);
      cudaSetDevice(d.id);
      (void)cudaGetLastError();
      const size_t img = (size_t)th * tw * 3, ob = (size_t)tokens * 1536;
      size_t src_total = 0, tmp_max = 0;
      for (int k = lo; k < hi; ++k) {
        const int i = grp[k];
        src_total += (size_t)heights[i] * widths[i] * channels;
        tmp_max = std::max(tmp_max, (size_t)heights[i] * tw * 3);
      }
      int r = G4M_OK;
      if (ensure(d.io_src, src_total) || ensure(d.io_tmp, tmp_max * 4) || ensure(d.io_in, cnt * img * 4) ||
          ensure(d.io_out, cnt * ob * 4))
        r = fail(G4M_E_CUDA, "io allocation failed");
      cudaStream_t st = d.st;
      size_t off = 0;
      for (int k = lo; !r && k < hi; ++k) {  // upload and resize each source to the group's target size
        const int i = grp[k];
        const size_t bytes = (size_t)heights[i] * widths[i] * channels;
        if (cudaMemcpyAsync((uint8_t*)d.io_src.p + off, images[i], bytes, cudaMemcpyHostToDevice, st) ||
            vision_resize((const uint8_t*)d.io_src.p + off, heights[i], widths[i], channels, th, tw,
                          (float*)d.io_tmp.p, (float*)d.io_in.p + (size_t)(k - lo) * img, st))
          r = fail(G4M_E_CUDA, "image upload / resize failed");
        g_launches.fetch_add(2, std::memory_order_relaxed);
        off += bytes;
      }
      if (!r) r = vision_forward(ctx, d, cnt, (const float*)d.io_in.p, th, tw, max_soft_tokens, layer_count,
                                 (float*)d.io_out.p, st);
      for (int k = lo; !r && k < hi; ++k)
        if (cudaMemcpyAsync(out[grp[k]], (float*)d.io_out.p + (size_t)(k - lo) * ob, ob * 4, cudaMemcpyDeviceToHost, st))
          r = fail(G4M_E_CUDA, "embedding download failed");
      if (!r) r = finish(d, st);
      for (int k = lo; k < hi; ++k) {
        rcs[grp[k]] = r;
        if (r) msgs[grp[k]] = tl_err;
        else if (rows_out) rows_out[grp[k]] = tokens;
      }
    };
    if (G == 1) work(0);
    else {
      std::vector<std::thread> ths;
      for (int g = 0; g < G; ++g) ths.emplace_back(work, g);
      for (auto& t : ths) t.join();
    }
  }
  int first = G4M_OK;
  for (int i = 0; i < n; ++i) {
    if (status) status[i] = rcs[i];
    if (rcs[i] && !first) {
      first = rcs[i];
      tl_err = msgs[i];
    }
  }
  return first;
}

int g4m_selftest_wait_timeout(g4m_ctx* ctx, int di, long long budget_cycles) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || budget_cycles <= 0 || budget_cycles > 4000000000LL)
    return fail(G4M_E_ARG, "bad argument");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  (void)cudaGetLastError();
  cudaStream_t st = d.st;
  G4M_RUN("selftest_wait", selftest_wait_timeout(d.err, budget_cycles, st));
  return finish(d, st);  // reads and clears the error word: G4M_E_TIMEOUT expected
}

int g4m_vision_debug_hidden(g4m_ctx* ctx, int di, int which, float* host, size_t count) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || !host) return fail(G4M_E_ARG, "bad argument");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  const size_t need_n = (size_t)d.last_vision_rows * 768;
  const DevBuf& src = which == 0 ? d.vb.h0 : d.vb.h;
  if (!src.p || need_n == 0) return fail(G4M_E_ARG, "no vision stage output is available");
  if (count < need_n) return fail(G4M_E_ARG, "host buffer too small");
  if (cudaStreamSynchronize(d.st) || cudaMemcpy(host, src.p, need_n * 4, cudaMemcpyDeviceToHost))
    return fail(G4M_E_CUDA, "stage download failed");
  return G4M_OK;
}

int g4m_vision_layers(g4m_ctx* ctx, int di, int n, int height, int width, int first, int count, float* h) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || !h || n <= 0) return fail(G4M_E_ARG, "bad argument");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  if (first < 0 || count < 1 || first + count > d.vw.layers) return fail(G4M_E_ARG, "layer range outside the checkpoint");
  int rc = vision_check_quant(d.vw, first + count);
  if (rc) return rc;
  const int gh = height / 16, gw = width / 16, N = gh * gw;
  if (gh * 16 != height || gw * 16 != width || gh % 3 || gw % 3) return fail(G4M_E_SHAPE, "image size must be a multiple of 48");
  rc = ensure_vision_layout(d, gh, gw, (gh / 3) * (gw / 3));
  if (rc) return rc;
  const long M = (long)n * N;
  rc = ensure_vision_buffers(d, n, N, (long)n * (gh / 3) * (gw / 3));
  if (rc) return rc;
  VisionBuffers& b = d.vb;
  cudaStream_t st = d.st;
  G4M_LAUNCH(cudaMemcpyAsync(b.h.p, h, M * 768 * 4, cudaMemcpyHostToDevice, st));
  RowArgs r;
  memset(&r, 0, sizeof(r));
  r.rows = M;
  r.d = 768;
  r.eps = 1e-6f;
  r.h_in = (const float*)b.h.p;
  r.w_next = d.vw.L[first].n_in;
  next_scales(r, d.vw.L[first].sin_qkv, 3, (__half*)b.a_c.p);
  r.a_hi = (__half*)b.a_hi.p;
  r.a_lo = (__half*)b.a_lo.p;
  r.lda = 768;
  G4M_RUN("rows", fused_rows(r, st));
  rc = vision_layer_range(ctx, d, n, N, first, count, st);
  if (rc) return rc;
  G4M_LAUNCH(cudaMemcpyAsync(h, b.h.p, M * 768 * 4, cudaMemcpyDeviceToHost, st));
  return finish(d, st);
}

int g4m_profile_begin(g4m_ctx* ctx, int di) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size()) return fail(G4M_E_ARG, "bad context or device index");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  d.prof.clear();
  d.ev_used = 0;
  d.prof_on = true;
  return G4M_OK;
}

int g4m_profile_end(g4m_ctx* ctx, int di, char* buf, size_t cap) {
  if (!ctx || di < 0 || di >= (int)ctx->devs.size() || !buf || cap == 0) return fail(G4M_E_ARG, "bad argument");
  Device& d = *ctx->devs[di];
  std::lock_guard<std::mutex> lk(d.mu);
  cudaSetDevice(d.id);
  d.prof_on = false;
  std::vector<std::string> labels;
  std::vector<double> ms;
  std::vector<long> cnt;
  for (const ProfRec& r : d.prof) {
    if (cudaEventSynchronize(r.b) != cudaSuccess) return fail(G4M_E_CUDA, "profile event wait failed");
    float t = 0.f;
    cudaEventElapsedTime(&t, r.a, r.b);
    size_t i = 0;
    while (i < labels.size() && labels[i] != r.label) ++i;
    if (i == labels.size()) {
      labels.push_back(r.label);
      ms.push_back(0);
      cnt.push_back(0);
    }
    ms[i] += t;
    cnt[i] += 1;
  }
  std::string js = "{";
  for (size_t i = 0; i < labels.size(); ++i) {
    char tmp[160];
    snprintf(tmp, sizeof(tmp), "%s\"%s\": [%ld, %.6f]", i ? ", " : "", labels[i].c_str(), cnt[i], ms[i]);
    js += tmp;
  }
  js += "}";
  d.prof.clear();
  d.ev_used = 0;
  if (js.size() + 1 > cap) return fail(G4M_E_ARG, "profile buffer too small");
  memcpy(buf, js.c_str(), js.size() + 1);
  return G4M_OK;
}

long long g4m_kernel_launches(void) { return g_launches.load(); }

int g4m_image_token_layout(int height, int width, int patch_size, int max_soft_tokens, int pooling_kernel_size,
                           int64_t* out6) {
  if (!out6) return fail(G4M_E_ARG, "null output");
  return image_layout(height, width, patch_size, max_soft_tokens, pooling_kernel_size, out6);
}

int64_t g4m_audio_soft_token_count(int64_t samples, int frame_length, int hop_length, int audio_seq_length) {
  // computeGemma4AudioSoftTokenCount, src/preprocess/audio.ts:4-20
  const double fsu = frame_length + 1.0, pad_left = floor(frame_length / 2.0);
  const double nmel = floor(((double)samples + pad_left - fsu) / hop_length) + 1;
  if (nmel <= 0) return 0;
  double t = nmel;
  for (int l = 0; l < 2; ++l) t = floor((t + 2 * 1 - 3) / 2) + 1;
  return (int64_t)(t < audio_seq_length ? t : audio_seq_length);
}

double g4m_checksum_floats(const float* v, int64_t n) {
  // checksumFloats, src/utils/math.ts:3-12 (double arithmetic as in JS)
  const double mod = 1000000007.0;
  double c = 0;
  const int64_t lim = n < 4096 ? n : 4096;
  for (int64_t i = 0; i < lim; ++i) {
    const double x = (double)v[i] * 1000000.0, f = floor(x);
    const double r = (x - f >= 0.5) ? f + 1 : f;
    c = fmod(c + r * (double)(i + 1), mod);
    if (c < 0) c += mod;
  }
  return c;
}

}  // extern "C"
