// Internal kernel launch interface of the g4m library (not the public C ABI;
// that is include/g4m.h).  All launchers are asynchronous on `st`.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace g4m {

// srqScalar's integer code (src/kernels/qat.ts:489-492): clamp(round(v / s),
// -128, 127) with JS Math.round (ties toward +inf).  The quotient is v * (1/s)
// corrected once by its fma residual, q + (v - q s) / s (Markstein, IBM J.
// Res. Develop. 34(1), 1990), which recovers the rounded quotient v / s
// without a division per element; inv_s = 1 / s is computed once by the caller.
__device__ __forceinline__ float srq_code(float v, float s, float inv_s) {
  const float q0 = v * inv_s;
  const float q = fmaf(fmaf(-q0, s, v), inv_s, q0);
  const float f = floorf(q);
  const float r = (q - f >= 0.5f) ? f + 1.0f : f;
  return fminf(fmaxf(r, -128.0f), 127.0f);
}

enum Epi : int {
  EPI_F32 = 0,         // y = srq(acc * row_scale * col_scale[n], s_out) (+ bias[n]) -> f32
  EPI_GELU_GATE = 2,   // tile halves (gate | up) -> gelu_tanh(gate) * up -> fp16 hi/lo
  EPI_SILU = 3,        // silu(srq(acc * s_w)) -> fp16 hi/lo
  EPI_GLU = 4,         // tile halves (value | gate) -> value * sigmoid(gate) -> f32
  EPI_QKV_VISION = 5,  // head RMSNorm + 2-D RoPE + attention layouts (fp16 hi/lo)
  EPI_PATCH = 6,       // acc + pos_x row + pos_y row -> f32
};

// Static input-activation quantisation (input_activation_scale s != 0,
// srqScalar in src/kernels/qat.ts:489-492): an operand producer stores the
// integer code clamp(round(x / s), -128, 127) as a signed byte in place of
// the hi/lo split (a code plane of K bytes per row), the GEMM runs one
// kind::i8 term on the codes against int8 weights with exact int32
// accumulation, and its epilogue scales by s.  Projections that share an input (q / k / v, gate / up) keep their own
// s, so their GEMM selects the code plane per output region (amode):
//   amode 0  one A for the whole GEMM (terms 1..3 as above)
//   amode 1  one code plane per proj_width-column region, chosen per tile
//            (a_hi region 0, a_lo region 1, a_c region 2)
//   amode 2  tile halves: columns [0, BN/2) use a_hi, [BN/2, BN) a_lo (the
//            interleaved gate | up layout)
struct GemmOperands {
  const __half* a_hi;  // [M, K]
  const __half* a_lo;  // [M, K] (terms >= 2; amode 1/2: the second code plane)
  const __half* b_hi;  // [N, K]
  const __half* b_lo;  // [N, K] (terms == 3)
  const __half* a_c;   // [M, K] amode 1: the third code plane
};

struct GemmArgs {
  int M, N, K;
  // K chunking of the accumulation, in 64-wide k-blocks (0: one chunk).  The
  // tensor core adds each product into the running f32 accumulator with a
  // truncating alignment, so the accumulation error grows with the
  // accumulator's magnitude; with chunks, every chunk starts from zero in a
  // second TMEM buffer and the epilogue adds it into the tile's total with
  // round-to-nearest f32 adds.
  int chunk_kb;
  const float* col_scale;  // [N] per-output-channel weight scale (may be null for EPI_F32)
  float row_scale;         // 1, or s_in when A holds integer codes
  float row_scale_b;       // amode 1/2: s_in of region / half 1 (else = row_scale)
  float row_scale_c;       // amode 1: s_in of region 2
  float s_code;            // EPI_GELU_GATE / EPI_SILU: store codes for the next GEMM's s_in (0: hi/lo)
  float s_out, s_out_b, s_out_c;
  const float* bias;       // [N] or null
  float* out_f32;
  long ldo;
  __half* out_hi;
  __half* out_lo;
  long ldh;
  // EPI_QKV_VISION
  int proj_width;          // 768: columns of one of q / k / v
  int heads;
  float eps;
  const float* qn_w;       // [64]
  const float* kn_w;       // [64]
  const float* rope_cs;    // [rows_per_image][32] (cos, sin) pairs
  __half *q_hi, *q_lo, *k_hi, *k_lo, *vt_hi, *vt_lo;
  // EPI_QKV_VISION / EPI_PATCH
  int rows_per_image;
  int vt_pitch;            // row pitch (keys) of V^T, a multiple of 64
  const int* pos_xy;       // [rows_per_image][2]
  const float* posx_rows;  // [P][N]
  const float* posy_rows;  // [P][N]
  int* err;                // device error word
};

cudaError_t gemm_launch(int bn, int terms, int epi, const GemmOperands& op, const GemmArgs& args, cudaStream_t st,
                        int max_ctas = 0, int amode = 0);
bool make_tmap_f16(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);
bool make_tmap_i8(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);
// Any cols with a 16-byte-multiple row pitch `pitch_elems` (>= cols).
bool make_tmap_f16_any(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch_elems,
                       uint32_t box_rows);

cudaError_t prep_a(const float* x, long rows, int cols, float s_in, const float* row_scale, __half* hi, __half* lo,
                   cudaStream_t st);
cudaError_t prep_w(const void* src, int kind, int bits, int rows, int cols, const int* map, __half* hi, __half* lo,
                   cudaStream_t st);
cudaError_t prep_w_i8(const void* src, int kind, int bits, int rows, int cols, const int* map, int8_t* dst,
                      cudaStream_t st);

// ---------------------------------------------------------------------------
// Row kernels (norms, residuals) -- kernels_rows.cu
// ---------------------------------------------------------------------------
struct RowArgs {
  long rows;
  int d;
  float eps;
  const float* y;          // optional: delta to normalise (w_post) and add
  const float* w_post;     // RMSNorm weight applied to y (null: y added raw)
  float res_scale;         // h += res_scale * norm(y)
  const float* h_in;       // residual input (null: h = norm(y) or y)
  const float* w_out;      // optional RMSNorm of the new residual (audio norm_out)
  float* h_out;            // residual output (may alias h_in)
  const float* w_next;     // optional RMSNorm producing the next GEMM operand
  float s_in_next;         // 0: hi/lo planes.  Else signed-byte codes for s_in_next in a_hi (lda bytes per row),
  float s_in_b, s_in_c;    // and (when non-zero) codes for s_in_b in a_lo, for s_in_c in a_c
  __half* a_hi;
  __half* a_lo;
  __half* a_c;
  long lda;
};
cudaError_t fused_rows(const RowArgs& r, cudaStream_t st);
// One-warp kernel whose bounded wait expires after `budget` cycles (sets *err).
cudaError_t selftest_wait_timeout(int* err, long long budget, cudaStream_t st);

// Vision helpers -- kernels_vision.cu
cudaError_t vision_patch_operand(const float* pixels, int n_images, int height, int width, int patch, __half* hi,
                                 __half* lo, cudaStream_t st);
cudaError_t vision_pool_operand(const float* h, const int* pool_idx, int n_images, int rows_per_image, int tokens,
                                int k2, int d, float eps, float* pooled_out, __half* hi, __half* lo, cudaStream_t st);
// RGB(A) uint8 [h][w][c] (c = 3 or 4) -> [th][tw][3] f32 in [0, 1]: antialiased
// linear resize, 8-bit rounding, 1/255 rescale.  tmp: [h][tw][3] f32.
cudaError_t vision_resize(const uint8_t* src, int h, int w, int c, int th, int tw, float* tmp, float* dst,
                          cudaStream_t st);
// s_code != 0: O is stored as signed-byte codes for the o_proj input scale (o_hi only, 768 bytes per row).
cudaError_t vision_attention_simt(const __half* q_hi, const __half* q_lo, const __half* k_hi, const __half* k_lo,
                                  const __half* vt_hi, const __half* vt_lo, int bh, int n, int vt_pitch, int heads,
                                  __half* o_hi, __half* o_lo, float s_code, cudaStream_t st);
cudaError_t vision_attention_tc(const __half* q_hi, const __half* q_lo, const __half* k_hi, const __half* k_lo,
                                const __half* vt_hi, const __half* vt_lo, int bh, int n, int vt_pitch, int heads,
                                __half* o_hi, __half* o_lo, float s_code, int* err, cudaStream_t st);

// Audio helpers -- kernels_audio.cu
// mel_rng: [128][2] first / last non-zero FFT bin of each mel channel.
cudaError_t audio_logmel(const float* samples, const long* sample_off, const long* sample_len, const int* frame_off,
                         const int* frames, int clips, int total_frames, const float* window, const float* mel,
                         const int* mel_rng, const double2* twiddle, float* features, cudaStream_t st);
// Subsample convs.  Layer-0 rows of clip i start at row t0off[i] of the fp16
// hi / lo planes l0h, l0l ([l0_rows][64][128]; a zero row precedes and
// follows every clip); output rows at packed row row0[i], rows[i] of them.
// w0: layer-0 weights [128][9]; w0stat: their moments (wbar[9], then
// G[k][l] for k <= l, 45 values) for the LayerNorm statistics;
// w1_hi / w1_lo: layer-1 weights [9 taps][32 out][128 in].  (subsample_sm100.cu)
cudaError_t audio_subsample_tc(const float* feats, const int* frame_off, const int* frames, const int* t0off,
                               long l0_rows, const int* row0, const int* rows, int clips, int max_t0, int max_rows,
                               const float* w0, const double* w0stat, const float* n0, const __half* w1_hi,
                               const __half* w1_lo, const float* n1, float eps, __half* l0h, __half* l0l,
                               __half* a_hi, __half* a_lo, int* err, cudaStream_t st);
// Chunked audio attention over runs of up to kAudioAttnRun consecutive
// 12-row blocks: run i covers blocks [run_blk0[i], +kAudioAttnRun) of clip
// run_clip[i], clipped to the clip's block count.
constexpr int kAudioAttnRun = 8;
cudaError_t audio_attention_blocks(const float* qkv, const float* relk, const float* qmul, const int* run_clip,
                                   const int* run_blk0, int nruns, const int* row0, const int* rows, float kscale,
                                   float softcap, __half* o_hi, __half* o_lo, float s_code, cudaStream_t st);
cudaError_t audio_lconv_rows(const float* g, const float* dw, const float* nw, const int* row_clip, const int* row0,
                             long rows, float eps, __half* a_hi, __half* a_lo, float s_code, int* err,
                             cudaStream_t st);
cudaError_t gather_rows(const float* src, const int* rows_idx, long n, int d, float* dst, cudaStream_t st);
cudaError_t row_inv_rms_operand(const float* x, long rows, int d, float eps, __half* hi, __half* lo, cudaStream_t st);
cudaError_t add_bias_rows(float* y, const float* b, long rows, int d, cudaStream_t st);

}  // namespace g4m
