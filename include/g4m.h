/*
 * g4m.h -- C ABI of the B200 (sm_100a) Gemma 4 E2B media towers.
 *
 * Drop-in boundary for the compute path of ClinDesk-AI/gemma-4-webgpu-kernels-multimodal.
 * Plain pointers and sizes only; no CUDA or framework types.  Every function
 * returns G4M_OK (0) or a G4M_E_* status; g4m_last_error() returns the
 * message of the calling thread's last failure.  Host buffers are owned by
 * the caller and are not retained past return.
 */
#ifndef G4M_H
#define G4M_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4M_ABI_VERSION 1

#if defined(G4M_BUILD) && defined(__GNUC__)
#define G4M_API __attribute__((visibility("default")))
#else
#define G4M_API
#endif

enum g4m_status {
  G4M_OK = 0,
  G4M_E_ARG = 1,         /* invalid argument */
  G4M_E_SHAPE = 2,       /* dimensions do not match (reference: "... does not match dimensions") */
  G4M_E_DTYPE = 3,       /* tensor dtype / shape assert failed (src/io/safetensors.ts:177-190) */
  G4M_E_CUDA = 4,        /* CUDA runtime error */
  G4M_E_TIMEOUT = 5,     /* a device-side bounded wait expired (error word set by a kernel) */
  G4M_E_CANCELLED = 6,   /* g4m_cancel() observed between layers (AbortSignal in the reference) */
  G4M_E_IO = 7,          /* checkpoint file missing or malformed */
  G4M_E_NOT_LOADED = 8,  /* the tower's weights are not loaded */
  G4M_E_UNSUPPORTED = 9, /* valid input this build does not handle (message says which) */
  G4M_E_LAYOUT = 10      /* image layout error (src/preprocess/image.ts:225,237,249) */
};

typedef struct g4m_ctx g4m_ctx;
typedef struct g4m_linear g4m_linear;

/* ------------------------------------------------------------------ context */

/* Create a context on `n_devices` CUDA devices (NULL/0: device 0).  Replaces
 * the per-call navigator.gpu adapter/device request of
 * src/vision/index.ts:29-37 and src/audio/index.ts:41-49; a context lives
 * across calls and keeps weights resident. */
G4M_API g4m_ctx* g4m_create(const int* devices, int n_devices);
G4M_API void g4m_destroy(g4m_ctx* ctx);
G4M_API int g4m_device_count(const g4m_ctx* ctx);

/* Message of the calling thread's last failure ("" if none). */
G4M_API const char* g4m_last_error(void);

/* Load every vision / audio / embedder tensor present in a local
 * safetensors file onto each device of the context, converted once into the
 * kernels' resident layouts.  Replaces the per-layer, per-call tensor fetches
 * (loadSafetensorsTensorData, src/io/safetensors.ts:24-77, and the loaders in
 * src/vision/encoder.ts, src/audio/encoder.ts, src/kernels/qat.ts:159-197)
 * with their dtype/shape asserts. */
G4M_API int g4m_load_weights(g4m_ctx* ctx, const char* safetensors_path);
/* Bit 0: vision tower + embedder loaded; bit 1: audio tower + embedder loaded. */
G4M_API int g4m_loaded_towers(const g4m_ctx* ctx);

/* Request cancellation of running embed calls; they stop between layers
 * and return G4M_E_CANCELLED (AbortSignal checks, src/vision/encoder.ts:179). */
G4M_API void g4m_cancel(g4m_ctx* ctx);
G4M_API void g4m_clear_cancel(g4m_ctx* ctx);

/* Keep stage outputs for g4m_vision_debug_hidden (off by default: it adds a
 * device copy of the patch embeddings per call). */
G4M_API int g4m_set_debug(g4m_ctx* ctx, int on);

/* ----------------------------------------------------------- QAT linear */

/* y[rows,out] = srq(fround(sum_c srq(x[r,c], s_in) * w[o,c]) * w_scale[o], s_out) (+ bias[o])
 * on device `device_index` of the context; host pointers.
 *   bits == 0: w is int8 [out, in]                (runQatI8LinearWebGpu, src/kernels/qat.ts:601-759)
 *   bits 2/4/8: w is uint8 packed codes [out, in*bits/8], zero point 2^(bits-1)
 *                                                  (runPackedQatLinearWebGpu, src/kernels/qat.ts:263-432)
 * bias may be NULL; with a bias the output is fround(y + bias) as the audio
 * output projection does (src/audio/kernels.ts:405-411). */
G4M_API int g4m_qat_linear(g4m_ctx* ctx, int device_index, const float* x, int rows, int in, int out, const void* w, int bits,
                   const float* w_scale, float s_in, float s_out, const float* bias, float* y);

/* Resident-weight form of g4m_qat_linear for callers that keep activations
 * in device memory: prepare once (host weights), then run on device
 * pointers on the given CUDA stream (NULL = default stream). */
G4M_API int g4m_linear_prepare(g4m_ctx* ctx, int device_index, const void* w, int bits, int out, int in, const float* w_scale,
                       float s_in, float s_out, const float* bias, g4m_linear** out_linear);
G4M_API int g4m_linear_run(g4m_linear* lin, const float* x_dev, int rows, float* y_dev, void* stream);
G4M_API void g4m_linear_free(g4m_linear* lin);

/* g4m_linear_run without any device allocation (no reference counterpart:
 * the reference's WebGPU runner creates its buffers per call).  The fp16
 * activation operand is staged in a static 16 MiB device array (two planes
 * of 4,194,304 elements) instead of a per-linear buffer grown by cudaMalloc,
 * so a call never allocates, frees or grows memory.  Limit: rows * in <=
 * 4,194,304, else G4M_E_SHAPE and nothing is launched.  The first call on
 * each device looks up the array's address (cudaGetSymbolAddress, which may
 * load the module); make that first call before any stream capture.  All
 * calls on one device share the array: calls in flight at the same time on
 * one device race and must be serialised by the caller. */
G4M_API int g4m_linear_run_noalloc(g4m_linear* lin, const float* x_dev, int rows, float* y_dev, void* stream);

/* ------------------------------------------------------------- vision */

/* Image embeddings for n images of one size (computeGemma4VisionImageEmbeddings,
 * src/vision/index.ts:12-148, batched).  pixels[i] is RGB float32
 * [height][width][3] in [0, 1] (uint8 / 255 as the reference rescales,
 * src/preprocess/image.ts:145-147), already at the token layout's target
 * size.  out[i] receives [soft_tokens][1536] float32; rows_out[i] the token
 * count; status[i] the per-image status.  Images are sharded across the
 * context's devices. */
G4M_API int g4m_vision_embed_batch(g4m_ctx* ctx, int n, const float* const* pixels, int height, int width,
                           int max_soft_tokens, int layer_count, float* const* out, int* rows_out, int* status);

/* Device-resident form on one device: pixels_dev is [n][height][width][3],
 * out_dev [n * soft_tokens][1536]; asynchronous on `stream` (NULL = default). */
G4M_API int g4m_vision_embed_device(g4m_ctx* ctx, int device_index, int n, const float* pixels_dev, int height, int width,
                            int max_soft_tokens, int layer_count, float* out_dev, void* stream);

/* Image embeddings for n decoded 8-bit images of any size
 * (computeGemma4VisionImageEmbeddings with preprocessGemma4ImageBlob,
 * src/vision/index.ts:12-148, src/preprocess/image.ts:104-162, batched):
 * images[i] is RGB or RGBA uint8 [heights[i]][widths[i]][channels].  Each
 * image is resized on the device to its token layout's target size
 * (antialiased linear filter, 8-bit rounding, 1/255 rescale) and embedded;
 * images with the same target size share a batch.  out[i] receives
 * [soft_tokens_i][1536] float32, rows_out[i] the token count, status[i]. */
G4M_API int g4m_vision_embed_images(g4m_ctx* ctx, int n, const uint8_t* const* images, const int* heights,
                                    const int* widths, int channels, int max_soft_tokens, int layer_count,
                                    float* const* out, int* rows_out, int* status);

/* The resize step of g4m_vision_embed_images on its own (host buffers):
 * uint8 [height][width][channels] -> float32 [target_height][target_width][3]
 * in [0, 1] (replaces the canvas drawImage + getImageData * rescaleFactor of
 * src/preprocess/image.ts:121-151). */
G4M_API int g4m_resize_rgb(g4m_ctx* ctx, int device_index, const uint8_t* src, int height, int width, int channels,
                           int target_height, int target_width, float* dst);

/* Stage outputs of the last g4m_vision_embed_device call on a device, for
 * layer-anchored parity checks: which = 0 patch embeddings [n*N][768],
 * 1 final hidden states [n*N][768].  Host copy; returns G4M_E_ARG if the
 * buffer is too small. */
G4M_API int g4m_vision_debug_hidden(g4m_ctx* ctx, int device_index, int which, float* host, size_t count);

/* Run layers [first, first+count) of the vision stack on host hidden
 * states h[n*N][768] in place (image size gives N and positions). */
G4M_API int g4m_vision_layers(g4m_ctx* ctx, int device_index, int n, int height, int width, int first, int count, float* h);

/* -------------------------------------------------------------- audio */

/* Audio embeddings for n clips (computeGemma4AudioEmbeddings,
 * src/audio/index.ts:12-183, batched).  samples[i] has lengths[i] mono
 * float32 samples at sampling_rate; max_samples caps each clip (0: 480000).
 * out[i] receives [rows_out[i]][1536] float32 (rows_out[i] <= 750); the
 * caller sizes out[i] for g4m_audio_soft_token_count(...) rows. */
G4M_API int g4m_audio_embed_batch(g4m_ctx* ctx, int n, const float* const* samples, const int64_t* lengths,
                          int sampling_rate, int layer_count, int64_t max_samples, float* const* out, int* rows_out,
                          int* status);

/* Device-resident form on one device: samples_dev holds the clips back to
 * back (offsets[i], lengths[i] in samples, host arrays); out_dev receives the
 * valid rows of every clip back to back; rows_out[i] per clip (host). */
G4M_API int g4m_audio_embed_device(g4m_ctx* ctx, int device_index, int n, const float* samples_dev, const int64_t* offsets,
                           const int64_t* lengths, int sampling_rate, int layer_count, int64_t max_samples,
                           float* out_dev, int* rows_out, void* stream);

/* Stage outputs of the last audio call on a device, packed rows, for
 * stage-anchored parity checks: which = 0 encoder input [rows][1024] (after
 * the subsample input projection; needs g4m_set_debug), 1 encoder output
 * [rows][1024] (after norm_out of the last layer), 2 the q | k | v
 * projections of the last layer run [rows][3072]. */
G4M_API int g4m_audio_debug_hidden(g4m_ctx* ctx, int device_index, int which, float* host, size_t count);

/* Run conformer layers [first, first+count) on host hidden states h
 * ([sum(rows_per_clip)][1024], clips packed back to back) in place. */
G4M_API int g4m_audio_layers(g4m_ctx* ctx, int device_index, int n, const int* rows_per_clip, int first, int count,
                             float* h);

/* ------------------------------------------------- host layout helpers */

/* computeGemma4ImageTokenLayout, src/preprocess/image.ts:4-30.
 * out6 = {target_h, target_w, grid_h, grid_w, max_patches, soft_tokens}. */
G4M_API int g4m_image_token_layout(int height, int width, int patch_size, int max_soft_tokens, int pooling_kernel_size,
                           int64_t* out6);

/* computeGemma4AudioSoftTokenCount, src/preprocess/audio.ts:4-20. */
G4M_API int64_t g4m_audio_soft_token_count(int64_t samples, int frame_length, int hop_length, int audio_seq_length);

/* checksumFloats, src/utils/math.ts:3-12 (first 4096 values). */
G4M_API double g4m_checksum_floats(const float* values, int64_t count);

/* ------------------------------------------------------ instrumentation */

/* Self-test of the device-side failure detection (no reference counterpart):
 * launches one warp that waits on a barrier nothing arrives on, through the
 * kernels' bounded wait with a budget of budget_cycles (1 .. 4e9), and
 * returns the resulting status: G4M_E_TIMEOUT with the kernel's error code in
 * g4m_last_error().  The error word is cleared, so the context stays usable.
 * Nothing faults or hangs. */
G4M_API int g4m_selftest_wait_timeout(g4m_ctx* ctx, int device_index, long long budget_cycles);

/* Per-launch CUDA-event timing on one device: begin, run calls, end.  The
 * end call waits for the recorded events and writes a JSON object
 * {"label": [launches, total_ms], ...} into buf. */
G4M_API int g4m_profile_begin(g4m_ctx* ctx, int device_index);
G4M_API int g4m_profile_end(g4m_ctx* ctx, int device_index, char* buf, size_t cap);

/* Kernels this library has launched in the process so far. */
G4M_API long long g4m_kernel_launches(void);

/* Library build identification (e.g. "g4m sm_100a abi 1"). */
G4M_API const char* g4m_version(void);

#ifdef __cplusplus
}
#endif

#endif /* G4M_H */
