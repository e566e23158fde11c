// Audio tower (placeholder until the conformer kernels land).
#include "../../include/g4m.h"
#include "g4m_kernels.h"
#include "runtime_internal.h"
#include "safetensors.h"

namespace g4m {
int load_audio(Device& d, const SafeTensors& f) {
  (void)d;
  (void)f;
  return G4M_OK;
}
}  // namespace g4m

using namespace g4m;
extern "C" {
int g4m_audio_embed_batch(g4m_ctx*, int, const float* const*, const int64_t*, int, int, int64_t, float* const*, int*,
                          int*) {
  return fail(G4M_E_UNSUPPORTED, "audio tower not built yet");
}
int g4m_audio_embed_device(g4m_ctx*, int, int, const float*, const int64_t*, const int64_t*, int, int, int64_t, float*,
                           int*, void*) {
  return fail(G4M_E_UNSUPPORTED, "audio tower not built yet");
}
}
