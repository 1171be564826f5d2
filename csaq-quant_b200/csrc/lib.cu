// Library identification, status strings and the per-thread CUDA error record.
#include <cstdlib>

#include "common.cuh"

namespace csaq {
static thread_local int g_last_cuda_error = 0;
void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = (int)e; }
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("CSAQ_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}
}  // namespace csaq

extern "C" const char* csaq_version(void) { return "csaq-b200 0.1.0 (sm_100a)"; }

extern "C" int csaq_last_cuda_error(void) { return csaq::g_last_cuda_error; }

extern "C" const char* csaq_status_string(int status) {
  switch (status) {
    case CSAQ_OK: return "ok";
    case CSAQ_ERR_ARG: return "invalid argument";
    case CSAQ_ERR_BITS: return "unsupported bit-width";
    case CSAQ_ERR_CUDA: return "CUDA launch failed";
    case CSAQ_ERR_TIMEOUT: return "bounded device wait timed out";
    case CSAQ_ERR_UNSUPPORTED: return "shape or alignment not supported by this kernel";
    case CSAQ_ERR_SCRATCH: return "call needs more scratch than the static buffer of csaq_decode_attention_static holds";
    default: return "unknown status";
  }
}
