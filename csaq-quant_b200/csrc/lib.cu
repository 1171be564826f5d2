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

#ifdef CSAQ_CHECKED
namespace {
struct GuardReader {
  int (*read)(unsigned long long*, long long*);
  int (*clear)();
};
// filled during static initialisation of the library's translation units
GuardReader g_readers[16];
int g_n_readers = 0;
}  // namespace
void register_guard_reader(int (*read)(unsigned long long*, long long*), int (*clear)()) {
  if (g_n_readers < 16) g_readers[g_n_readers++] = GuardReader{read, clear};
}
#endif
}  // namespace csaq

extern "C" int csaq_checked_build(void) {
#ifdef CSAQ_CHECKED
  return 1;
#else
  return 0;
#endif
}

extern "C" int csaq_guard_report(int64_t* count, int64_t* site, int64_t* value, int64_t* bound) {
  if (!count || !site || !value || !bound) return CSAQ_ERR_ARG;
  *count = *site = *value = *bound = 0;
#ifdef CSAQ_CHECKED
  if (cudaDeviceSynchronize() != cudaSuccess) return csaq::launch_status();
  for (int i = 0; i < csaq::g_n_readers; ++i) {
    unsigned long long n = 0;
    long long first[3] = {0, 0, 0};
    const int rc = csaq::g_readers[i].read(&n, first);
    if (rc) return rc;
    if (n && *count == 0) {
      *site = first[0];
      *value = first[1];
      *bound = first[2];
    }
    *count += (int64_t)n;
  }
  return CSAQ_OK;
#else
  return CSAQ_ERR_UNSUPPORTED;
#endif
}

extern "C" int csaq_guard_clear(void) {
#ifdef CSAQ_CHECKED
  if (cudaDeviceSynchronize() != cudaSuccess) return csaq::launch_status();
  for (int i = 0; i < csaq::g_n_readers; ++i) {
    const int rc = csaq::g_readers[i].clear();
    if (rc) return rc;
  }
  return CSAQ_OK;
#else
  return CSAQ_ERR_UNSUPPORTED;
#endif
}

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
