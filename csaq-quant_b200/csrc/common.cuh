// Shared device helpers for the csaq B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "csaq_b200.h"

namespace csaq {

// Thread-local record of the last CUDA launch error (csaq_last_cuda_error).
void set_last_cuda_error(cudaError_t e);

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return CSAQ_ERR_CUDA;
  }
  return CSAQ_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ── programmatic dependent launch ──────────────────────────────────────────
// A kernel started with launch_pdl may begin while its predecessor in the
// stream is still running. pdl_wait() returns once the predecessor grid has
// completed and its memory is visible; pdl_trigger() lets this grid's own
// successor be scheduled. For a plain launch both are no-ops. Every kernel
// launched this way calls pdl_wait() before it touches memory that another
// kernel of the stream writes. Kernels that do not prefetch call pdl_trigger()
// only after pdl_wait(), so at most one grid waits ahead of a running one and
// waiting grids do not pile up on the SMs. CSAQ_PDL=0 in the environment turns
// it off.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                      Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    (void)cudaGetLastError();
    return CSAQ_ERR_CUDA;
  }
  return launch_status();
}

// ── checked builds ──────────────────────────────────────────────────────────
// Built with -DCSAQ_CHECKED, CSAQ_GUARD(ok, site, value, bound) counts a failed
// index test in this translation unit's record, keeps the first failure's
// site, value and bound, and yields false so that the caller skips the
// access. A translation unit that uses it declares its record once with
// CSAQ_GUARD_RECORD(), which also registers a host-side reader of the record
// with the library (csaq_guard_report sums them). In the default build the
// guard is the constant true and the record is empty: no code is added.
#ifdef CSAQ_CHECKED
void register_guard_reader(int (*read)(unsigned long long* count, long long* first), int (*clear)());
#define CSAQ_GUARD_RECORD()                                                                             \
  static __device__ unsigned long long g_guard_count;                                                   \
  static __device__ long long g_guard_first[3];                                                         \
  static __device__ __forceinline__ bool guard_check(bool ok, int site, long long v, long long bound) {  \
    if (ok) return true;                                                                                \
    if (atomicAdd(&g_guard_count, 1ull) == 0ull) {                                                      \
      g_guard_first[0] = site;                                                                          \
      g_guard_first[1] = v;                                                                             \
      g_guard_first[2] = bound;                                                                         \
    }                                                                                                   \
    return false;                                                                                       \
  }                                                                                                     \
  static int guard_read(unsigned long long* count, long long* first) {                                  \
    if (cudaMemcpyFromSymbol(count, g_guard_count, sizeof(*count)) != cudaSuccess ||                    \
        cudaMemcpyFromSymbol(first, g_guard_first, 3 * sizeof(long long)) != cudaSuccess)               \
      return launch_status();                                                                           \
    return CSAQ_OK;                                                                                     \
  }                                                                                                     \
  static int guard_clear() {                                                                            \
    const unsigned long long z = 0ull;                                                                  \
    const long long zf[3] = {0, 0, 0};                                                                  \
    if (cudaMemcpyToSymbol(g_guard_count, &z, sizeof(z)) != cudaSuccess ||                              \
        cudaMemcpyToSymbol(g_guard_first, zf, sizeof(zf)) != cudaSuccess)                               \
      return launch_status();                                                                           \
    return CSAQ_OK;                                                                                     \
  }                                                                                                     \
  static const bool g_guard_registered = (register_guard_reader(guard_read, guard_clear), true);
#define CSAQ_GUARD(ok, site, v, bound) guard_check((ok), (site), (long long)(v), (long long)(bound))
#else
#define CSAQ_GUARD_RECORD()
#define CSAQ_GUARD(ok, site, v, bound) true
#endif

inline int dtype_size(int dt) {
  switch (dt) {
    case CSAQ_DT_F32: return 4;
    case CSAQ_DT_F16: return 2;
    case CSAQ_DT_BF16: return 2;
    default: return 0;
  }
}

inline int64_t packed_row_bytes(int64_t cols, int bits) {
  switch (bits) {
    case 8: return cols;
    case 4: return (cols + 1) / 2;
    case 2: return (cols + 3) / 4;
    case 16: return cols * 2;
    default: return -1;
  }
}

// Exact widening of one element to fp32.
__device__ __forceinline__ float load_as_f32(const void* p, int dt, int64_t i) {
  if (dt == CSAQ_DT_F32) return reinterpret_cast<const float*>(p)[i];
  if (dt == CSAQ_DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}

// Bit pattern of a value (the intrinsics, not pointer casts, which the
// compiler may not honour for the 16-bit classes).
template <typename T> __device__ __forceinline__ uint32_t bits_of(T v);
template <> __device__ __forceinline__ uint32_t bits_of<float>(float v) { return __float_as_uint(v); }
template <> __device__ __forceinline__ uint32_t bits_of<__half>(__half v) { return __half_as_ushort(v); }
template <> __device__ __forceinline__ uint32_t bits_of<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat16_as_ushort(v);
}

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}

// ── torch CPU arithmetic, one IEEE rounding per op ─────────────────────────
// torch.clamp propagates NaN (fminf/fmaxf would drop it).
__device__ __forceinline__ float clamp_nan(float v, float lo, float hi) {
  if (v != v) return v;
  return fminf(fmaxf(v, lo), hi);
}

// .to(torch.int32) on x86: truncation; NaN and out-of-range give INT32_MIN.
__device__ __forceinline__ int32_t to_i32_x86(float v) {
  if (!(v >= -2147483648.0f && v < 2147483648.0f)) return INT32_MIN;
  return __float2int_rz(v);
}

// _compute_scale_zp for one (min, max) pair (csaq/kernels.py:495-508).
__device__ __forceinline__ void scale_zp(float w_min, float w_max, int bits, float& scale,
                                         int32_t& zp) {
  const float n_levels = (float)((1 << bits) - 1);
  if (!(w_max > w_min)) w_max = __fadd_rn(w_min, 1e-8f);
  scale = __fdiv_rn(__fsub_rn(w_max, w_min), n_levels);
  const float z = rintf(__fdiv_rn(-w_min, scale));
  zp = to_i32_x86(clamp_nan(z, 0.0f, n_levels));
}

// _quantize_rows for one element (csaq/kernels.py:511-523).
__device__ __forceinline__ int32_t quant_one(float w, float scale, int32_t zp, int bits) {
  const float n_levels = (float)((1 << bits) - 1);
  const float v = rintf(__fadd_rn(__fdiv_rn(w, scale), (float)zp));
  return to_i32_x86(clamp_nan(v, 0.0f, n_levels));
}

// (q - zp) * scale in fp32 (csaq/kernels.py:611, 619, 465).
__device__ __forceinline__ float dequant_one(int32_t q, int32_t zp, float scale) {
  return __fmul_rn(__fsub_rn((float)q, (float)zp), scale);
}

}  // namespace csaq
