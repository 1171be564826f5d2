// Bit-exact quantisation primitives: scale/zero point, quantise + pack,
// unpack, dequantise, requantise, fp16 cast.
//
// Every float operation mirrors the torch CPU arithmetic of csaq-quant with
// one IEEE rounding per op (explicit __f*_rn intrinsics, -fmad=false for this
// file), so codes, scales, zero points and dequantised values match the
// reference bit for bit.

#include "common.cuh"

namespace csaq {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t code_mask(int bits) { return (1u << bits) - 1u; }

// ── per-(row, group) scale / zero point, one warp per group ────────────────
// Per-channel: group = [0, cols), no padding. Per-group: group g covers
// [g*gs, (g+1)*gs); columns past `cols` are the zero padding of
// csaq/kernels.py:132-137 and take part in min/max.
__global__ void group_scales_kernel(const void* __restrict__ W, int dt, int64_t rows, int64_t cols,
                                    int64_t ld_w, int bits, int64_t gs, int64_t n_groups,
                                    float* __restrict__ scales, int32_t* __restrict__ zps) {
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows * n_groups) return;
  const int64_t r = warp / n_groups, g = warp % n_groups;
  const int64_t c0 = g * gs;
  const int64_t c1 = c0 + gs;  // exclusive; may exceed cols (padding)
  float mn = INFINITY, mx = -INFINITY;
  for (int64_t c = c0 + lane; c < c1; c += 32) {
    const float v = (c < cols) ? load_as_f32(W, dt, r * ld_w + c) : 0.0f;
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) {
    float s;
    int32_t z;
    scale_zp(mn, mx, bits, s, z);
    scales[warp] = s;
    zps[warp] = z;
  }
}

__global__ void row_absmax_kernel(const void* __restrict__ W, int dt, int64_t rows, int64_t cols,
                                  int64_t ld_w, float* __restrict__ out) {
  const int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  float m = 0.0f;
  for (int64_t c = lane; c < cols; c += 32) m = fmaxf(m, fabsf(load_as_f32(W, dt, r * ld_w + c)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) out[r] = m;
}

// ── quantise + pack, one thread per output byte ────────────────────────────
__global__ void quant_pack_rows_kernel(const void* __restrict__ W, int dt, int64_t rows, int64_t cols,
                                       int64_t ld_w, int bits, int64_t gs,
                                       const float* __restrict__ scales,
                                       const int32_t* __restrict__ zps, int64_t ld_s, int scale_mode,
                                       const int32_t* __restrict__ src_row, int requant,
                                       uint8_t* __restrict__ out, int64_t row_bytes) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * row_bytes) return;
  const int64_t r = idx / row_bytes, j = idx % row_bytes;
  const int per_byte = 8 / bits;
  const int64_t srow = scale_mode == 0 ? r : (scale_mode == 1 ? 0 : (int64_t)src_row[r]);
  uint32_t byte = 0;
  for (int t = 0; t < per_byte; ++t) {
    const int64_t c = j * per_byte + t;
    if (c >= cols) break;  // the zero padding of _pack
    const int64_t g = (gs > 0) ? c / gs : 0;
    const float s = scales[srow * ld_s + g];
    const int32_t z = zps[srow * ld_s + g];
    int32_t q = quant_one(load_as_f32(W, dt, r * ld_w + c), s, z, bits);
    if (requant) q = quant_one(dequant_one(q, z, s), s, z, bits);
    byte |= ((uint32_t)q & code_mask(bits)) << (t * bits);
  }
  out[idx] = (uint8_t)byte;
}

// ── fused per-group quantise + pack: 128-bit loads, shuffle min/max ────────
// Each thread owns V = 16 / sizeof(T) consecutive columns; TPG = gs / V lanes
// form a group. Requires cols % V == 0 and 16-byte aligned rows.
template <typename T, int BITS>
__global__ void quant_pack_fused_kernel(const T* __restrict__ W, int64_t rows, int64_t cols,
                                        int64_t ld_w, int tpg, int64_t n_groups,
                                        uint8_t* __restrict__ out, int64_t row_bytes,
                                        float* __restrict__ scales, int32_t* __restrict__ zps) {
  constexpr int V = 16 / sizeof(T);
  constexpr int OUT_BYTES = V * BITS / 8;
  const int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t tpr = n_groups * tpg;  // threads per row
  const int64_t r = t / tpr;
  const int64_t tr = t % tpr;
  const int64_t c0 = tr * V;
  const bool live = r < rows;
  const bool in_cols = live && c0 < cols;
  float v[V];
  if (in_cols) {
    const uint4 raw = __ldg(reinterpret_cast<const uint4*>(W + r * ld_w + c0));
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = to_f32<T>(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = 0.0f;  // padding zeros join min/max
  }
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < V; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
  for (int o = 1; o < tpg; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  float s;
  int32_t z;
  scale_zp(mn, mx, BITS, s, z);
  if (live && (tr % tpg) == 0) {
    const int64_t gi = r * n_groups + tr / tpg;
    scales[gi] = s;
    zps[gi] = z;
  }
  if (!in_cols) return;
  // pack V codes into OUT_BYTES bytes
  uint64_t word = 0;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const uint32_t q = (uint32_t)quant_one(v[i], s, z, BITS) & ((1u << BITS) - 1u);
    word |= (uint64_t)q << (i * BITS);
  }
  uint8_t* dst = out + r * row_bytes + c0 * BITS / 8;
  if constexpr (OUT_BYTES == 8) {
    *reinterpret_cast<uint64_t*>(dst) = word;
  } else if constexpr (OUT_BYTES == 4) {
    *reinterpret_cast<uint32_t*>(dst) = (uint32_t)word;
  } else if constexpr (OUT_BYTES == 2) {
    *reinterpret_cast<uint16_t*>(dst) = (uint16_t)word;
  } else {
    *dst = (uint8_t)word;
  }
}

template <typename T>
int launch_fused(const void* W, int64_t rows, int64_t cols, int64_t ld_w, int bits, int64_t gs,
                 uint8_t* q, float* s, int32_t* z, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const int tpg = (int)(gs / V);
  const int64_t n_groups = (cols + gs - 1) / gs;
  const int64_t row_bytes = packed_row_bytes(cols, bits);
  const int64_t threads = rows * n_groups * tpg;
  const int64_t blocks = (threads + kThreads - 1) / kThreads;
  const T* w = reinterpret_cast<const T*>(W);
  switch (bits) {
    case 2: quant_pack_fused_kernel<T, 2><<<blocks, kThreads, 0, st>>>(w, rows, cols, ld_w, tpg, n_groups, q, row_bytes, s, z); break;
    case 4: quant_pack_fused_kernel<T, 4><<<blocks, kThreads, 0, st>>>(w, rows, cols, ld_w, tpg, n_groups, q, row_bytes, s, z); break;
    case 8: quant_pack_fused_kernel<T, 8><<<blocks, kThreads, 0, st>>>(w, rows, cols, ld_w, tpg, n_groups, q, row_bytes, s, z); break;
    default: return CSAQ_ERR_BITS;
  }
  return launch_status();
}

__global__ void cast_f16_kernel(const void* __restrict__ W, int dt, int64_t rows, int64_t cols,
                                int64_t ld_w, __half* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, c = i % cols;
  out[i] = __float2half_rn(load_as_f32(W, dt, r * ld_w + c));
}

__global__ void pack_kernel(const int32_t* __restrict__ q, int bits, int64_t rows, int64_t cols,
                            uint8_t* __restrict__ out, int64_t row_bytes) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * row_bytes) return;
  const int64_t r = idx / row_bytes, j = idx % row_bytes;
  const int per_byte = 8 / bits;
  uint32_t byte = 0;
  for (int t = 0; t < per_byte; ++t) {
    const int64_t c = j * per_byte + t;
    if (c >= cols) break;
    byte |= (((uint32_t)q[r * cols + c]) & 0xFFu & code_mask(bits)) << (t * bits);
  }
  out[idx] = (uint8_t)byte;
}

__device__ __forceinline__ int32_t code_at(const uint8_t* __restrict__ row, int64_t c, int bits) {
  if (bits == 8) return row[c];
  if (bits == 4) return (row[c >> 1] >> ((c & 1) * 4)) & 0xF;
  return (row[c >> 2] >> ((c & 3) * 2)) & 0x3;
}

__global__ void unpack_kernel(const uint8_t* __restrict__ p, int bits, int64_t rows, int64_t cols,
                              int64_t row_bytes, int32_t* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, c = i % cols;
  out[i] = code_at(p + r * row_bytes, c, bits);
}

__global__ void float_to_int_kernel(const float* __restrict__ W, const float* __restrict__ s,
                                    const int32_t* __restrict__ z, int bits, int64_t rows,
                                    int64_t cols, int32_t* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols;
  out[i] = quant_one(W[i], s[r], z[r], bits);
}

template <typename T>
__global__ void dequant_kernel(const uint8_t* __restrict__ p, const float* __restrict__ s,
                               const int32_t* __restrict__ z, int bits, int64_t rows, int64_t cols,
                               int64_t gs, int64_t n_groups, int64_t row_bytes, int nan_to_num,
                               T* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int64_t r = i / cols, c = i % cols;
  float w;
  if (bits == 16) {
    w = __half2float(reinterpret_cast<const __half*>(p + r * row_bytes)[c]);
  } else {
    const int64_t g = gs > 0 ? c / gs : 0;
    w = dequant_one(code_at(p + r * row_bytes, c, bits), z[r * n_groups + g], s[r * n_groups + g]);
    if (nan_to_num) {
      if (w != w) w = 0.0f;
      else if (w == INFINITY) w = 65504.0f;
      else if (w == -INFINITY) w = -65504.0f;
    }
  }
  out[i] = from_f32<T>(w);
}

// The same dequantisation, eight consecutive columns of a row per thread:
// one 2/4/8/16-byte code load, one scale and zero point, and 16- or 32-byte
// stores, with 32-bit index arithmetic. Needs cols % 8 == 0, a group size that
// is a multiple of 8 (or per-channel), and aligned buffers (csaq_dequant
// checks). Column c + k of an octet is nibble k of the 4-bit word, bit pair k
// of the 2-bit one, byte k of the 8-bit one and half k of the 16-bit one.
template <typename T, int BITS>
__global__ void dequant8_kernel(const uint8_t* __restrict__ p, const float* __restrict__ s,
                                const int32_t* __restrict__ z, int rows, int octs, int gs_oct, int n_groups,
                                int64_t row_bytes, int nan_to_num, T* __restrict__ out) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= int64_t(rows) * octs) return;
  const int r = (int)(i / octs), o = (int)(i - int64_t(r) * octs);
  const uint8_t* rp = p + int64_t(r) * row_bytes;
  float w[8];
  if constexpr (BITS == 16) {
    const uint4 v = reinterpret_cast<const uint4*>(rp)[o];
    const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = __half2float(h[k]);
  } else {
    const int g = gs_oct ? o / gs_oct : 0;
    const float sc = s[int64_t(r) * n_groups + g];
    const int32_t zp = z[int64_t(r) * n_groups + g];
    int32_t q[8];
    if constexpr (BITS == 8) {
      const uint2 v = reinterpret_cast<const uint2*>(rp)[o];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        q[k] = (v.x >> (8 * k)) & 0xFF;
        q[k + 4] = (v.y >> (8 * k)) & 0xFF;
      }
    } else if constexpr (BITS == 4) {
      const uint32_t v = reinterpret_cast<const uint32_t*>(rp)[o];
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = (v >> (4 * k)) & 0xF;
    } else {
      const uint32_t v = reinterpret_cast<const uint16_t*>(rp)[o];
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = (v >> (2 * k)) & 0x3;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float x = dequant_one(q[k], zp, sc);
      if (nan_to_num) {
        if (x != x) x = 0.0f;
        else if (x == INFINITY) x = 65504.0f;
        else if (x == -INFINITY) x = -65504.0f;
      }
      w[k] = x;
    }
  }
  T* dst = out + int64_t(r) * octs * 8 + int64_t(o) * 8;
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(w[0], w[1], w[2], w[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(w[4], w[5], w[6], w[7]);
  } else {
    uint4 v;
    T* e = reinterpret_cast<T*>(&v);
#pragma unroll
    for (int k = 0; k < 8; ++k) e[k] = from_f32<T>(w[k]);
    *reinterpret_cast<uint4*>(dst) = v;
  }
}

inline int64_t blocks_for(int64_t n) { return (n + kThreads - 1) / kThreads; }

inline bool is_per_channel(int64_t gs, int64_t cols) { return gs <= 0 || gs >= cols; }

template <typename T>
int launch_dequant8_t(const uint8_t* q, const float* s, const int32_t* z, int bits, int rows, int octs, int gs_oct,
                      int n_groups, int64_t rb, int nan, T* out, cudaStream_t st) {
  const int64_t blocks = blocks_for(int64_t(rows) * octs);
  switch (bits) {
    case 16: dequant8_kernel<T, 16><<<blocks, kThreads, 0, st>>>(q, s, z, rows, octs, gs_oct, n_groups, rb, nan, out); break;
    case 8: dequant8_kernel<T, 8><<<blocks, kThreads, 0, st>>>(q, s, z, rows, octs, gs_oct, n_groups, rb, nan, out); break;
    case 4: dequant8_kernel<T, 4><<<blocks, kThreads, 0, st>>>(q, s, z, rows, octs, gs_oct, n_groups, rb, nan, out); break;
    default: dequant8_kernel<T, 2><<<blocks, kThreads, 0, st>>>(q, s, z, rows, octs, gs_oct, n_groups, rb, nan, out); break;
  }
  return launch_status();
}

int launch_dequant8(const uint8_t* q, const float* s, const int32_t* z, int bits, int rows, int octs, int gs_oct,
                    int n_groups, int64_t rb, int nan, int out_dtype, void* out, cudaStream_t st) {
  if (out_dtype == CSAQ_DT_F32)
    return launch_dequant8_t(q, s, z, bits, rows, octs, gs_oct, n_groups, rb, nan, reinterpret_cast<float*>(out), st);
  if (out_dtype == CSAQ_DT_F16)
    return launch_dequant8_t(q, s, z, bits, rows, octs, gs_oct, n_groups, rb, nan, reinterpret_cast<__half*>(out), st);
  return launch_dequant8_t(q, s, z, bits, rows, octs, gs_oct, n_groups, rb, nan,
                           reinterpret_cast<__nv_bfloat16*>(out), st);
}

}  // namespace
}  // namespace csaq

using namespace csaq;

extern "C" int64_t csaq_packed_row_bytes(int64_t cols, int bits) {
  if (cols < 0) return -1;
  return packed_row_bytes(cols, bits);
}

extern "C" int csaq_group_scales(const void* W, int w_dtype, int64_t rows, int64_t cols,
                                 int64_t ld_w, int bits, int64_t group_size, float* scales,
                                 int32_t* zero_points, float* row_absmax, void* stream) {
  if (!W || !scales || !zero_points || rows < 0 || cols <= 0 || ld_w < cols) return CSAQ_ERR_ARG;
  if (!dtype_size(w_dtype)) return CSAQ_ERR_ARG;
  if (bits != 2 && bits != 4 && bits != 8) return CSAQ_ERR_BITS;
  if (rows == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  const bool pc = is_per_channel(group_size, cols);
  const int64_t gs = pc ? cols : group_size;
  const int64_t n_groups = pc ? 1 : (cols + gs - 1) / gs;
  const int64_t threads = rows * n_groups * 32;
  group_scales_kernel<<<blocks_for(threads), kThreads, 0, st>>>(W, w_dtype, rows, cols, ld_w, bits,
                                                                 gs, n_groups, scales, zero_points);
  int rc = launch_status();
  if (rc || !row_absmax) return rc;
  row_absmax_kernel<<<blocks_for(rows * 32), kThreads, 0, st>>>(W, w_dtype, rows, cols, ld_w,
                                                                row_absmax);
  return launch_status();
}

extern "C" int csaq_quant_pack_rows(const void* W, int w_dtype, int64_t rows, int64_t cols,
                                    int64_t ld_w, int bits, int64_t group_size,
                                    const float* scales, const int32_t* zero_points, int64_t ld_s,
                                    int scale_mode, const int32_t* src_row, int requant,
                                    uint8_t* qdata, void* stream) {
  if (!W || !scales || !zero_points || !qdata || rows < 0 || cols <= 0 || ld_w < cols) return CSAQ_ERR_ARG;
  if (!dtype_size(w_dtype) || scale_mode < 0 || scale_mode > 2 || (scale_mode == 2 && !src_row))
    return CSAQ_ERR_ARG;
  if (bits != 2 && bits != 4 && bits != 8) return CSAQ_ERR_BITS;
  if (rows == 0) return CSAQ_OK;
  const int64_t gs = is_per_channel(group_size, cols) ? 0 : group_size;
  const int64_t n_groups = gs ? (cols + gs - 1) / gs : 1;
  if (ld_s < n_groups) return CSAQ_ERR_ARG;
  const int64_t rb = packed_row_bytes(cols, bits);
  quant_pack_rows_kernel<<<blocks_for(rows * rb), kThreads, 0, as_stream(stream)>>>(
      W, w_dtype, rows, cols, ld_w, bits, gs, scales, zero_points, ld_s, scale_mode, src_row,
      requant, qdata, rb);
  return launch_status();
}

extern "C" int csaq_quant_pack(const void* W, int w_dtype, int64_t rows, int64_t cols, int64_t ld_w,
                               int bits, int64_t group_size, uint8_t* qdata, float* scales,
                               int32_t* zero_points, void* stream) {
  if (!W || !qdata || !scales || !zero_points || rows < 0 || cols <= 0 || ld_w < cols) return CSAQ_ERR_ARG;
  const int es = dtype_size(w_dtype);
  if (!es) return CSAQ_ERR_ARG;
  if (bits != 2 && bits != 4 && bits != 8) return CSAQ_ERR_BITS;
  if (rows == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  if (!is_per_channel(group_size, cols)) {
    const int V = 16 / es;
    const int64_t tpg = group_size / V;
    const int out_bytes = V * bits / 8;
    const bool pow2 = tpg > 0 && tpg <= 32 && (tpg & (tpg - 1)) == 0;
    const bool aligned = (reinterpret_cast<uintptr_t>(W) % 16 == 0) && ((ld_w * es) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(qdata) % out_bytes == 0);
    if (group_size % V == 0 && pow2 && cols % V == 0 && aligned) {
      switch (w_dtype) {
        case CSAQ_DT_F32: return launch_fused<float>(W, rows, cols, ld_w, bits, group_size, qdata, scales, zero_points, st);
        case CSAQ_DT_F16: return launch_fused<__half>(W, rows, cols, ld_w, bits, group_size, qdata, scales, zero_points, st);
        default: return launch_fused<__nv_bfloat16>(W, rows, cols, ld_w, bits, group_size, qdata, scales, zero_points, st);
      }
    }
  }
  int rc = csaq_group_scales(W, w_dtype, rows, cols, ld_w, bits, group_size, scales, zero_points,
                             nullptr, stream);
  if (rc) return rc;
  const int64_t n_groups = is_per_channel(group_size, cols) ? 1 : (cols + group_size - 1) / group_size;
  return csaq_quant_pack_rows(W, w_dtype, rows, cols, ld_w, bits, group_size, scales, zero_points,
                              n_groups, 0, nullptr, 0, qdata, stream);
}

extern "C" int csaq_cast_f16(const void* W, int w_dtype, int64_t rows, int64_t cols, int64_t ld_w,
                             uint16_t* out, void* stream) {
  if (!W || !out || rows < 0 || cols < 0 || ld_w < cols || !dtype_size(w_dtype)) return CSAQ_ERR_ARG;
  if (rows * cols == 0) return CSAQ_OK;
  cast_f16_kernel<<<blocks_for(rows * cols), kThreads, 0, as_stream(stream)>>>(
      W, w_dtype, rows, cols, ld_w, reinterpret_cast<__half*>(out));
  return launch_status();
}

extern "C" int csaq_pack(const int32_t* q, int bits, int64_t rows, int64_t cols, uint8_t* out,
                         void* stream) {
  if (!q || !out || rows < 0 || cols < 0) return CSAQ_ERR_ARG;
  if (bits != 2 && bits != 4 && bits != 8) return CSAQ_ERR_BITS;
  const int64_t rb = packed_row_bytes(cols, bits);
  if (rows * rb == 0) return CSAQ_OK;
  pack_kernel<<<blocks_for(rows * rb), kThreads, 0, as_stream(stream)>>>(q, bits, rows, cols, out, rb);
  return launch_status();
}

extern "C" int csaq_unpack(const uint8_t* packed, int bits, int64_t rows, int64_t cols,
                           int32_t* out, void* stream) {
  if (!packed || !out || rows < 0 || cols < 0) return CSAQ_ERR_ARG;
  if (bits != 2 && bits != 4 && bits != 8) return CSAQ_ERR_BITS;
  if (rows * cols == 0) return CSAQ_OK;
  unpack_kernel<<<blocks_for(rows * cols), kThreads, 0, as_stream(stream)>>>(
      packed, bits, rows, cols, packed_row_bytes(cols, bits), out);
  return launch_status();
}

extern "C" int csaq_float_to_int(const float* W, const float* scales, const int32_t* zero_points,
                                 int bits, int64_t rows, int64_t cols, int32_t* out, void* stream) {
  if (!W || !scales || !zero_points || !out || rows < 0 || cols < 0) return CSAQ_ERR_ARG;
  if (bits < 1 || bits > 8) return CSAQ_ERR_BITS;
  if (rows * cols == 0) return CSAQ_OK;
  float_to_int_kernel<<<blocks_for(rows * cols), kThreads, 0, as_stream(stream)>>>(
      W, scales, zero_points, bits, rows, cols, out);
  return launch_status();
}

extern "C" int csaq_dequant(const uint8_t* qdata, const float* scales, const int32_t* zero_points,
                            int bits, int64_t rows, int64_t cols, int64_t group_size, int nan_to_num,
                            int out_dtype, void* out, void* stream) {
  if (!qdata || !out || rows < 0 || cols < 0 || !dtype_size(out_dtype)) return CSAQ_ERR_ARG;
  if (bits != 2 && bits != 4 && bits != 8 && bits != 16) return CSAQ_ERR_BITS;
  if (bits != 16 && (!scales || !zero_points)) return CSAQ_ERR_ARG;
  if (rows * cols == 0) return CSAQ_OK;
  const int64_t gs = is_per_channel(group_size, cols) ? 0 : group_size;
  const int64_t n_groups = gs ? (cols + gs - 1) / gs : 1;
  const int64_t rb = packed_row_bytes(cols, bits);
  const int64_t n = rows * cols;
  cudaStream_t st = as_stream(stream);
  const int align = bits == 16 ? 16 : bits;  // bytes of one octet's codes
  if (cols % 8 == 0 && (gs == 0 || gs % 8 == 0) && rows <= INT32_MAX && cols / 8 <= INT32_MAX &&
      n_groups <= INT32_MAX && reinterpret_cast<uintptr_t>(qdata) % align == 0 &&
      reinterpret_cast<uintptr_t>(out) % 16 == 0)
    return launch_dequant8(qdata, scales, zero_points, bits, (int)rows, (int)(cols / 8), (int)(gs / 8),
                           (int)n_groups, rb, nan_to_num, out_dtype, out, st);
  switch (out_dtype) {
    case CSAQ_DT_F32:
      dequant_kernel<float><<<blocks_for(n), kThreads, 0, st>>>(qdata, scales, zero_points, bits, rows, cols, gs, n_groups, rb, nan_to_num, reinterpret_cast<float*>(out));
      break;
    case CSAQ_DT_F16:
      dequant_kernel<__half><<<blocks_for(n), kThreads, 0, st>>>(qdata, scales, zero_points, bits, rows, cols, gs, n_groups, rb, nan_to_num, reinterpret_cast<__half*>(out));
      break;
    default:
      dequant_kernel<__nv_bfloat16><<<blocks_for(n), kThreads, 0, st>>>(qdata, scales, zero_points, bits, rows, cols, gs, n_groups, rb, nan_to_num, reinterpret_cast<__nv_bfloat16*>(out));
      break;
  }
  return launch_status();
}
