// On-device sampling for decode and self-speculative decoding at temperature > 0
// (csaq/inference.py:269-304 `_sample`, :482-518 the rejection-sampling accept).
//
// csaq_sample_rows draws one token per logit row: logits are clamped to
// [-50, 50] (NaN -> 0), divided by the temperature; with top_p < 1 the
// smallest set of largest logits whose preceding mass does not exceed top_p is
// kept (the reference sorts; here a bisection on the logit value finds the
// same set: token j stays iff the mass of the tokens strictly above it is at
// most top_p); then one token is drawn from the kept softmax mass by inverse
// CDF in index order.
//
// csaq_spec_sample_verify turns the verify logits into the `vt` row that
// csaq_spec_accept consumes: for draft position k it accepts the draft token d
// with probability min(1, p_v(d) / p_d(d)) (softmax of logits / T, no clamp and
// no top-p, as the reference), else draws from max(p_v - p_d, 0) and stops;
// when every draft token is accepted it samples the token after them from the
// verify logits. The reference compares draft position k with verify row k+1
// (csaq/inference.py:486); here row k, the verifier's prediction at that
// position. A resampled token never equals the rejected draft token (its
// residual is 0), so csaq_spec_accept's longest-prefix rule reproduces the
// decision.
//
// Random numbers: Philox (curand) with subsequence = row or sequence, and an
// offset of 256 draws per call from a device call counter that the last CTA of
// each launch advances (a call draws at most 2K + 1 <= 129 per sequence), so
// the calls can be captured in a CUDA graph and replayed.

#include <curand_kernel.h>

#include "common.cuh"

namespace csaq {
namespace {

constexpr int kSThreads = 1024;

// a logit row stored as n_parts slices of part_len values (tensor-parallel vocabulary slices)
template <typename T>
struct PartRows {
  const T* base;
  int n_parts;
  int64_t part_stride, ld, part_len;
  __device__ __forceinline__ float at(int64_t m, int64_t j) const {
    if (n_parts == 1) return to_f32<T>(base[m * ld + j]);
    const int64_t r = j / part_len, i = j - r * part_len;
    return to_f32<T>(base[r * part_stride + m * ld + i]);
  }
  __device__ __forceinline__ int64_t V() const { return (int64_t)n_parts * part_len; }
};

__device__ __forceinline__ float block_reduce(float v, bool is_max, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? fmaxf(v, w) : v + w;
  }
  __syncthreads();  // red is reused by consecutive reductions
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (int)(blockDim.x >> 5) ? red[lane] : (is_max ? -INFINITY : 0.0f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? fmaxf(v, w) : v + w;
    }
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ float clean(float x) {
  if (x != x) return 0.0f;
  return fminf(fmaxf(x, -50.0f), 50.0f);  // +-inf clamp too
}

// Inverse CDF over the index order: the first index j whose cumulative weight
// w(j) exceeds u (u in [0, total)); every thread scans a contiguous segment.
template <typename W>
__device__ int64_t inverse_cdf(int64_t V, float u, W weight, float* red, int64_t* pick) {
  const int64_t seg = (V + blockDim.x - 1) / blockDim.x;
  const int64_t a = threadIdx.x * seg, b = a + seg < V ? a + seg : V;
  float s = 0.0f;
  for (int64_t j = a; j < b; ++j) s += weight(j);
  // block exclusive scan of the segment sums
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  if (threadIdx.x == 0) *pick = -1;
  __syncthreads();
  if (warp == 0) {
    float w = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += t;
    }
    red[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  const float before = (warp > 0 ? red[warp - 1] : 0.0f) + incl - s;
  if (s > 0.0f && u >= before && u < before + s) {
    float c = before;
    int64_t j = a, last = -1;
    for (; j < b; ++j) {
      const float w = weight(j);
      if (w > 0.0f) last = j;
      c += w;
      if (u < c && w > 0.0f) break;
    }
    *pick = j < b ? j : last;
  }
  __syncthreads();
  int64_t r = *pick;
  if (r < 0) {  // u at the very top (rounding): the last index with weight
    __syncthreads();
    if (threadIdx.x == 0) {
      int64_t last = 0;
      for (int64_t j = V - 1; j >= 0; --j)
        if (weight(j) > 0.0f) {
          last = j;
          break;
        }
      *pick = last;
    }
    __syncthreads();
    r = *pick;
  }
  return r;
}

// One token from row m: clamp, / temperature, top-p, softmax, inverse CDF.
template <typename T>
__device__ int64_t sample_one(const PartRows<T>& R, int64_t m, float inv_t, float top_p, float u01, float* red,
                              int64_t* pick) {
  const int64_t V = R.V();
  float mx = -INFINITY;
  for (int64_t j = threadIdx.x; j < V; j += blockDim.x) mx = fmaxf(mx, clean(R.at(m, j)) * inv_t);
  const float zmax = block_reduce(mx, true, red);
  float s = 0.0f;
  for (int64_t j = threadIdx.x; j < V; j += blockDim.x) s += __expf(clean(R.at(m, j)) * inv_t - zmax);
  const float Z = block_reduce(s, false, red);
  float lo = -INFINITY;  // keep z > lo
  if (top_p < 1.0f) {
    // M(v) = mass strictly above v, non-increasing in v; the kept tokens are
    // those with M(z) <= top_p, i.e. z > lo at the converged boundary
    float a = zmax - 120.0f, b = zmax;
    for (int it = 0; it < 48; ++it) {
      const float mid = 0.5f * (a + b);
      if (!(mid > a && mid < b)) break;
      float mm = 0.0f;
      for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
        const float z = clean(R.at(m, j)) * inv_t;
        if (z > mid) mm += __expf(z - zmax);
      }
      if (block_reduce(mm, false, red) / Z <= top_p)
        b = mid;
      else
        a = mid;
    }
    lo = a;
  }
  float kept = 0.0f;
  for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
    const float z = clean(R.at(m, j)) * inv_t;
    if (z > lo) kept += __expf(z - zmax);
  }
  const float S = block_reduce(kept, false, red);
  const float u = fminf(u01, 1.0f) * S;
  return inverse_cdf(V, u, [&](int64_t j) {
    const float z = clean(R.at(m, j)) * inv_t;
    return z > lo ? __expf(z - zmax) : 0.0f;
  }, red, pick);
}

__device__ __forceinline__ void advance_counter(uint64_t* ctr) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(reinterpret_cast<unsigned long long*>(ctr + 1), 1ull) == gridDim.x - 1ull) {
      ctr[1] = 0ull;
      ctr[0] += 1ull;
      __threadfence();
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kSThreads) sample_rows_kernel(PartRows<T> R, float inv_t, float top_p, uint64_t seed,
                                                                uint64_t* ctr, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ int64_t pick;
  __shared__ uint64_t call;
  if (threadIdx.x == 0) call = ctr[0];
  __syncthreads();
  const int64_t m = blockIdx.x;
  curandStatePhilox4_32_10_t st;
  curand_init(seed, (unsigned long long)m, call * 256ull, &st);
  const float u = curand_uniform(&st);
  const int64_t tok = sample_one(R, m, inv_t, top_p, u, red, &pick);
  if (threadIdx.x == 0) out[m] = tok;
  advance_counter(ctr);
}

// p(j) = exp(z_j - zmax) / Z of logits / T (no clamp) for one row
template <typename T>
struct Soft {
  float zmax, Z, inv_t;
};

template <typename ROW>
__device__ Soft<float> softmax_stats(ROW row, int64_t V, float inv_t, float* red) {
  float mx = -INFINITY;
  for (int64_t j = threadIdx.x; j < V; j += blockDim.x) mx = fmaxf(mx, row(j) * inv_t);
  const float zmax = block_reduce(mx, true, red);
  float s = 0.0f;
  for (int64_t j = threadIdx.x; j < V; j += blockDim.x) s += __expf(row(j) * inv_t - zmax);
  return Soft<float>{zmax, block_reduce(s, false, red), inv_t};
}

template <typename T>
__global__ void __launch_bounds__(kSThreads)
    spec_sample_kernel(const int64_t* __restrict__ draft, const T* __restrict__ dlog, PartRows<T> R, int K,
                       float inv_t, float top_p, uint64_t seed, uint64_t* ctr, int64_t* __restrict__ vt) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[32];
  __shared__ int64_t pick;
  __shared__ uint64_t call;
  if (threadIdx.x == 0) call = ctr[0];
  __syncthreads();
  const int64_t b = blockIdx.x, B = gridDim.x, V = R.V();
  curandStatePhilox4_32_10_t st;
  curand_init(seed, (unsigned long long)b, call * 256ull, &st);
  int k = 0;
  for (; k < K; ++k) {
    const int64_t vrow = b * (K + 1) + k;
    const T* drow = dlog + ((int64_t)k * B + b) * V;
    auto vz = [&](int64_t j) { return R.at(vrow, j); };
    auto dz = [&](int64_t j) { return to_f32<T>(drow[j]); };
    const Soft<float> sv = softmax_stats(vz, V, inv_t, red);
    const Soft<float> sd = softmax_stats(dz, V, inv_t, red);
    const int64_t d = draft[b * K + k];
    const float pv = __expf(vz(d) * inv_t - sv.zmax) / sv.Z;
    const float pd = __expf(dz(d) * inv_t - sd.zmax) / sd.Z;
    const float ratio = pv / fmaxf(pd, 1e-10f);
    const float u = curand_uniform(&st);
    if (u < fminf(1.0f, ratio)) {
      if (threadIdx.x == 0) vt[b * (K + 1) + k] = d;
      continue;
    }
    // residual max(p_v - p_d, 0)
    auto res = [&](int64_t j) {
      return fmaxf(__expf(vz(j) * inv_t - sv.zmax) / sv.Z - __expf(dz(j) * inv_t - sd.zmax) / sd.Z, 0.0f);
    };
    float s = 0.0f;
    for (int64_t j = threadIdx.x; j < V; j += blockDim.x) s += res(j);
    const float S = block_reduce(s, false, red);
    const float u2 = curand_uniform(&st);
    int64_t tok;
    if (S > 1e-8f) {
      tok = inverse_cdf(V, fminf(u2, 1.0f) * S, res, red, &pick);
    } else {  // no residual mass: the verifier's most likely token
      float best = -INFINITY;
      int64_t bi = 0;
      for (int64_t j = threadIdx.x; j < V; j += blockDim.x) {
        const float z = vz(j);
        if (z > best) { best = z; bi = j; }
      }
      const float bm = block_reduce(best, true, red);
      if (threadIdx.x == 0) pick = V;
      __syncthreads();
      if (best == bm) atomicMin(reinterpret_cast<unsigned long long*>(&pick), (unsigned long long)bi);
      __syncthreads();
      tok = pick;
    }
    if (threadIdx.x == 0) vt[b * (K + 1) + k] = tok;
    break;
  }
  if (k == K) {  // every draft token accepted: the verifier's next token
    const float u = curand_uniform(&st);
    const int64_t tok = sample_one(R, b * (K + 1) + K, inv_t, top_p, u, red, &pick);
    if (threadIdx.x == 0) vt[b * (K + 1) + K] = tok;
  }
  advance_counter(ctr);
}

}  // namespace
}  // namespace csaq

using namespace csaq;

extern "C" int csaq_sample_rows(const void* logits, int n_parts, int64_t part_stride, int64_t ld, int64_t part_len,
                                int64_t rows, float temperature, float top_p, uint64_t seed, uint64_t* counter,
                                int64_t* out, int dtype, void* stream) {
  if (!logits || !counter || !out || n_parts < 1 || part_len < 1 || rows < 0 || ld < part_len) return CSAQ_ERR_ARG;
  if (!(temperature > 0.0f) || !(top_p > 0.0f)) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16 && dtype != CSAQ_DT_F32) return CSAQ_ERR_ARG;
  if (rows == 0) return CSAQ_OK;
  if (rows > INT32_MAX) return CSAQ_ERR_UNSUPPORTED;
  const float inv_t = 1.0f / fmaxf(temperature, 1e-8f);
  cudaStream_t st = as_stream(stream);
  const dim3 grid((unsigned)rows);
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(sample_rows_kernel<__nv_bfloat16>, grid, dim3(kSThreads), 0, st,
                      PartRows<__nv_bfloat16>{(const __nv_bfloat16*)logits, n_parts, part_stride, ld, part_len},
                      inv_t, top_p, seed, counter, out);
  if (dtype == CSAQ_DT_F16)
    return launch_pdl(sample_rows_kernel<__half>, grid, dim3(kSThreads), 0, st,
                      PartRows<__half>{(const __half*)logits, n_parts, part_stride, ld, part_len}, inv_t, top_p, seed,
                      counter, out);
  return launch_pdl(sample_rows_kernel<float>, grid, dim3(kSThreads), 0, st,
                    PartRows<float>{(const float*)logits, n_parts, part_stride, ld, part_len}, inv_t, top_p, seed,
                    counter, out);
}

extern "C" int csaq_spec_sample_verify(const int64_t* draft, const void* draft_logits, const void* verify_logits,
                                       int n_parts, int64_t part_stride, int64_t ld, int64_t part_len, int64_t B,
                                       int64_t K, float temperature, float top_p, uint64_t seed, uint64_t* counter,
                                       int64_t* vt, int dtype, void* stream) {
  if (!draft || !draft_logits || !verify_logits || !counter || !vt || n_parts < 1 || part_len < 1 || B < 0 ||
      K < 1 || ld < part_len)
    return CSAQ_ERR_ARG;
  if (!(temperature > 0.0f) || !(top_p > 0.0f)) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16 && dtype != CSAQ_DT_F32) return CSAQ_ERR_ARG;
  if (B == 0) return CSAQ_OK;
  if (B > INT32_MAX || K > 64) return CSAQ_ERR_UNSUPPORTED;
  const float inv_t = 1.0f / fmaxf(temperature, 1e-8f);
  cudaStream_t st = as_stream(stream);
  const dim3 grid((unsigned)B);
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(spec_sample_kernel<__nv_bfloat16>, grid, dim3(kSThreads), 0, st, draft,
                      (const __nv_bfloat16*)draft_logits,
                      PartRows<__nv_bfloat16>{(const __nv_bfloat16*)verify_logits, n_parts, part_stride, ld, part_len},
                      (int)K, inv_t, top_p, seed, counter, vt);
  if (dtype == CSAQ_DT_F16)
    return launch_pdl(spec_sample_kernel<__half>, grid, dim3(kSThreads), 0, st, draft, (const __half*)draft_logits,
                      PartRows<__half>{(const __half*)verify_logits, n_parts, part_stride, ld, part_len}, (int)K,
                      inv_t, top_p, seed, counter, vt);
  return launch_pdl(spec_sample_kernel<float>, grid, dim3(kSThreads), 0, st, draft, (const float*)draft_logits,
                    PartRows<float>{(const float*)verify_logits, n_parts, part_stride, ld, part_len}, (int)K, inv_t,
                    top_p, seed, counter, vt);
}
