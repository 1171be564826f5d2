// RMSNorm of one row by one CTA (HF LlamaRMSNorm / Qwen2RMSNorm):
// y = w * T(x * rsqrt(mean(x^2) + eps)), fp32 arithmetic, T = bf16 or fp16.
// Shared by the RMSNorm kernel and the tensor-parallel combine that ends in
// the next RMSNorm, so both give the same bits.
#pragma once

#include "common.cuh"

namespace csaq {

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32<T>(from_f32<T>(v));
}

constexpr int kNormThreads = 256;
constexpr int kNormVec = 4;  // 16-byte vectors per thread kept in registers (H <= 8192)

// Sum over the CTA: a butterfly in each warp, then one over the warp sums.
template <typename T>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  return red[0];
}

// One row by the calling CTA (kNormThreads threads; red: 32 shared floats).
// Rows whose length is a multiple of 8 (16-byte aligned) take a vector path:
// every thread loads its x and w vectors up front (one memory round trip),
// keeps x in registers and writes 16-byte stores.
template <typename T>
__device__ __forceinline__ void rmsnorm_row(const T* __restrict__ xr, const T* __restrict__ w, T* __restrict__ yr,
                                            int H, float eps, float* red) {
  const bool vec = (H % 8 == 0) && H <= kNormThreads * 8 * kNormVec &&
                   (reinterpret_cast<uintptr_t>(xr) % 16 == 0) && (reinterpret_cast<uintptr_t>(yr) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(w) % 16 == 0);
  if (vec) {
    const int nv = H / 8;
    uint4 xv[kNormVec], wv[kNormVec];
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      if (i < nv) {
        xv[j] = reinterpret_cast<const uint4*>(xr)[i];
        wv[j] = reinterpret_cast<const uint4*>(w)[i];
      }
    }
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      if (i < nv) {
        const T* e = reinterpret_cast<const T*>(&xv[j]);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float v = to_f32<T>(e[t]);
          ss = fmaf(v, v, ss);
        }
      }
    }
    const float r = rsqrtf(block_sum<T>(ss, red) / (float)H + eps);
#pragma unroll
    for (int j = 0; j < kNormVec; ++j) {
      const int i = threadIdx.x + j * kNormThreads;
      if (i < nv) {
        const T* e = reinterpret_cast<const T*>(&xv[j]);
        const T* we = reinterpret_cast<const T*>(&wv[j]);
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int t = 0; t < 8; ++t) oe[t] = from_f32<T>(to_f32<T>(we[t]) * round_to<T>(to_f32<T>(e[t]) * r));
        reinterpret_cast<uint4*>(yr)[i] = o;
      }
    }
    return;
  }
  float ss = 0.0f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = to_f32<T>(xr[i]);
    ss = fmaf(v, v, ss);
  }
  const float r = rsqrtf(block_sum<T>(ss, red) / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float n = round_to<T>(to_f32<T>(xr[i]) * r);
    yr[i] = from_f32<T>(to_f32<T>(w[i]) * n);
  }
}

}  // namespace csaq
