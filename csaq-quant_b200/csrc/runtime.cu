// Decoder-runtime kernels around the quantised linears: RMSNorm, rotary
// embedding + KV-cache write, decode attention, SiLU-gate and the on-device
// greedy acceptance of a self-speculative block.
//
// Layouts (bf16 or fp16, "T" below): hidden states (M, H) row-major with
// M = B * S tokens (S tokens per sequence in this step, sequence-major);
// KV cache (B, Hkv, Lmax, D); per-sequence start positions pos0[B] (the
// position of the step's first token). Token (b, s) sits at position pos0[b]+s.

#include <mutex>

#include "common.cuh"

namespace csaq {
namespace {

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// ── RMSNorm (HF Llama/Qwen2): y = w * T(x * rsqrt(mean(x^2) + eps)) ─────────
template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, int64_t ldx, const T* __restrict__ w,
                               T* __restrict__ y, int64_t ldy, int H, float eps) {
  pdl_wait();
  pdl_trigger();
  const int64_t row = blockIdx.x;
  const T* xr = x + row * ldx;
  __shared__ float red[32];
  float ss = 0.0f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = to_f32<T>(xr[i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float n = round_to<T>(to_f32<T>(xr[i]) * r);
    y[row * ldy + i] = from_f32<T>(to_f32<T>(w[i]) * n);
  }
}

// ── rotary embedding of q and k + KV-cache write ────────────────────────────
// q (M, Hq*D), k/v (M, Hkv*D) may be row slices of one fused buffer (ld_*).
// cos/sin: (Lmax, D) fp32 holding the model-dtype-rounded values.
// rotate_half convention: out_i = x_i cos_i - x_{i+D/2} sin_i (i < D/2),
//                         out_i = x_i cos_i + x_{i-D/2} sin_i (i >= D/2).
template <typename T>
__global__ void rope_kv_kernel(const T* __restrict__ q, int64_t ldq, const T* __restrict__ k,
                               int64_t ldk, const T* __restrict__ v, int64_t ldv,
                               const int32_t* __restrict__ pos0, int S, int Hq, int Hkv, int D,
                               const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                               T* __restrict__ q_out, T* __restrict__ k_cache,
                               T* __restrict__ v_cache, int Lmax) {
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.x;  // token
  const int b = (int)(m / S), s = (int)(m % S);
  const int pos = pos0[b] + s;
  const float* cs = cos_t + (int64_t)pos * D;
  const float* sn = sin_t + (int64_t)pos * D;
  const int half = D / 2;
  for (int idx = threadIdx.x; idx < (Hq + Hkv) * D; idx += blockDim.x) {
    const int hh = idx / D, i = idx % D;
    const bool is_q = hh < Hq;
    const int h = is_q ? hh : hh - Hq;
    const T* src = is_q ? q + m * ldq + (int64_t)h * D : k + m * ldk + (int64_t)h * D;
    const float xi = to_f32<T>(src[i]);
    const float xo = to_f32<T>(src[i < half ? i + half : i - half]);
    const float r = i < half ? fmaf(xi, cs[i], -xo * sn[i]) : fmaf(xi, cs[i], xo * sn[i]);
    if (is_q) {
      q_out[(m * Hq + h) * D + i] = from_f32<T>(r);
    } else {
      const int64_t c = (((int64_t)b * Hkv + h) * Lmax + pos) * D + i;
      k_cache[c] = from_f32<T>(r);
      v_cache[c] = v[m * ldv + (int64_t)h * D + i];
    }
  }
}

// ── decode attention (GQA, causal over the new tokens) ──────────────────────
// Grid (B * Hkv, n_split). CTA (bh, sp) scores keys [sp*kChunk, (sp+1)*kChunk)
// for the R = S * G query rows of its KV head (G = Hq / Hkv), writes partial
// (max, sum, o[D]) per row, and the last CTA of (bh) to finish (atomic ticket,
// no waiting) merges the partials and writes the output. The ticket counter
// is reset by that CTA, so the workspace needs zeroing only once.
constexpr int kChunk = 64;
constexpr int kAttnWarps = 4;

template <typename T>
__global__ void __launch_bounds__(kAttnWarps * 32) attention_kernel(
    const T* __restrict__ q, const T* __restrict__ k_cache, const T* __restrict__ v_cache,
    const int32_t* __restrict__ pos0, int S, int Hq, int Hkv, int Lmax, float scale,
    float* __restrict__ part, int32_t* __restrict__ tickets, T* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = 128;
  const int bh = blockIdx.x, sp = blockIdx.y, n_split = gridDim.y;
  const int b = bh / Hkv, h = bh % Hkv;
  const int G = Hq / Hkv, R = S * G;
  const int len = pos0[b] + S;  // keys visible to the last new token
  const int k0 = sp * kChunk;
  __shared__ __align__(16) T ks[kChunk][D];
  __shared__ __align__(16) T vs[kChunk][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_keys = max(0, min(kChunk, len - k0));
  const T* kb = k_cache + (((int64_t)b * Hkv + h) * Lmax + k0) * D;
  const T* vb = v_cache + (((int64_t)b * Hkv + h) * Lmax + k0) * D;
  for (int e = threadIdx.x; e < n_keys * D / 8; e += blockDim.x) {
    reinterpret_cast<uint4*>(&ks[0][0])[e] = reinterpret_cast<const uint4*>(kb)[e];
    reinterpret_cast<uint4*>(&vs[0][0])[e] = reinterpret_cast<const uint4*>(vb)[e];
  }
  __syncthreads();
  // partial layout: [bh][sp][r][D + 2]
  float* pbase = part + ((int64_t)bh * n_split + sp) * R * (D + 2);
  for (int r = warp; r < R; r += kAttnWarps) {
    const int s = r / G, hq = h * G + r % G;
    const int qpos = pos0[b] + s;  // attends keys 0..qpos
    const T* qr = q + (((int64_t)b * S + s) * Hq + hq) * D;
    float qv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) qv[i] = to_f32<T>(qr[lane * 4 + i]) * scale;
    const int kmax = min(n_keys, qpos - k0 + 1);
    float m = -INFINITY, l = 0.0f, o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int j = 0; j < kmax; ++j) {
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) d = fmaf(qv[i], to_f32<T>(ks[j][lane * 4 + i]), d);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      const float mn = fmaxf(m, d);
      const float corr = __expf(m - mn), p = __expf(d - mn);
      l = l * corr + p;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = fmaf(o[i], corr, p * to_f32<T>(vs[j][lane * 4 + i]));
      m = mn;
    }
    float* pr = pbase + (int64_t)r * (D + 2);
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[lane * 4 + i] = o[i];
    if (lane == 0) { pr[D] = m; pr[D + 1] = l; }
  }
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) is_last = (atomicAdd(&tickets[bh], 1) == n_split - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  for (int r = warp; r < R; r += kAttnWarps) {
    const int s = r / G, hq = h * G + r % G;
    float M_ = -INFINITY;
    for (int p = 0; p < n_split; ++p)
      M_ = fmaxf(M_, __ldcg(part + (((int64_t)bh * n_split + p) * R + r) * (D + 2) + D));
    float L = 0.0f, o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int p = 0; p < n_split; ++p) {
      const float* pr = part + (((int64_t)bh * n_split + p) * R + r) * (D + 2);
      const float mp = __ldcg(pr + D);
      if (mp == -INFINITY) continue;
      const float w = __expf(mp - M_);
      L = fmaf(__ldcg(pr + D + 1), w, L);
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = fmaf(__ldcg(pr + lane * 4 + i), w, o[i]);
    }
    T* orow = out + (((int64_t)b * S + s) * Hq + hq) * D;
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) orow[lane * 4 + i] = from_f32<T>(o[i] * inv);
  }
  if (threadIdx.x == 0) tickets[bh] = 0;
}

// ── SiLU gate (HF LlamaMLP): h = T(silu(g)) * u, rounded to T ───────────────
template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, int64_t ldg, const T* __restrict__ u,
                                int64_t ldu, T* __restrict__ h, int64_t ldh, int64_t M, int N) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= M * N) return;
  const int64_t m = i / N, n = i % N;
  const float gv = to_f32<T>(g[m * ldg + n]);
  const float sv = round_to<T>(gv / (1.0f + __expf(-gv)));
  h[m * ldh + n] = from_f32<T>(sv * to_f32<T>(u[m * ldu + n]));
}

// ── greedy self-speculative acceptance ──────────────────────────────────────
// Per sequence b: draft[b][0..K-1], verify argmax vt[b][0..K] (vt[k] follows
// the context plus draft[0..k-1]). Accept the longest prefix with
// draft[k] == vt[k], then append vt[j] (the correction, or the bonus token
// when j == K). Appends into out_tokens[b][n_out[b] ...] (capacity cap),
// advances pos0[b] by j + 1 while the sequence still has tokens to produce,
// stores next_tok[b] = the token to feed next (the correction / bonus).
// stats[0] += accepted draft tokens, stats[1] += rejected, stats[2] += blocks.
__global__ void accept_kernel(const int64_t* __restrict__ draft, const int64_t* __restrict__ vt,
                              int B, int K, int32_t* __restrict__ pos0,
                              int64_t* __restrict__ out_tokens, int32_t* __restrict__ n_out, int cap,
                              int64_t* __restrict__ next_tok, int32_t* __restrict__ n_new_out,
                              int64_t* __restrict__ stats, int32_t* __restrict__ remaining) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int j = 0;
  while (j < K && draft[(int64_t)b * K + j] == vt[(int64_t)b * (K + 1) + j]) ++j;
  const int n_new_all = j + 1;
  const int room = remaining[b];
  const int n_new = n_new_all < room ? n_new_all : room;
  int o = n_out[b];
  for (int t = 0; t < n_new && o < cap; ++t, ++o) {
    out_tokens[(int64_t)b * cap + o] = (t < j) ? draft[(int64_t)b * K + t] : vt[(int64_t)b * (K + 1) + j];
  }
  n_out[b] = o;
  if (room > 0) pos0[b] += n_new_all;  // a finished sequence stays put (cache bounds)
  remaining[b] = room - n_new;
  next_tok[b] = vt[(int64_t)b * (K + 1) + j];
  n_new_out[b] = n_new;
  if (room > 0) {
    atomicAdd(reinterpret_cast<unsigned long long*>(&stats[0]), (unsigned long long)min(j, room));
    atomicAdd(reinterpret_cast<unsigned long long*>(&stats[1]), (unsigned long long)(K - min(j, room)));
    atomicAdd(reinterpret_cast<unsigned long long*>(&stats[2]), 1ull);
  }
}

// Plain greedy step bookkeeping: append tok[b], advance pos0[b] by 1 while the
// sequence still has tokens to produce.
__global__ void commit_kernel(const int64_t* __restrict__ tok, int B, int32_t* __restrict__ pos0,
                              int64_t* __restrict__ out_tokens, int32_t* __restrict__ n_out, int cap,
                              int64_t* __restrict__ next_tok, int32_t* __restrict__ remaining) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  if (remaining[b] <= 0) return;  // a finished sequence stays put (cache bounds)
  if (n_out[b] < cap) {
    out_tokens[(int64_t)b * cap + n_out[b]] = tok[b];
    n_out[b] += 1;
  }
  remaining[b] -= 1;
  pos0[b] += 1;
  next_tok[b] = tok[b];
}

inline int64_t blocks_for(int64_t n, int t = 256) { return (n + t - 1) / t; }

}  // namespace
}  // namespace csaq

using namespace csaq;

extern "C" int csaq_rmsnorm(const void* x, int64_t ldx, const void* w, void* y, int64_t ldy,
                            int64_t M, int64_t H, float eps, int dtype, void* stream) {
  if (!x || !w || !y || M < 0 || H <= 0 || ldx < H || ldy < H) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  if (M == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(rmsnorm_kernel<__nv_bfloat16>, dim3(M), dim3(256), 0, st, (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, ldy, (int)H, eps);
  else
    return launch_pdl(rmsnorm_kernel<__half>, dim3(M), dim3(256), 0, st, (const __half*)x, ldx, (const __half*)w, (__half*)y, ldy, (int)H, eps);
}

extern "C" int csaq_rope_kv(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                            int64_t ldv, const int32_t* pos0, int64_t B, int64_t S, int64_t Hq,
                            int64_t Hkv, int64_t D, const float* cos_t, const float* sin_t,
                            void* q_out, void* k_cache, void* v_cache, int64_t Lmax, int dtype,
                            void* stream) {
  if (!q || !k || !v || !pos0 || !cos_t || !sin_t || !q_out || !k_cache || !v_cache) return CSAQ_ERR_ARG;
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || D % 2 || Lmax <= 0) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  cudaStream_t st = as_stream(stream);
  const int64_t M = B * S;
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(rope_kv_kernel<__nv_bfloat16>, dim3(M), dim3(256), 0, st, (const __nv_bfloat16*)q, ldq, (const __nv_bfloat16*)k, ldk, (const __nv_bfloat16*)v, ldv, pos0, (int)S, (int)Hq, (int)Hkv, (int)D, cos_t, sin_t, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_cache, (__nv_bfloat16*)v_cache, (int)Lmax);
  else
    return launch_pdl(rope_kv_kernel<__half>, dim3(M), dim3(256), 0, st, (const __half*)q, ldq, (const __half*)k, ldk, (const __half*)v, ldv, pos0, (int)S, (int)Hq, (int)Hkv, (int)D, cos_t, sin_t, (__half*)q_out, (__half*)k_cache, (__half*)v_cache, (int)Lmax);
}

extern "C" int64_t csaq_attention_workspace_floats(int64_t B, int64_t S, int64_t Hq, int64_t Hkv,
                                                   int64_t D, int64_t Lmax) {
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || Lmax <= 0) return -1;
  const int64_t n_split = (Lmax + kChunk - 1) / kChunk;
  return B * Hkv * n_split * S * (Hq / Hkv) * (D + 2);
}

extern "C" int csaq_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                                     const int32_t* pos0, int64_t B, int64_t S, int64_t Hq,
                                     int64_t Hkv, int64_t D, int64_t Lmax, float scale, float* part,
                                     int32_t* tickets, void* out, int dtype, void* stream) {
  if (!q || !k_cache || !v_cache || !pos0 || !part || !tickets || !out) return CSAQ_ERR_ARG;
  if (D != 128) return CSAQ_ERR_UNSUPPORTED;
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Lmax <= 0) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  const dim3 grid((unsigned)(B * Hkv), (unsigned)((Lmax + kChunk - 1) / kChunk));
  cudaStream_t st = as_stream(stream);
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(attention_kernel<__nv_bfloat16>, dim3(grid), dim3(kAttnWarps * 32), 0, st, (const __nv_bfloat16*)q, (const __nv_bfloat16*)k_cache, (const __nv_bfloat16*)v_cache, pos0, (int)S, (int)Hq, (int)Hkv, (int)Lmax, scale, part, tickets, (__nv_bfloat16*)out);
  else
    return launch_pdl(attention_kernel<__half>, dim3(grid), dim3(kAttnWarps * 32), 0, st, (const __half*)q, (const __half*)k_cache, (const __half*)v_cache, pos0, (int)S, (int)Hq, (int)Hkv, (int)Lmax, scale, part, tickets, (__half*)out);
}

extern "C" int csaq_silu_mul(const void* g, int64_t ldg, const void* u, int64_t ldu, void* h,
                             int64_t ldh, int64_t M, int64_t N, int dtype, void* stream) {
  if (!g || !u || !h || M < 0 || N <= 0) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  if (M == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(silu_mul_kernel<__nv_bfloat16>, dim3(blocks_for(M * N)), dim3(256), 0, st, (const __nv_bfloat16*)g, ldg, (const __nv_bfloat16*)u, ldu, (__nv_bfloat16*)h, ldh, M, (int)N);
  else
    return launch_pdl(silu_mul_kernel<__half>, dim3(blocks_for(M * N)), dim3(256), 0, st, (const __half*)g, ldg, (const __half*)u, ldu, (__half*)h, ldh, M, (int)N);
}

extern "C" int csaq_spec_accept(const int64_t* draft, const int64_t* verify_argmax, int64_t B,
                                int64_t K, int32_t* pos0, int64_t* out_tokens, int32_t* n_out,
                                int64_t cap, int64_t* next_tok, int32_t* n_new, int64_t* stats,
                                int32_t* remaining, void* stream) {
  if (!draft || !verify_argmax || !pos0 || !out_tokens || !n_out || !next_tok || !n_new || !stats || !remaining)
    return CSAQ_ERR_ARG;
  if (B <= 0 || K <= 0 || cap <= 0) return CSAQ_ERR_ARG;
  return launch_pdl(accept_kernel, dim3(blocks_for(B, 128)), dim3(128), 0, as_stream(stream), draft,
                    verify_argmax, (int)B, (int)K, pos0, out_tokens, n_out, (int)cap, next_tok, n_new, stats,
                    remaining);
}

extern "C" int csaq_greedy_commit(const int64_t* tok, int64_t B, int32_t* pos0, int64_t* out_tokens,
                                  int32_t* n_out, int64_t cap, int64_t* next_tok, int32_t* remaining,
                                  void* stream) {
  if (!tok || !pos0 || !out_tokens || !n_out || !next_tok || !remaining || B <= 0 || cap <= 0)
    return CSAQ_ERR_ARG;
  return launch_pdl(commit_kernel, dim3(blocks_for(B, 128)), dim3(128), 0, as_stream(stream), tok, (int)B,
                    pos0, out_tokens, n_out, (int)cap, next_tok, remaining);
}

// ── csaq_decode_attention_static: decode attention with library-owned scratch
// For callers with no device allocator of their own (see the header). The
// scratch holds what csaq_decode_attention's `part` and `tickets` hold: the
// per-chunk partial softmax results (rewritten by every call) and one ticket
// per (sequence, KV head), which must start at zero and which every completed
// call leaves at zero.
static __device__ __align__(256) uint8_t g_attn_scratch[CSAQ_ATTENTION_STATIC_SCRATCH_BYTES];

namespace csaq {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_attn_mu;
void* g_attn_ptr[kMaxDevices];

// Once per device, with that device current: the buffer's address, zero-filled.
int attn_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return CSAQ_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return CSAQ_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_attn_mu);
  if (!g_attn_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e == cudaSuccess) e = cudaMemset(p, 0, CSAQ_ATTENTION_STATIC_SCRATCH_BYTES);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return CSAQ_ERR_CUDA;
    }
    g_attn_ptr[dev] = p;
  }
  *out = g_attn_ptr[dev];
  return CSAQ_OK;
}
}  // namespace
}  // namespace csaq

extern "C" int csaq_decode_attention_static(const void* q, const void* k_cache, const void* v_cache,
                                            const int32_t* pos0, int64_t B, int64_t S, int64_t Hq,
                                            int64_t Hkv, int64_t D, int64_t Lmax, float scale, void* out,
                                            int dtype, void* stream) {
  if (!q || !k_cache || !v_cache || !pos0 || !out) return CSAQ_ERR_ARG;
  const int64_t floats = csaq_attention_workspace_floats(B, S, Hq, Hkv, D, Lmax);
  if (floats < 0) return CSAQ_ERR_ARG;
  const int64_t part_bytes = (floats * 4 + 255) / 256 * 256;
  if (part_bytes + B * Hkv * 4 > CSAQ_ATTENTION_STATIC_SCRATCH_BYTES) return CSAQ_ERR_SCRATCH;
  void* scratch = nullptr;
  const int rc = attn_scratch(&scratch);
  if (rc) return rc;
  float* part = reinterpret_cast<float*>(scratch);
  int32_t* tickets = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(scratch) + part_bytes);
  return csaq_decode_attention(q, k_cache, v_cache, pos0, B, S, Hq, Hkv, D, Lmax, scale, part, tickets, out,
                               dtype, stream);
}
