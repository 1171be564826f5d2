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
#include "rmsnorm.cuh"

namespace csaq {
namespace {

CSAQ_GUARD_RECORD()

// ── RMSNorm (HF Llama/Qwen2): one CTA per row (rmsnorm.cuh) ────────────────
template <typename T>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const T* __restrict__ x, int64_t ldx,
                                                               const T* __restrict__ w, T* __restrict__ y,
                                                               int64_t ldy, int H, float eps) {
  pdl_trigger();  // the next kernel may launch now; it waits for this one before reading y
  pdl_wait();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  rmsnorm_row<T>(x + row * ldx, w, y + row * ldy, H, eps, red);
}

// ── rotary embedding of q and k + KV-cache write ────────────────────────────
// q (M, Hq*D), k/v (M, Hkv*D) may be row slices of one fused buffer (ld_*).
// cos/sin: (Lmax, D) fp32 holding the model-dtype-rounded values.
// rotate_half convention: out_i = x_i cos_i - x_{i+D/2} sin_i (i < D/2),
//                         out_i = x_i cos_i + x_{i-D/2} sin_i (i >= D/2).
// One thread per (token, head, 8 rotary pairs): it loads x[i..i+8) and
// x[i+D/2..i+D/2+8) of its head (16-byte vectors) and the matching cos/sin,
// so every rotation is local and all loads go out in one round trip. Heads
// Hq .. Hq+Hkv-1 are the key heads (rotated into the cache); the value
// heads are copied to the cache by threads of their own.
template <typename T>
__global__ void rope_kv_kernel(const T* __restrict__ q, int64_t ldq, const T* __restrict__ k,
                               int64_t ldk, const T* __restrict__ v, int64_t ldv,
                               const int32_t* __restrict__ pos0, int S, int Hq, int Hkv, int D,
                               const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                               T* __restrict__ q_out, T* __restrict__ k_cache,
                               T* __restrict__ v_cache, int Lmax) {
  pdl_wait();
  pdl_trigger();
  const int64_t m = blockIdx.y;  // token
  const int b = (int)(m / S), s = (int)(m % S);
  const int pos = pos0[b] + s;
  if (!CSAQ_GUARD(pos >= 0 && pos < Lmax, CSAQ_GUARD_ROPE_POS, pos, Lmax)) return;
  const int half = D / 2, gpr = half / 8;  // 8-pair groups per head
  const int rot = (Hq + Hkv) * gpr;          // rotation work items of the token
  const int cpy = Hkv * (D / 8);             // value vectors of the token
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx < rot) {
    const int hh = idx / gpr, i0 = (idx % gpr) * 8;
    const bool is_q = hh < Hq;
    const int h = is_q ? hh : hh - Hq;
    const T* src = is_q ? q + m * ldq + (int64_t)h * D : k + m * ldk + (int64_t)h * D;
    const uint4 a = *reinterpret_cast<const uint4*>(src + i0);
    const uint4 c = *reinterpret_cast<const uint4*>(src + i0 + half);
    const float* cs = cos_t + (int64_t)pos * D;
    const float* sn = sin_t + (int64_t)pos * D;
    float ca[8], sa[8], cb[8], sb[8];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float4 c0 = reinterpret_cast<const float4*>(cs + i0)[t];
      const float4 s0 = reinterpret_cast<const float4*>(sn + i0)[t];
      const float4 c1 = reinterpret_cast<const float4*>(cs + i0 + half)[t];
      const float4 s1 = reinterpret_cast<const float4*>(sn + i0 + half)[t];
      ca[4 * t] = c0.x; ca[4 * t + 1] = c0.y; ca[4 * t + 2] = c0.z; ca[4 * t + 3] = c0.w;
      sa[4 * t] = s0.x; sa[4 * t + 1] = s0.y; sa[4 * t + 2] = s0.z; sa[4 * t + 3] = s0.w;
      cb[4 * t] = c1.x; cb[4 * t + 1] = c1.y; cb[4 * t + 2] = c1.z; cb[4 * t + 3] = c1.w;
      sb[4 * t] = s1.x; sb[4 * t + 1] = s1.y; sb[4 * t + 2] = s1.z; sb[4 * t + 3] = s1.w;
    }
    const T* ae = reinterpret_cast<const T*>(&a);
    const T* ce = reinterpret_cast<const T*>(&c);
    uint4 lo, hi;
    T* le = reinterpret_cast<T*>(&lo);
    T* he = reinterpret_cast<T*>(&hi);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float x0 = to_f32<T>(ae[t]), x1 = to_f32<T>(ce[t]);
      le[t] = from_f32<T>(fmaf(x0, ca[t], -x1 * sa[t]));
      he[t] = from_f32<T>(fmaf(x1, cb[t], x0 * sb[t]));
    }
    T* dst = is_q ? q_out + (m * Hq + h) * D : k_cache + (((int64_t)b * Hkv + h) * Lmax + pos) * D;
    *reinterpret_cast<uint4*>(dst + i0) = lo;
    *reinterpret_cast<uint4*>(dst + i0 + half) = hi;
  } else if (idx < rot + cpy) {
    const int j = idx - rot, h = j / (D / 8), i0 = (j % (D / 8)) * 8;
    *reinterpret_cast<uint4*>(v_cache + (((int64_t)b * Hkv + h) * Lmax + pos) * D + i0) =
        *reinterpret_cast<const uint4*>(v + m * ldv + (int64_t)h * D + i0);
  }
}

// 16-byte asynchronous global -> shared copies
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src));
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// ── decode attention (GQA, causal over the new tokens) ──────────────────────
// Grid (B * Hkv, n_split). CTA (bh, sp) scores keys [sp*kChunk, (sp+1)*kChunk)
// for the R = S * G query rows of its KV head (G = Hq / Hkv), writes partial
// (max, sum, o[D]) per row, and the last CTA of (bh) to finish (atomic ticket,
// no waiting) merges the partials and writes the output. The ticket counter
// is reset by that CTA, so the workspace needs zeroing only once.
// The CTA stages its query rows in shared memory (dynamic, R x D) with one
// round trip, so the per-row loops below start without a global load, and the
// merge issues its partial loads in batches (no branch on loaded values).
constexpr int kChunk = 64;
constexpr int kAttnWarps = 16;
constexpr int kMergeBatch = 16;  // partials whose loads are issued together in the merge
constexpr int kKeyBlock = 8;     // keys scored together: independent dot products, one shuffle tree
// With up to kGroupRowsMax query rows, each row's chunk is scored as
// kKeyGroups groups of kChunk / kKeyGroups keys by different warps (a warp per
// (row, group)), whose partial states meet in shared memory and are combined
// in group order: the 16 warps share the work of a few rows.
constexpr int kKeyGroups = 4;
constexpr int kGroupRowsMax = 32;
__host__ __device__ constexpr int key_groups(int R) { return R <= kGroupRowsMax ? kKeyGroups : 1; }

// ROPE: the launch also does csaq_rope_kv's work for the step's tokens (same
// expressions, so the same bits): q holds the unrotated queries (rows ldq
// apart), every CTA rotates its own query rows into shared memory, and the CTA
// whose chunk holds a new position rotates that key and copies its value from
// knew / vnew (rows ldq apart) into shared memory and into the cache.
struct RopeArgs {
  const void* knew;
  const void* vnew;
  int64_t ldq;
  const float* cos_t;
  const float* sin_t;
};

// csaq_rope_kv's rotation of 8 pairs (x[i0..i0+8), x[i0+D/2..i0+D/2+8)) at `pos`
template <typename T, int D>
__device__ __forceinline__ void rope8(const T* src, int i0, const float* cos_t, const float* sin_t, int pos,
                                      uint4& lo, uint4& hi) {
  constexpr int half = D / 2;
  const uint4 a = *reinterpret_cast<const uint4*>(src + i0);
  const uint4 c = *reinterpret_cast<const uint4*>(src + i0 + half);
  const float* cs = cos_t + (int64_t)pos * D;
  const float* sn = sin_t + (int64_t)pos * D;
  float ca[8], sa[8], cb[8], sb[8];
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const float4 c0 = reinterpret_cast<const float4*>(cs + i0)[t];
    const float4 s0 = reinterpret_cast<const float4*>(sn + i0)[t];
    const float4 c1 = reinterpret_cast<const float4*>(cs + i0 + half)[t];
    const float4 s1 = reinterpret_cast<const float4*>(sn + i0 + half)[t];
    ca[4 * t] = c0.x; ca[4 * t + 1] = c0.y; ca[4 * t + 2] = c0.z; ca[4 * t + 3] = c0.w;
    sa[4 * t] = s0.x; sa[4 * t + 1] = s0.y; sa[4 * t + 2] = s0.z; sa[4 * t + 3] = s0.w;
    cb[4 * t] = c1.x; cb[4 * t + 1] = c1.y; cb[4 * t + 2] = c1.z; cb[4 * t + 3] = c1.w;
    sb[4 * t] = s1.x; sb[4 * t + 1] = s1.y; sb[4 * t + 2] = s1.z; sb[4 * t + 3] = s1.w;
  }
  const T* ae = reinterpret_cast<const T*>(&a);
  const T* ce = reinterpret_cast<const T*>(&c);
  T* le = reinterpret_cast<T*>(&lo);
  T* he = reinterpret_cast<T*>(&hi);
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const float x0 = to_f32<T>(ae[t]), x1 = to_f32<T>(ce[t]);
    le[t] = from_f32<T>(fmaf(x0, ca[t], -x1 * sa[t]));
    he[t] = from_f32<T>(fmaf(x1, cb[t], x0 * sb[t]));
  }
}

template <typename T, int D, bool ROPE>
__global__ void __launch_bounds__(kAttnWarps * 32) attention_kernel(
    const T* __restrict__ q, T* __restrict__ k_cache, T* __restrict__ v_cache,
    const int32_t* __restrict__ pos0, int S, int Hq, int Hkv, int Lmax, float scale,
    float* __restrict__ part, int32_t* __restrict__ tickets, T* __restrict__ out, const RopeArgs ra) {
  constexpr int E = D / 32;  // head elements per lane
  constexpr int half = D / 2, gpr = half / 8;
  const int bh = blockIdx.x, sp = blockIdx.y, n_split = gridDim.y;
  const int b = bh / Hkv, h = bh % Hkv;
  const int G = Hq / Hkv, R = S * G;
  pdl_trigger();  // the next kernel may launch now; it waits for this one before reading out
  // pos0 and the cache below pos0 were written before the step began (by the
  // host-ordered position update and by this layer's attention of earlier
  // steps); only the kernels of the current layer, which start once their
  // predecessor's CTAs are all running, can still be in flight: the chunk's
  // old keys and values are copied before waiting, the new ones (from the
  // predecessor's q/k/v) after
  const int p0 = pos0[b];
  // every CTA of this head sees the same p0, so all of them skip together and
  // the merge ticket stays consistent
  if (!CSAQ_GUARD(p0 >= 0 && p0 + S <= Lmax, CSAQ_GUARD_ATTN_POS, p0, Lmax - S)) return;
  const int len = p0 + S;  // keys visible to the last new token
  const int k0 = sp * kChunk;
  __shared__ __align__(16) T ks[kChunk][D];
  __shared__ __align__(16) T vs[kChunk][D];
  extern __shared__ __align__(16) uint8_t attn_dyn[];
  T* qs = reinterpret_cast<T*>(attn_dyn);  // [R][D] the (rotated) query rows, unscaled
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_keys = max(0, min(kChunk, len - k0));
  const int n_old = max(0, min(n_keys, p0 - k0));
  const T* kb = k_cache + (((int64_t)b * Hkv + h) * Lmax + k0) * D;
  const T* vb = v_cache + (((int64_t)b * Hkv + h) * Lmax + k0) * D;
  for (int e = threadIdx.x; e < n_old * D / 8; e += blockDim.x) {
    cp_async16(reinterpret_cast<uint4*>(&ks[0][0]) + e, reinterpret_cast<const uint4*>(kb) + e);
    cp_async16(reinterpret_cast<uint4*>(&vs[0][0]) + e, reinterpret_cast<const uint4*>(vb) + e);
  }
  pdl_wait();
  if constexpr (ROPE) {
    // the chunk's new positions: rotated keys and copied values, into shared
    // memory and the cache (work items as csaq_rope_kv: 8 rotary pairs, or one
    // 16-byte value vector); then the query rows, rotated
    const int n_new = n_keys - n_old;
    for (int w = threadIdx.x; w < n_new * (gpr + D / 8); w += blockDim.x) {
      const int j = n_old + w / (gpr + D / 8), item = w % (gpr + D / 8);
      const int pos = k0 + j;
      const int64_t m = (int64_t)b * S + (pos - p0);  // token row of the step
      if (item < gpr) {
        const int i0 = item * 8;
        uint4 lo, hi;
        rope8<T, D>(reinterpret_cast<const T*>(ra.knew) + m * ra.ldq + (int64_t)h * D, i0, ra.cos_t, ra.sin_t, pos,
                    lo, hi);
        T* kc = k_cache + (((int64_t)b * Hkv + h) * Lmax + pos) * D;
        *reinterpret_cast<uint4*>(&ks[j][i0]) = lo;
        *reinterpret_cast<uint4*>(&ks[j][i0 + half]) = hi;
        *reinterpret_cast<uint4*>(kc + i0) = lo;
        *reinterpret_cast<uint4*>(kc + i0 + half) = hi;
      } else {
        const int i0 = (item - gpr) * 8;
        const uint4 v4 =
            *reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(ra.vnew) + m * ra.ldq + (int64_t)h * D + i0);
        *reinterpret_cast<uint4*>(&vs[j][i0]) = v4;
        *reinterpret_cast<uint4*>(v_cache + (((int64_t)b * Hkv + h) * Lmax + pos) * D + i0) = v4;
      }
    }
    for (int w = threadIdx.x; w < R * gpr; w += blockDim.x) {
      const int r = w / gpr, i0 = (w % gpr) * 8;
      const int s = r / G, hq = h * G + r % G;
      uint4 lo, hi;
      rope8<T, D>(q + ((int64_t)b * S + s) * ra.ldq + (int64_t)hq * D, i0, ra.cos_t, ra.sin_t, p0 + s, lo, hi);
      *reinterpret_cast<uint4*>(qs + (int64_t)r * D + i0) = lo;
      *reinterpret_cast<uint4*>(qs + (int64_t)r * D + i0 + half) = hi;
    }
  } else {
    for (int e = n_old * D / 8 + threadIdx.x; e < n_keys * D / 8; e += blockDim.x) {
      cp_async16(reinterpret_cast<uint4*>(&ks[0][0]) + e, reinterpret_cast<const uint4*>(kb) + e);
      cp_async16(reinterpret_cast<uint4*>(&vs[0][0]) + e, reinterpret_cast<const uint4*>(vb) + e);
    }
    for (int e = threadIdx.x; e < R * (D / 8); e += blockDim.x) {
      const int r = e / (D / 8), i0 = (e % (D / 8)) * 8;
      const int s = r / G, hq = h * G + r % G;
      cp_async16(qs + (int64_t)r * D + i0, q + (((int64_t)b * S + s) * Hq + hq) * D + i0);
    }
  }
  cp_async_commit_wait_all();
  __syncthreads();
  // partial layout: [bh][sp][r][D + 2]
  float* pbase = part + ((int64_t)bh * n_split + sp) * R * (D + 2);
  const int NG = key_groups(R), kq = kChunk / NG;
  // with NG > 1: the groups' states [r][g][D + 2], after the staged query rows
  float* gpart = reinterpret_cast<float*>(attn_dyn + ((int64_t)R * D * sizeof(T) + 15) / 16 * 16);
  for (int task = warp; task < R * NG; task += kAttnWarps) {
    const int r = task / NG, grp = task - r * NG;
    const int s = r / G;
    const int qpos = p0 + s;  // attends keys 0..qpos
    float qv[E];
#pragma unroll
    for (int i = 0; i < E; ++i) qv[i] = to_f32<T>(qs[(int64_t)r * D + lane * E + i]) * scale;
    const int kmax = min(n_keys, qpos - k0 + 1);
    const int j0 = grp * kq, j1 = min(kmax, j0 + kq);  // this group's keys
    float m = -INFINITY, l = 0.0f, o[E];
#pragma unroll
    for (int i = 0; i < E; ++i) o[i] = 0.0f;
    int j = j0;
    for (; j + kKeyBlock <= j1; j += kKeyBlock) {  // a block of keys: independent dot products
      float d[kKeyBlock];
#pragma unroll
      for (int t = 0; t < kKeyBlock; ++t) {
        d[t] = 0.0f;
#pragma unroll
        for (int i = 0; i < E; ++i) d[t] = fmaf(qv[i], to_f32<T>(ks[j + t][lane * E + i]), d[t]);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int t = 0; t < kKeyBlock; ++t) d[t] += __shfl_xor_sync(0xffffffffu, d[t], off);
      float mn = m;
#pragma unroll
      for (int t = 0; t < kKeyBlock; ++t) mn = fmaxf(mn, d[t]);
      const float corr = __expf(m - mn);
      float p[kKeyBlock], ps = 0.0f;
#pragma unroll
      for (int t = 0; t < kKeyBlock; ++t) {
        p[t] = __expf(d[t] - mn);
        ps += p[t];
      }
      l = fmaf(l, corr, ps);
#pragma unroll
      for (int i = 0; i < E; ++i) {
        float acc = o[i] * corr;
#pragma unroll
        for (int t = 0; t < kKeyBlock; ++t) acc = fmaf(p[t], to_f32<T>(vs[j + t][lane * E + i]), acc);
        o[i] = acc;
      }
      m = mn;
    }
    for (; j < j1; ++j) {
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < E; ++i) d = fmaf(qv[i], to_f32<T>(ks[j][lane * E + i]), d);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
      const float mn = fmaxf(m, d);
      const float corr = __expf(m - mn), p = __expf(d - mn);
      l = l * corr + p;
#pragma unroll
      for (int i = 0; i < E; ++i) o[i] = fmaf(o[i], corr, p * to_f32<T>(vs[j][lane * E + i]));
      m = mn;
    }
    float* pr = NG == 1 ? pbase + (int64_t)r * (D + 2) : gpart + (int64_t)task * (D + 2);
#pragma unroll
    for (int i = 0; i < E; ++i) pr[lane * E + i] = o[i];
    if (lane == 0) { pr[D] = m; pr[D + 1] = l; }
  }
  if (NG > 1) {
    __syncthreads();
    // the chunk's state of each row from its groups, in group order; a group
    // without keys holds m = -inf, l = 0, o = 0 (weight 0), and a row without
    // keys in this chunk keeps that state
    for (int r = warp; r < R; r += kAttnWarps) {
      const float* gp = gpart + (int64_t)r * NG * (D + 2);
      float M_ = -INFINITY;
      for (int g = 0; g < NG; ++g) M_ = fmaxf(M_, gp[g * (D + 2) + D]);
      float L = 0.0f, o[E];
#pragma unroll
      for (int i = 0; i < E; ++i) o[i] = 0.0f;
      if (M_ != -INFINITY) {
        for (int g = 0; g < NG; ++g) {
          const float w = __expf(gp[g * (D + 2) + D] - M_);
          L = fmaf(gp[g * (D + 2) + D + 1], w, L);
#pragma unroll
          for (int i = 0; i < E; ++i) o[i] = fmaf(gp[g * (D + 2) + lane * E + i], w, o[i]);
        }
      }
      float* pr = pbase + (int64_t)r * (D + 2);
#pragma unroll
      for (int i = 0; i < E; ++i) pr[lane * E + i] = o[i];
      if (lane == 0) { pr[D] = M_; pr[D + 1] = L; }
    }
  }
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) is_last = (atomicAdd(&tickets[bh], 1) == n_split - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // merge, in chunk order: an empty chunk left m = -inf, l = 0, o = 0, whose
  // weight exp(-inf - M) is 0, so every chunk is added without a branch on the
  // loaded values and the loads of a batch go out together; with at most one
  // batch of chunks the maxima come from the same loads (one round trip)
  for (int r = warp; r < R; r += kAttnWarps) {
    const int s = r / G, hq = h * G + r % G;
    const float* prow = part + ((int64_t)bh * n_split * R + r) * (D + 2);  // chunk p at + p * R * (D + 2)
    const int64_t pstride = (int64_t)R * (D + 2);
    float M_ = -INFINITY;  // the maxima (a maximum is exact in any order)
    const bool one_batch = n_split <= kMergeBatch;
    if (!one_batch) {  // lane-parallel first; one batch finds them among its own loads
      for (int p = lane; p < n_split; p += 32) M_ = fmaxf(M_, __ldcg(prow + p * pstride + D));
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) M_ = fmaxf(M_, __shfl_xor_sync(0xffffffffu, M_, off));
    }
    float L = 0.0f, o[E];
#pragma unroll
    for (int i = 0; i < E; ++i) o[i] = 0.0f;
    for (int p0b = 0; p0b < n_split; p0b += kMergeBatch) {
      float mb[kMergeBatch], lb[kMergeBatch], ob[kMergeBatch][E];
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        const bool ok = p0b + u < n_split;
        const float* pr = prow + (p0b + u) * pstride;
        mb[u] = ok ? __ldcg(pr + D) : -INFINITY;
        lb[u] = ok ? __ldcg(pr + D + 1) : 0.0f;
#pragma unroll
        for (int i = 0; i < E; ++i) ob[u][i] = ok ? __ldcg(pr + lane * E + i) : 0.0f;
      }
      if (one_batch) {
#pragma unroll
        for (int u = 0; u < kMergeBatch; ++u) M_ = fmaxf(M_, mb[u]);
      }
#pragma unroll
      for (int u = 0; u < kMergeBatch; ++u) {
        if (p0b + u >= n_split) break;
        const float w = __expf(mb[u] - M_);
        L = fmaf(lb[u], w, L);
#pragma unroll
        for (int i = 0; i < E; ++i) o[i] = fmaf(ob[u][i], w, o[i]);
      }
    }
    T* orow = out + (((int64_t)b * S + s) * Hq + hq) * D;
    const float inv = L > 0.0f ? 1.0f / L : 0.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) orow[lane * E + i] = from_f32<T>(o[i] * inv);
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

// ── tensor-parallel combine: out = T(out + sum_r parts[r]) in rank order ─────
// parts: n_parts slices of (M, N) at part_stride elements apart, rows ld_p
// apart; the fp32 sum runs over the ranks in order, so the result does not
// depend on how many tokens share the call.
template <typename T>
__global__ void rank_sum_kernel(const T* __restrict__ parts, int n_parts, int64_t part_stride, int64_t ld_p,
                                T* __restrict__ out, int64_t ldo, int64_t M, int N, int add_out) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= M * N) return;
  const int64_t m = i / N, n = i - m * N;
  float v = add_out ? to_f32<T>(out[m * ldo + n]) : 0.0f;
  for (int r = 0; r < n_parts; ++r) v = __fadd_rn(v, to_f32<T>(parts[r * part_stride + m * ld_p + n]));
  out[m * ldo + n] = from_f32<T>(v);
}

// ── argmax over vocabulary slices ───────────────────────────────────────────
// Row m of the logits is the concatenation of n_parts slices of part_len
// values (slice r at part_stride * r, rows ld apart); idx[m] is the global
// index of the largest value, the smallest such index on ties (as
// torch.argmax). One CTA per row.
constexpr int kArgThreads = 1024;

template <typename T>
__global__ void __launch_bounds__(kArgThreads) argmax_kernel(const T* __restrict__ logits, int n_parts,
                                                             int64_t part_stride, int64_t ld, int64_t part_len,
                                                             int64_t* __restrict__ idx) {
  pdl_trigger();
  pdl_wait();
  const int64_t m = blockIdx.x;
  float best = -INFINITY;
  int64_t bi = INT64_MAX;
  auto take = [&](float v, int64_t g) {
    if (v > best || (v == best && g < bi)) { best = v; bi = g; }
  };
  for (int r = 0; r < n_parts; ++r) {
    const T* row = logits + r * part_stride + m * ld;
    int64_t j0 = 0;
    if (reinterpret_cast<uintptr_t>(row) % 16 == 0) {
      // 8 values per 16-byte load, four loads in flight per thread
      const int64_t n8 = part_len / 8;
      const uint4* rv = reinterpret_cast<const uint4*>(row);
      for (int64_t j = threadIdx.x; j < n8; j += 4 * (int64_t)blockDim.x) {
        uint4 q[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t jj = j + u * (int64_t)blockDim.x;
          q[u] = jj < n8 ? __ldcs(rv + jj) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t jj = j + u * (int64_t)blockDim.x;
          if (jj >= n8) break;
          const T* e = reinterpret_cast<const T*>(&q[u]);
#pragma unroll
          for (int t = 0; t < 8; ++t) take(to_f32<T>(e[t]), r * part_len + 8 * jj + t);
        }
      }
      j0 = n8 * 8;
    }
    for (int64_t j = j0 + threadIdx.x; j < part_len; j += blockDim.x) take(to_f32<T>(row[j]), r * part_len + j);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int64_t si[32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sv[warp] = best; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    best = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x >> 5) ? si[lane] : INT64_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) idx[m] = bi == INT64_MAX ? 0 : bi;
  }
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
    return launch_pdl(rmsnorm_kernel<__nv_bfloat16>, dim3(M), dim3(kNormThreads), 0, st, (const __nv_bfloat16*)x, ldx, (const __nv_bfloat16*)w, (__nv_bfloat16*)y, ldy, (int)H, eps);
  else
    return launch_pdl(rmsnorm_kernel<__half>, dim3(M), dim3(kNormThreads), 0, st, (const __half*)x, ldx, (const __half*)w, (__half*)y, ldy, (int)H, eps);
}

extern "C" int csaq_rope_kv(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                            int64_t ldv, const int32_t* pos0, int64_t B, int64_t S, int64_t Hq,
                            int64_t Hkv, int64_t D, const float* cos_t, const float* sin_t,
                            void* q_out, void* k_cache, void* v_cache, int64_t Lmax, int dtype,
                            void* stream) {
  if (!q || !k || !v || !pos0 || !cos_t || !sin_t || !q_out || !k_cache || !v_cache) return CSAQ_ERR_ARG;
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || D % 2 || Lmax <= 0) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  // 16-byte vectors of 8 rotary pairs: D % 16 == 0, rows 16-byte aligned
  auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (D % 16 || ldq % 8 || ldk % 8 || ldv % 8 || !a16(q) || !a16(k) || !a16(v) || !a16(q_out) ||
      !a16(k_cache) || !a16(v_cache) || !a16(cos_t) || !a16(sin_t))
    return CSAQ_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  const int64_t M = B * S;
  const int64_t work = (Hq + Hkv) * (D / 16) + Hkv * (D / 8);
  const dim3 grid((unsigned)((work + 255) / 256), (unsigned)M);
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(rope_kv_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, (const __nv_bfloat16*)q, ldq,
                      (const __nv_bfloat16*)k, ldk, (const __nv_bfloat16*)v, ldv, pos0, (int)S, (int)Hq, (int)Hkv,
                      (int)D, cos_t, sin_t, (__nv_bfloat16*)q_out, (__nv_bfloat16*)k_cache,
                      (__nv_bfloat16*)v_cache, (int)Lmax);
  return launch_pdl(rope_kv_kernel<__half>, grid, dim3(256), 0, st, (const __half*)q, ldq, (const __half*)k, ldk,
                    (const __half*)v, ldv, pos0, (int)S, (int)Hq, (int)Hkv, (int)D, cos_t, sin_t,
                    (__half*)q_out, (__half*)k_cache, (__half*)v_cache, (int)Lmax);
}

extern "C" int64_t csaq_attention_workspace_floats(int64_t B, int64_t S, int64_t Hq, int64_t Hkv,
                                                   int64_t D, int64_t Lmax) {
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0 || D <= 0 || Lmax <= 0) return -1;
  const int64_t n_split = (Lmax + kChunk - 1) / kChunk;
  return B * Hkv * n_split * S * (Hq / Hkv) * (D + 2);
}

// multiprocessors of the current device (looked up once)
int sm_count() {
  static int n = 0;
  if (n <= 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
  }
  return n;
}

// dynamic shared memory of the staged query rows, at least kAttnSpreadBytes:
// with the static K/V tiles that is more than half an SM's shared memory, so
// the CTAs of a launch land on distinct SMs even when the launch starts while
// the previous kernel still holds most of them (an SM freed early would
// otherwise take several CTAs, which then share its issue slots)
constexpr int kAttnQBytesMax = 160 * 1024;
constexpr int kAttnSpreadBytes = 96 * 1024;

template <typename T, bool ROPE = false>
static int launch_attention(int64_t D, dim3 grid, cudaStream_t st, const void* q, const void* k_cache,
                            const void* v_cache, const int32_t* pos0, int64_t S, int64_t Hq, int64_t Hkv,
                            int64_t Lmax, float scale, float* part, int32_t* tickets, void* out,
                            const RopeArgs& ra = RopeArgs{}) {
  auto kern = D == 64 ? attention_kernel<T, 64, ROPE> : attention_kernel<T, 128, ROPE>;
  const int64_t R = S * (Hq / Hkv);
  int64_t qbytes = (R * D * (int64_t)sizeof(T) + 15) / 16 * 16;  // the staged query rows
  if (R <= kGroupRowsMax) qbytes += R * key_groups((int)R) * (D + 2) * (int64_t)sizeof(float);  // group states
  if (qbytes > kAttnQBytesMax) return CSAQ_ERR_UNSUPPORTED;
  // spread only a grid that fits one wave: a larger one (many sequences) keeps
  // several CTAs per SM rather than running wave after wave
  if ((int64_t)grid.x * grid.y <= sm_count()) qbytes = qbytes > kAttnSpreadBytes ? qbytes : kAttnSpreadBytes;
  static bool opted[2] = {false, false};
  bool& done = opted[D == 64 ? 0 : 1];
  if (!done) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnQBytesMax) != cudaSuccess)
      return launch_status();
    done = true;
  }
  return launch_pdl(kern, grid, dim3(kAttnWarps * 32), (size_t)qbytes, st, (const T*)q, (T*)k_cache, (T*)v_cache,
                    pos0, (int)S, (int)Hq, (int)Hkv, (int)Lmax, scale, part, tickets, (T*)out, ra);
}

extern "C" int csaq_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                                     const int32_t* pos0, int64_t B, int64_t S, int64_t Hq,
                                     int64_t Hkv, int64_t D, int64_t Lmax, float scale, float* part,
                                     int32_t* tickets, void* out, int dtype, void* stream) {
  if (!q || !k_cache || !v_cache || !pos0 || !part || !tickets || !out) return CSAQ_ERR_ARG;
  if (D != 128 && D != 64) return CSAQ_ERR_UNSUPPORTED;
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Lmax <= 0) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  const dim3 grid((unsigned)(B * Hkv), (unsigned)((Lmax + kChunk - 1) / kChunk));
  cudaStream_t st = as_stream(stream);
  if (dtype == CSAQ_DT_BF16)
    return launch_attention<__nv_bfloat16>(D, grid, st, q, k_cache, v_cache, pos0, S, Hq, Hkv, Lmax, scale, part,
                                           tickets, out);
  return launch_attention<__half>(D, grid, st, q, k_cache, v_cache, pos0, S, Hq, Hkv, Lmax, scale, part, tickets,
                                  out);
}

extern "C" int csaq_decode_attention_rope(const void* q, const void* k, const void* v, int64_t ld,
                                          const int32_t* pos0, int64_t B, int64_t S, int64_t Hq, int64_t Hkv,
                                          int64_t D, const float* cos_t, const float* sin_t, void* k_cache,
                                          void* v_cache, int64_t Lmax, float scale, float* part, int32_t* tickets,
                                          void* out, int dtype, void* stream) {
  if (!q || !k || !v || !pos0 || !cos_t || !sin_t || !k_cache || !v_cache || !part || !tickets || !out)
    return CSAQ_ERR_ARG;
  if (D != 128 && D != 64) return CSAQ_ERR_UNSUPPORTED;
  if (B <= 0 || S <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || Lmax <= 0 || ld < Hq * D) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  auto a16 = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  if (ld % 8 || !a16(q) || !a16(k) || !a16(v) || !a16(k_cache) || !a16(v_cache) || !a16(cos_t) || !a16(sin_t))
    return CSAQ_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)(B * Hkv), (unsigned)((Lmax + kChunk - 1) / kChunk));
  cudaStream_t st = as_stream(stream);
  const RopeArgs ra{k, v, ld, cos_t, sin_t};
  if (dtype == CSAQ_DT_BF16)
    return launch_attention<__nv_bfloat16, true>(D, grid, st, q, k_cache, v_cache, pos0, S, Hq, Hkv, Lmax, scale,
                                                 part, tickets, out, ra);
  return launch_attention<__half, true>(D, grid, st, q, k_cache, v_cache, pos0, S, Hq, Hkv, Lmax, scale, part,
                                        tickets, out, ra);
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

extern "C" int csaq_rank_sum(const void* parts, int n_parts, int64_t part_stride, int64_t ld_parts, void* out,
                             int64_t ldo, int64_t M, int64_t N, int add_out, int dtype, void* stream) {
  if (!parts || !out || n_parts < 1 || M < 0 || N <= 0 || ld_parts < N || ldo < N) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  if (M == 0) return CSAQ_OK;
  const dim3 grid((unsigned)((M * N + 255) / 256));
  cudaStream_t st = as_stream(stream);
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(rank_sum_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, (const __nv_bfloat16*)parts, n_parts,
                      part_stride, ld_parts, (__nv_bfloat16*)out, ldo, M, (int)N, add_out);
  return launch_pdl(rank_sum_kernel<__half>, grid, dim3(256), 0, st, (const __half*)parts, n_parts, part_stride,
                    ld_parts, (__half*)out, ldo, M, (int)N, add_out);
}

extern "C" int csaq_argmax_parts(const void* logits, int n_parts, int64_t part_stride, int64_t ld,
                                 int64_t part_len, int64_t M, int64_t* idx, int dtype, void* stream) {
  if (!logits || !idx || n_parts < 1 || M < 0 || part_len <= 0 || ld < part_len) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  if (M == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(argmax_kernel<__nv_bfloat16>, dim3((unsigned)M), dim3(kArgThreads), 0, st,
                      (const __nv_bfloat16*)logits, n_parts, part_stride, ld, part_len, idx);
  return launch_pdl(argmax_kernel<__half>, dim3((unsigned)M), dim3(kArgThreads), 0, st, (const __half*)logits,
                    n_parts, part_stride, ld, part_len, idx);
}

// ── csaq_decode_attention_static: decode attention with library-owned scratch
// For callers with no device allocator of their own (see the header). The
// scratch holds what csaq_decode_attention's `part` and `tickets` hold. The
// tickets (one per sequence and KV head) sit in a fixed region at the start
// of the array, CSAQ_ATTENTION_STATIC_MAX_HEADS int32 slots that no call's
// partials reach; they start at zero and every completed call leaves the ones
// it used at zero, so a call finds its tickets at zero whatever the shape of
// the call before it. The per-chunk partial softmax results follow at
// kStaticPartOffset; every call rewrites the ones it reads.
static __device__ __align__(256) uint8_t g_attn_scratch[CSAQ_ATTENTION_STATIC_SCRATCH_BYTES];

namespace csaq {
namespace {
constexpr int kMaxDevices = 64;
constexpr int64_t kStaticPartOffset = CSAQ_ATTENTION_STATIC_MAX_HEADS * 4;  // bytes; a multiple of 256
static_assert(kStaticPartOffset % 256 == 0, "partials must stay 256-byte aligned");
std::mutex g_attn_mu;
void* g_attn_ptr[kMaxDevices];

// Once per device, with that device current: the buffer's address, zero-filled.
// The set-up synchronises the device, so it refuses to run while `st` is being
// captured into a graph (the capture would be invalidated).
int attn_scratch(cudaStream_t st, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return CSAQ_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return CSAQ_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_attn_mu);
  if (!g_attn_ptr[dev]) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(st, &cs);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return CSAQ_ERR_CUDA;
    }
    if (cs != cudaStreamCaptureStatusNone) return CSAQ_ERR_UNSUPPORTED;
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
  if (B * Hkv > CSAQ_ATTENTION_STATIC_MAX_HEADS) return CSAQ_ERR_SCRATCH;
  if (kStaticPartOffset + floats * 4 > CSAQ_ATTENTION_STATIC_SCRATCH_BYTES) return CSAQ_ERR_SCRATCH;
  void* scratch = nullptr;
  const int rc = attn_scratch(as_stream(stream), &scratch);
  if (rc) return rc;
  int32_t* tickets = reinterpret_cast<int32_t*>(scratch);
  float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch) + kStaticPartOffset);
  return csaq_decode_attention(q, k_cache, v_cache, pos0, B, S, Hq, Hkv, D, Lmax, scale, part, tickets, out,
                               dtype, stream);
}
