// Tensor-parallel combine over NVLink peer memory.
//
// After a row-split linear (o or down projection) every rank holds a partial
// output; the model needs their sum added to the residual stream, in a fixed
// (rank) order so that a token's result does not depend on how many tokens
// share the step. Instead of an NCCL all-gather followed by a summing kernel,
// one kernel per rank:
//   1. signals its peers that its partial is complete, by storing the new
//      exchange count into its slot of every peer's flag array (a release
//      store at system scope, through the peer mapping of that array);
//   2. waits, with a bounded spin, until every peer's slot in its own flag
//      array has reached that count;
//   3. reads every rank's partial straight from the rank's memory over NVLink
//      and writes out = T(out + sum_r part_r), in fp32, in rank order.
// The exchange count lives in device memory and is advanced by the kernel, so
// the launch can be captured in a CUDA graph and replayed. Buffers come from
// csaq_p2p_alloc and are mapped into the peers with the IPC helpers below.
// A partial buffer must not be rewritten before every peer has read it: the
// runtime alternates two buffers (o and down projections), and a rank writes
// a buffer again only after it has seen every peer's signal for the next
// exchange, which each peer sends after finishing its reads of this one.

#include <atomic>

#include "common.cuh"
#include "rmsnorm.cuh"

namespace csaq {
namespace {

constexpr long long kSpinLimit = 1ll << 22;  // default polls of a peer flag before giving up (a few seconds)
std::atomic<long long> g_spin_limit{kSpinLimit};  // csaq_p2p_set_spin_limit; read at each launch

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Steps 1 and 2 of the exchange (signal every peer, wait for every peer);
// returns the new exchange count.
__device__ __forceinline__ uint64_t exchange_signal_wait(const csaq_p2p_group& G, long long spin_limit) {
  __shared__ uint64_t s_seq;
  if (threadIdx.x == 0) s_seq = *G.seq;
  __syncthreads();
  const uint64_t want = s_seq + 1;
  // every CTA signals (the same value): no CTA depends on another being
  // resident. The partial was written by a kernel that has completed, so the
  // release store alone orders it before the flag for the peers.
  if (threadIdx.x < (unsigned)G.n_ranks && (int)threadIdx.x != G.rank) st_release_sys(G.flags[threadIdx.x] + G.rank, want);
  // after one abandoned wait the group is broken: later exchanges do not wait
  // again (their results are wrong, and the error count says so)
  if (threadIdx.x < (unsigned)G.n_ranks && (int)threadIdx.x != G.rank && *(volatile uint32_t*)G.err == 0u) {
    const uint64_t* f = G.flags[G.rank] + threadIdx.x;
    long long i = 0;
    while (ld_acquire_sys(f) < want) {
      if (++i == spin_limit) {
        atomicAdd(G.err, 1u);
        break;
      }
      if (i > 1024) __nanosleep(32);  // spin first: the peer is usually microseconds away
    }
  }
  __syncthreads();
  return want;
}

// the last CTA to finish advances the exchange count for the next launch
__device__ __forceinline__ void exchange_done(const csaq_p2p_group& G, uint64_t want) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(G.ticket, 1u) == gridDim.x - 1) {
      *G.ticket = 0u;
      *G.seq = want;
      __threadfence();
    }
  }
}

template <typename T>
__global__ void tp_exchange_kernel(const csaq_p2p_group G, int64_t part_offset, int64_t ld_p, T* __restrict__ out,
                                   int64_t ldo, int64_t M, int N, long long spin_limit) {
  pdl_trigger();
  pdl_wait();  // this rank's partial, written by the previous kernel, is complete
  const uint64_t want = exchange_signal_wait(G, spin_limit);
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < M * N; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float v = to_f32<T>(out[m * ldo + n]);
    for (int r = 0; r < G.n_ranks; ++r)
      v = __fadd_rn(v, to_f32<T>(__ldcg(reinterpret_cast<const T*>(G.parts[r]) + part_offset + m * ld_p + n)));  // not from L1
    out[m * ldo + n] = from_f32<T>(v);
  }
  exchange_done(G, want);
}

// The exchange followed by the RMSNorm that reads its result (the next
// layer's input norm or the post-attention norm), one CTA per row: the row's
// sum out = T(out + sum_r part_r) in rank order exactly as tp_exchange_kernel
// forms it, then xn = RMSNorm(out) exactly as rmsnorm_kernel does. One
// launch instead of two, the same bits.
template <typename T>
__global__ void __launch_bounds__(kNormThreads)
    tp_exchange_norm_kernel(const csaq_p2p_group G, int64_t part_offset, int64_t ld_p, T* __restrict__ out,
                            int64_t ldo, int64_t M, int N, const T* __restrict__ w, T* __restrict__ xn,
                            int64_t ldn, float eps, long long spin_limit) {
  pdl_trigger();
  pdl_wait();
  const uint64_t want = exchange_signal_wait(G, spin_limit);
  __shared__ float red[32];
  bool vec = N % 8 == 0 && N <= kNormThreads * 8 * kNormVec && ldo % 8 == 0 && ldn % 8 == 0 &&
             ld_p % 8 == 0 && part_offset % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
             reinterpret_cast<uintptr_t>(xn) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0;
  for (int r = 0; r < G.n_ranks; ++r) vec = vec && reinterpret_cast<uintptr_t>(G.parts[r]) % 16 == 0;
  for (int64_t m = blockIdx.x; m < M; m += gridDim.x) {
    T* orow = out + m * ldo;
    if (vec) {
      // the row's 16-byte vectors i = thread + j * kNormThreads, as rmsnorm_row
      // assigns them: every rank's vectors are loaded before any is added, so
      // the peers' partials cost one NVLink round trip
      const int nv = N / 8;
      uint4 xv[kNormVec], wv[kNormVec];
      float acc[kNormVec][8];
#pragma unroll
      for (int j = 0; j < kNormVec; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < nv) {
          xv[j] = reinterpret_cast<const uint4*>(orow)[i];
          wv[j] = reinterpret_cast<const uint4*>(w)[i];
        }
      }
#pragma unroll
      for (int j = 0; j < kNormVec; ++j) {
        const T* e = reinterpret_cast<const T*>(&xv[j]);
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[j][t] = to_f32<T>(e[t]);
      }
      for (int r = 0; r < G.n_ranks; ++r) {
        const uint4* pr = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(G.parts[r]) + part_offset + m * ld_p);
        uint4 pv[kNormVec];
#pragma unroll
        for (int j = 0; j < kNormVec; ++j) {
          const int i = threadIdx.x + j * kNormThreads;
          if (i < nv) pv[j] = __ldcg(pr + i);  // not from L1
        }
#pragma unroll
        for (int j = 0; j < kNormVec; ++j) {
          const T* e = reinterpret_cast<const T*>(&pv[j]);
#pragma unroll
          for (int t = 0; t < 8; ++t) acc[j][t] = __fadd_rn(acc[j][t], to_f32<T>(e[t]));
        }
      }
      // out = T(sum), then RMSNorm of the rounded row, as rmsnorm_row computes it
      float ss = 0.0f;
#pragma unroll
      for (int j = 0; j < kNormVec; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < nv) {
          T* e = reinterpret_cast<T*>(&xv[j]);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            e[t] = from_f32<T>(acc[j][t]);
            const float v = to_f32<T>(e[t]);
            ss = fmaf(v, v, ss);
          }
          reinterpret_cast<uint4*>(orow)[i] = xv[j];
        }
      }
      const float rn = rsqrtf(block_sum<T>(ss, red) / (float)N + eps);
      T* yr = xn + m * ldn;
#pragma unroll
      for (int j = 0; j < kNormVec; ++j) {
        const int i = threadIdx.x + j * kNormThreads;
        if (i < nv) {
          const T* e = reinterpret_cast<const T*>(&xv[j]);
          const T* we = reinterpret_cast<const T*>(&wv[j]);
          uint4 o;
          T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
          for (int t = 0; t < 8; ++t) oe[t] = from_f32<T>(to_f32<T>(we[t]) * round_to<T>(to_f32<T>(e[t]) * rn));
          reinterpret_cast<uint4*>(yr)[i] = o;
        }
      }
      __syncthreads();  // red is reused by the next row
      continue;
    }
    for (int n = threadIdx.x; n < N; n += blockDim.x) {
      float v = to_f32<T>(orow[n]);
      for (int r = 0; r < G.n_ranks; ++r)
        v = __fadd_rn(v, to_f32<T>(__ldcg(reinterpret_cast<const T*>(G.parts[r]) + part_offset + m * ld_p + n)));
      orow[n] = from_f32<T>(v);
    }
    __syncthreads();  // the row is written: the norm's loads below see it
    rmsnorm_row<T>(orow, w, xn + m * ldn, N, eps, red);
    __syncthreads();
  }
  exchange_done(G, want);
}

}  // namespace
}  // namespace csaq

using namespace csaq;

extern "C" int csaq_p2p_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes <= 0) return CSAQ_ERR_ARG;
  *ptr = nullptr;
  if (cudaMalloc(ptr, (size_t)bytes) != cudaSuccess) return launch_status();
  if (cudaMemset(*ptr, 0, (size_t)bytes) != cudaSuccess) return launch_status();
  if (cudaDeviceSynchronize() != cudaSuccess) return launch_status();
  return CSAQ_OK;
}

extern "C" int csaq_p2p_free(void* ptr) {
  if (!ptr) return CSAQ_OK;
  return cudaFree(ptr) == cudaSuccess ? CSAQ_OK : launch_status();
}

extern "C" int csaq_ipc_handle(const void* ptr, uint8_t* handle) {
  if (!ptr || !handle) return CSAQ_ERR_ARG;
  static_assert(sizeof(cudaIpcMemHandle_t) == CSAQ_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return launch_status();
  memcpy(handle, &h, sizeof(h));
  return CSAQ_OK;
}

extern "C" int csaq_ipc_open(const uint8_t* handle, void** ptr) {
  if (!handle || !ptr) return CSAQ_ERR_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  if (cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return launch_status();
  return CSAQ_OK;
}

extern "C" int csaq_ipc_close(void* ptr) {
  if (!ptr) return CSAQ_OK;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? CSAQ_OK : launch_status();
}

extern "C" int csaq_tp_exchange_sum(const csaq_p2p_group* group, int64_t part_offset, int64_t ld_parts, void* out,
                                    int64_t ldo, int64_t M, int64_t N, int dtype, void* stream) {
  if (!group || !out || M < 0 || N <= 0 || ld_parts < N || ldo < N || part_offset < 0) return CSAQ_ERR_ARG;
  const csaq_p2p_group& G = *group;
  if (G.n_ranks < 1 || G.n_ranks > CSAQ_MAX_RANKS || G.rank < 0 || G.rank >= G.n_ranks || !G.seq || !G.ticket ||
      !G.err)
    return CSAQ_ERR_ARG;
  for (int r = 0; r < G.n_ranks; ++r)
    if (!G.parts[r] || !G.flags[r]) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  if (N > INT32_MAX) return CSAQ_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  // one wave of CTAs at most, so that every CTA is resident while the others spin
  const int64_t need = (M * N + 255) / 256;
  const unsigned grid = (unsigned)(need < 1 ? 1 : (need > 128 ? 128 : need));
  const long long spin = g_spin_limit.load();
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(tp_exchange_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, G, part_offset, ld_parts,
                      reinterpret_cast<__nv_bfloat16*>(out), ldo, M, (int)N, spin);
  return launch_pdl(tp_exchange_kernel<__half>, dim3(grid), dim3(256), 0, st, G, part_offset, ld_parts,
                    reinterpret_cast<__half*>(out), ldo, M, (int)N, spin);
}

extern "C" int csaq_tp_exchange_sum_rmsnorm(const csaq_p2p_group* group, int64_t part_offset, int64_t ld_parts,
                                            void* out, int64_t ldo, int64_t M, int64_t N, const void* norm_w,
                                            void* xn, int64_t ldn, float eps, int dtype, void* stream) {
  if (!group || !out || !norm_w || !xn || M < 0 || N <= 0 || ld_parts < N || ldo < N || ldn < N ||
      part_offset < 0 || !(eps >= 0.0f))
    return CSAQ_ERR_ARG;
  const csaq_p2p_group& G = *group;
  if (G.n_ranks < 1 || G.n_ranks > CSAQ_MAX_RANKS || G.rank < 0 || G.rank >= G.n_ranks || !G.seq || !G.ticket ||
      !G.err)
    return CSAQ_ERR_ARG;
  for (int r = 0; r < G.n_ranks; ++r)
    if (!G.parts[r] || !G.flags[r]) return CSAQ_ERR_ARG;
  if (dtype != CSAQ_DT_F16 && dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  if (N > INT32_MAX) return CSAQ_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  // one CTA per row, at most one wave; rows beyond it are taken in turn
  const unsigned grid = (unsigned)(M < 1 ? 1 : (M > 128 ? 128 : M));
  const long long spin = g_spin_limit.load();
  if (dtype == CSAQ_DT_BF16)
    return launch_pdl(tp_exchange_norm_kernel<__nv_bfloat16>, dim3(grid), dim3(kNormThreads), 0, st, G, part_offset,
                      ld_parts, reinterpret_cast<__nv_bfloat16*>(out), ldo, M, (int)N,
                      reinterpret_cast<const __nv_bfloat16*>(norm_w), reinterpret_cast<__nv_bfloat16*>(xn), ldn, eps,
                      spin);
  return launch_pdl(tp_exchange_norm_kernel<__half>, dim3(grid), dim3(kNormThreads), 0, st, G, part_offset, ld_parts,
                    reinterpret_cast<__half*>(out), ldo, M, (int)N, reinterpret_cast<const __half*>(norm_w),
                    reinterpret_cast<__half*>(xn), ldn, eps, spin);
}

extern "C" int csaq_p2p_set_spin_limit(int64_t polls) {
  if (polls < 1) return CSAQ_ERR_ARG;
  g_spin_limit.store(polls);
  return CSAQ_OK;
}

extern "C" int csaq_p2p_errors(const csaq_p2p_group* group, int64_t* count) {
  if (!group || !group->err || !count) return CSAQ_ERR_ARG;
  uint32_t v = 0;
  if (cudaMemcpy(&v, group->err, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) return launch_status();
  *count = v;
  return CSAQ_OK;
}
