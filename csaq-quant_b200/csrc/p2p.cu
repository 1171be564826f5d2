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

template <typename T>
__global__ void tp_exchange_kernel(const csaq_p2p_group G, int64_t part_offset, int64_t ld_p, T* __restrict__ out,
                                   int64_t ldo, int64_t M, int N, long long spin_limit) {
  pdl_wait();  // this rank's partial, written by the previous kernel, is complete
  pdl_trigger();
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
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < M * N; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / N, n = i - m * N;
    float v = to_f32<T>(out[m * ldo + n]);
    for (int r = 0; r < G.n_ranks; ++r)
      v = __fadd_rn(v, to_f32<T>(__ldcg(reinterpret_cast<const T*>(G.parts[r]) + part_offset + m * ld_p + n)));  // not from L1
    out[m * ldo + n] = from_f32<T>(v);
  }
  // the last CTA to finish advances the exchange count for the next launch
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
