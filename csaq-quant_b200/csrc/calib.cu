// Calibration kernels: co-activation masks, popcount intersection counts,
// Jaccard threshold bits, the seed-order clique partition and the salience
// accumulator.
//
// Mask layout ("channel-major bits"): mask[c][w] is a uint32 whose bit b is
// token 32*w + b of channel c; tokens past the end are 0. With this layout the
// intersection count of channels i and j is sum_w popc(mask[i][w] & mask[j][w])
// and the activation count f_i is sum_w popc(mask[i][w]), both exact integers,
// equal to the fp32 matmul counts of csaq/core.py:261-263.

#include "common.cuh"

namespace csaq {
namespace {

constexpr int kThreads = 256;

// ── masks ───────────────────────────────────────────────────────────────────
// One thread per channel, 32 tokens per block row: act[t][c] reads are
// coalesced across channels; each thread writes one 32-bit word.
// mode 0: act > thr (compared in fp32; every fp16/bf16 value and thr = 0.5
//         are exact in fp32, so this is the comparison in the input dtype).
// mode 1: |act| >= tok_thr[t] (top-k hook of csaq/core.py:143-155), compared
//         on the magnitude bit patterns, which order like the values.
template <typename T>
__global__ void mask_kernel(const T* __restrict__ act, int64_t n_tok, int64_t C, int64_t ld,
                            int mode, float thr, const uint32_t* __restrict__ tok_thr,
                            uint32_t* __restrict__ bits, int64_t ld_bits, int64_t word_off) {
  const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t w = blockIdx.y;  // token word
  if (c >= C) return;
  uint32_t word = 0;
  const int64_t t0 = w * 32;
#pragma unroll 4
  for (int b = 0; b < 32; ++b) {
    const int64_t t = t0 + b;
    if (t >= n_tok) break;
    const T v = act[t * ld + c];
    bool on;
    if (mode == 0) {
      on = to_f32<T>(v) > thr;
    } else {
      const uint32_t mag = bits_of<T>(v) & (sizeof(T) == 2 ? 0x7FFFu : 0x7FFFFFFFu);
      on = mag >= tok_thr[t];
    }
    word |= (uint32_t)on << b;
  }
  bits[c * ld_bits + word_off + w] = word;
}

// The same masks from 16-byte loads: a thread reads V = 16/sizeof(T)
// channels of one token per load (a warp reads 512 contiguous bytes of a
// token row) and builds V words of 32 tokens; a CTA covers 32*V channels x
// 256 tokens and writes each channel's 8 words (32 contiguous bytes) through
// shared memory, so the bit stores are whole sectors. Needs C and ld to be
// multiples of V and a 16-byte aligned act.
template <typename T>
__global__ void __launch_bounds__(256) mask_vec_kernel(const T* __restrict__ act, int64_t n_tok, int64_t C,
                                                       int64_t ld, int mode, float thr,
                                                       const uint32_t* __restrict__ tok_thr,
                                                       uint32_t* __restrict__ bits, int64_t ld_bits,
                                                       int64_t word_off) {
  constexpr int V = 16 / sizeof(T);
  constexpr int CH = 32 * V;
  constexpr uint32_t MAG = sizeof(T) == 2 ? 0x7FFFu : 0x7FFFFFFFu;
  __shared__ uint32_t tile[CH][9];
  const int g = threadIdx.x & 31, wy = threadIdx.x >> 5;
  const int64_t c0 = int64_t(blockIdx.x) * CH;
  const int64_t cg = c0 + g * V;
  const int64_t t0 = (int64_t(blockIdx.y) * 8 + wy) * 32;
  uint32_t word[V];
#pragma unroll
  for (int q = 0; q < V; ++q) word[q] = 0u;
  auto take = [&](int b, const uint4& v) {
    const T* e = reinterpret_cast<const T*>(&v);
    const uint32_t tt = mode == 1 ? __ldg(tok_thr + t0 + b) : 0u;
#pragma unroll
    for (int q = 0; q < V; ++q) {
      const bool on = mode == 0 ? to_f32<T>(e[q]) > thr : (bits_of<T>(e[q]) & MAG) >= tt;
      word[q] |= (uint32_t)on << b;
    }
  };
  if (cg < C && t0 < n_tok) {
    const uint4* src = reinterpret_cast<const uint4*>(act + t0 * ld + cg);
    const int64_t step = ld / V;  // one token row, in 16-byte units
    const int64_t left = n_tok - t0;
    if (left >= 32) {
#pragma unroll 8
      for (int b = 0; b < 32; ++b) take(b, __ldcs(src + b * step));
    } else {
      for (int b = 0; b < (int)left; ++b) take(b, __ldcs(src + b * step));
    }
  }
#pragma unroll
  for (int q = 0; q < V; ++q) tile[g * V + q][wy] = word[q];
  __syncthreads();
  const int64_t n_words = (n_tok + 31) / 32;
  for (int e = threadIdx.x; e < CH * 8; e += blockDim.x) {
    const int ch = e >> 3, ww = e & 7;
    const int64_t c = c0 + ch, w = int64_t(blockIdx.y) * 8 + ww;
    if (c < C && w < n_words) bits[c * ld_bits + word_off + w] = tile[ch][ww];
  }
}

// Per-token k-th largest |o| by radix select on magnitude bit patterns
// (16-bit types: 2 passes of 8 bits; fp32: 4 passes). One CTA per token.
template <typename T>
__global__ void topk_threshold_kernel(const T* __restrict__ out, int64_t C, int64_t ld, int64_t k,
                                      uint32_t* __restrict__ tok_thr) {
  constexpr int NB = sizeof(T) == 2 ? 16 : 32;
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_k;
  const T* row = out + int64_t(blockIdx.x) * ld;
  uint32_t prefix = 0;       // high bits fixed so far
  uint32_t need = (uint32_t)k;  // rank (1-based, from the top) inside the prefix bucket
  for (int shift = NB - 8; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const uint32_t hi_mask = (shift + 8 >= 32) ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int64_t c = threadIdx.x; c < C; c += blockDim.x) {
      const T v = row[c];
      const uint32_t mag = bits_of<T>(v) & (sizeof(T) == 2 ? 0x7FFFu : 0x7FFFFFFFu);
      if ((mag & hi_mask) == prefix) atomicAdd(&hist[(mag >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t acc = 0;
      int d = 255;
      for (; d > 0; --d) {
        if (acc + hist[d] >= need) break;
        acc += hist[d];
      }
      s_prefix = prefix | ((uint32_t)d << shift);
      s_k = need - acc;
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_k;
    __syncthreads();
  }
  if (threadIdx.x == 0) tok_thr[blockIdx.x] = prefix;
}

// ── co-activation counts ────────────────────────────────────────────────────
// 64x64 channel tile per CTA (upper-triangle tiles only, the lower tile is
// written by transposition); 256 threads each own 4x4 counts (strided by 16);
// words stream through shared memory 32 at a time.
constexpr int kTile = 64;
constexpr int kWordsPerStage = 32;

__global__ void __launch_bounds__(256) coact_kernel(const uint32_t* __restrict__ bits, int64_t C,
                                                    int64_t n_words, int64_t ld_bits,
                                                    int32_t* __restrict__ inter, int64_t ld_i,
                                                    int n_tiles) {
  // linear upper-triangle tile index -> (ti, tj), ti <= tj
  int64_t t = blockIdx.x;
  int ti = 0;
  while (t >= n_tiles - ti) { t -= n_tiles - ti; ++ti; }
  const int tj = ti + (int)t;
  __shared__ uint32_t sa[kWordsPerStage][kTile + 1];
  __shared__ uint32_t sb[kWordsPerStage][kTile + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads
  const int64_t i0 = (int64_t)ti * kTile, j0 = (int64_t)tj * kTile;
  uint32_t acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0;
  for (int64_t w0 = 0; w0 < n_words; w0 += kWordsPerStage) {
    // load 64 channels x 32 words for each side
    for (int e = threadIdx.x; e < kTile * kWordsPerStage; e += blockDim.x) {
      const int ch = e / kWordsPerStage, ww = e % kWordsPerStage;
      const int64_t w = w0 + ww;
      const int64_t ci = i0 + ch, cj = j0 + ch;
      sa[ww][ch] = (ci < C && w < n_words) ? bits[ci * ld_bits + w] : 0u;
      sb[ww][ch] = (cj < C && w < n_words) ? bits[cj * ld_bits + w] : 0u;
    }
    __syncthreads();
    // Three words at a time through a carry-save step: for x, y, z
    // popc(x) + popc(y) + popc(z) = popc(x ^ y ^ z) + 2 popc(maj(x, y, z)),
    // exact in integers. Two population counts (the XU pipe, 16 per SM and
    // clock, the kernel's bound) replace three; the XOR and majority are one
    // LOP3 each on the ALU pipe, which has room.
#pragma unroll 1
    for (int ww = 0; ww + 3 <= kWordsPerStage; ww += 3) {
      uint32_t a[3][4], b[3][4];
#pragma unroll
      for (int t = 0; t < 3; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          a[t][q] = sa[ww + t][ty + 16 * q];  // broadcast within a half-warp
          b[t][q] = sb[ww + t][tx + 16 * q];  // 16 consecutive banks
        }
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t x = a[0][p] & b[0][q], y = a[1][p] & b[1][q], z = a[2][p] & b[2][q];
          const uint32_t sum = x ^ y ^ z, carry = (x & y) | (z & (x ^ y));
          acc[p][q] += __popc(sum) + 2u * __popc(carry);
        }
    }
#pragma unroll
    for (int ww = kWordsPerStage / 3 * 3; ww < kWordsPerStage; ++ww) {
      uint32_t a[4], b[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        a[q] = sa[ww][ty + 16 * q];
        b[q] = sb[ww][tx + 16 * q];
      }
#pragma unroll
      for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[p][q] += __popc(a[p] & b[q]);
    }
    __syncthreads();
  }
  // thread (ty, tx) owns rows i0 + ty + 16p and columns j0 + tx + 16q
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const int64_t i = i0 + ty + 16 * p;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int64_t j = j0 + tx + 16 * q;
      if (i < C && j < C) {
        inter[i * ld_i + j] = (int32_t)acc[p][q];
        if (ti != tj) inter[j * ld_i + i] = (int32_t)acc[p][q];
      }
    }
  }
}

__global__ void popc_rows_kernel(const uint32_t* __restrict__ bits, int64_t C, int64_t n_words,
                                 int64_t ld_bits, int32_t* __restrict__ f) {
  const int64_t c = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (c >= C) return;
  uint32_t s = 0;
  for (int64_t w = lane; w < n_words; w += 32) s += __popc(bits[c * ld_bits + w]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) f[c] = (int32_t)s;
}

// J = I / max(f_i + f_j - I, 1) in fp32 (csaq/core.py:263-265) and the bit
// J >= thr (thr already rounded to fp32, as torch compares a float32 tensor
// with a Python float). One warp per 8 words (256 columns) of one row: eight
// independent coalesced loads per lane, one ballot per word.
__global__ void jaccard_bits_kernel(const int32_t* __restrict__ inter, int64_t ld_i,
                                    const int32_t* __restrict__ f, int64_t C, float thr,
                                    uint32_t* __restrict__ adj, int64_t ld_adj) {
  const int64_t gw = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t words_per_row = (C + 31) / 32;
  const int64_t groups = (words_per_row + 7) / 8;
  if (gw >= C * groups) return;  // whole warps
  const int64_t i = gw / groups, w0 = (gw % groups) * 8;
  const float fi = (float)__ldg(f + i);
  const int32_t* row = inter + i * ld_i;
  int32_t v[8], fj[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int64_t j = (w0 + k) * 32 + lane;
    v[k] = j < C ? __ldcs(row + j) : 0;
    fj[k] = j < C ? __ldg(f + j) : 0;
  }
  uint32_t mine = 0u;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int64_t j = (w0 + k) * 32 + lane;
    bool on = false;
    if (j < C) {
      const float I = (float)v[k];
      const float uni = fmaxf(__fsub_rn(__fadd_rn(fi, (float)fj[k]), I), 1.0f);
      on = __fdiv_rn(I, uni) >= thr;
    }
    const uint32_t word = __ballot_sync(0xffffffffu, on);
    if (lane == k) mine = word;
  }
  if (lane < 8 && w0 + lane < words_per_row) adj[i * ld_adj + w0 + lane] = mine;
}

// Seed-order greedy partition (csaq/core.py:268-285). Channels j < i are
// always taken when seed i is reached, so clique(i) = {i} + {j > i : adj[i][j]
// and j not taken}; labels[c] = index of c's clique in seed order. Bits of
// columns >= C are ignored.
//
// Pass 1 (row_tail_kernel, parallel): flag[i] = row i has a bit above the
// diagonal, i.e. seed i may take members. The flags are written into labels,
// which pass 2 overwrites.
// Pass 2, for C above what greedy_runs_kernel below serves (greedy_seq_kernel,
// one warp): walks the seeds 32 at a time (one word
// of channels). The taken bits of the current word live in a register; a
// seed without a flag costs a few register operations, and only flagged
// seeds read their row (L2-resident after pass 1) and update the taken set of
// later words in shared memory. Labels of the current word's channels are
// kept one per lane and stored once per word; members in later words are
// labelled directly, and their flag slots are not read again (they are taken).
__global__ void row_tail_kernel(const uint32_t* __restrict__ adj, int64_t ld_adj, int64_t C,
                                int32_t* __restrict__ flag) {
  const int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= C) return;  // whole warps
  const int64_t words = (C + 31) / 32, w0 = i >> 5;
  const uint32_t last = (C & 31) ? (1u << (C & 31)) - 1u : 0xffffffffu;
  const uint32_t* row = adj + i * ld_adj;
  uint32_t any = 0u;
  for (int64_t w = w0 + lane; w < words; w += 32) {
    uint32_t v = row[w];
    if (w == w0) v &= ~((2u << (i & 31)) - 1u);
    if (w == words - 1) v &= last;
    any |= v;
  }
  any = __any_sync(0xffffffffu, any != 0u);
  if (lane == 0) flag[i] = any ? 1 : 0;
}

__global__ void __launch_bounds__(32) greedy_seq_kernel(const uint32_t* __restrict__ adj, int64_t ld_adj, int C,
                                                        int32_t* labels, int32_t* __restrict__ n_cliques) {
  extern __shared__ uint32_t taken_s[];  // taken channels, one bit each
  const int lane = threadIdx.x;
  const int words = (C + 31) / 32;
  const uint32_t last = (C & 31) ? (1u << (C & 31)) - 1u : 0xffffffffu;
  for (int w = lane; w < words; w += 32) taken_s[w] = 0u;
  __syncwarp();
  int id = 0;
  int next_flag = lane < C ? labels[lane] : 0;
  for (int w0 = 0; w0 < words; ++w0) {
    const int i0 = w0 * 32;
    const int flag = next_flag;
    next_flag = i0 + 32 + lane < C ? labels[i0 + 32 + lane] : 0;  // in flight while this word runs
    uint32_t tw = taken_s[w0];  // uniform across the warp from here on
    const uint32_t taken0 = tw;
    const uint32_t flagged = __ballot_sync(0xffffffffu, flag != 0);
    const int nb = C - i0 < 32 ? C - i0 : 32;
    int my = 0;
    for (int b = 0; b < nb; ++b) {
      if (tw & (1u << b)) continue;
      tw |= 1u << b;
      if (lane == b) my = id;
      if (flagged & (1u << b)) {
        const uint32_t* row = adj + (int64_t)(i0 + b) * ld_adj;
        const uint32_t r0 = row[w0];
        int w = w0 + 1 + lane;
        uint32_t r = w < words ? row[w] : 0u;
        uint32_t m0 = r0 & ~tw & ~((2u << b) - 1u);
        if (w0 == words - 1) m0 &= last;
        tw |= m0;
        if ((m0 >> lane) & 1u) my = id;
        for (; w < words; w += 32) {
          const uint32_t rn = w + 32 < words ? row[w + 32] : 0u;
          uint32_t m = r & ~taken_s[w];
          if (w == words - 1) m &= last;
          if (m) {
            taken_s[w] |= m;
            do {
              const int bb = __ffs(m) - 1;
              m &= m - 1;
              labels[w * 32 + bb] = id;
            } while (m);
          }
          r = rn;
        }
        __syncwarp();
      }
      ++id;
    }
    if (lane < nb && !((taken0 >> lane) & 1u)) labels[i0 + lane] = my;
    __syncwarp();
  }
  if (lane == 0) *n_cliques = id;
}

// Pass 2 when both bit sets fit shared memory (C <= kRunMaxChannels): the
// same walk, but a run of open seeds without a flag (they take no members,
// so each is a singleton clique) is labelled in one step: lane l of the run
// gets id + the number of run seeds below it. Only flagged seeds cost a row
// read. The whole CTA first packs the flags (labels on entry) into a bit set,
// so the walk never waits on a global load for them.
constexpr int kRunMaxChannels = 819200;  // 2 bit sets of C/8 bytes in 200 KB

__global__ void __launch_bounds__(1024) greedy_runs_kernel(const uint32_t* __restrict__ adj, int64_t ld_adj,
                                                           int C, int32_t* labels,
                                                           int32_t* __restrict__ n_cliques) {
  extern __shared__ uint32_t bitsets[];
  const int words = (C + 31) / 32;
  uint32_t* taken_s = bitsets;
  uint32_t* flag_s = bitsets + words;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, n_warps = blockDim.x >> 5;
  for (int w = warp; w < words; w += n_warps) {
    const int c = w * 32 + lane;
    const uint32_t f = __ballot_sync(0xffffffffu, c < C && labels[c] != 0);
    if (lane == 0) {
      flag_s[w] = f;
      taken_s[w] = 0u;
    }
  }
  __syncthreads();
  if (warp != 0) return;
  const uint32_t last = (C & 31) ? (1u << (C & 31)) - 1u : 0xffffffffu;
  const uint32_t below = (1u << lane) - 1u;
  int id = 0;
  for (int w0 = 0; w0 < words; ++w0) {
    const int i0 = w0 * 32;
    const uint32_t valid = w0 == words - 1 ? last : 0xffffffffu;
    const uint32_t flagged = flag_s[w0];
    uint32_t tw = taken_s[w0];  // uniform across the warp from here on
    const uint32_t taken0 = tw;
    int my = 0;
    while (true) {
      const uint32_t open = ~tw & valid;
      if (!open) break;
      const uint32_t fl = open & flagged;
      const uint32_t run = fl ? (open & ((fl & (0u - fl)) - 1u)) : open;  // singletons before the next flagged seed
      if ((run >> lane) & 1u) my = id + __popc(run & below);
      id += __popc(run);
      tw |= run;
      if (!fl) break;
      const int b = __ffs(fl) - 1;
      tw |= 1u << b;
      if (lane == b) my = id;
      const uint32_t* row = adj + (int64_t)(i0 + b) * ld_adj;
      const uint32_t r0 = row[w0];
      int w = w0 + 1 + lane;
      uint32_t r = w < words ? row[w] : 0u;
      const uint32_t m0 = r0 & ~tw & ~((2u << b) - 1u) & valid;
      tw |= m0;
      if ((m0 >> lane) & 1u) my = id;
      for (; w < words; w += 32) {
        const uint32_t rn = w + 32 < words ? row[w + 32] : 0u;
        uint32_t m = r & ~taken_s[w];
        if (w == words - 1) m &= last;
        if (m) {
          taken_s[w] |= m;
          do {
            const int bb = __ffs(m) - 1;
            m &= m - 1;
            labels[w * 32 + bb] = id;
          } while (m);
        }
        r = rn;
      }
      __syncwarp();
      ++id;
    }
    if (((valid & ~taken0) >> lane) & 1u) labels[i0 + lane] = my;
    __syncwarp();
  }
  if (lane == 0) *n_cliques = id;
}

// ── salience: acc += |G * W| in fp32 (csaq/core.py:204-210) ────────────────
template <typename T>
__global__ void salience_kernel(const T* __restrict__ G, const T* __restrict__ W,
                                float* __restrict__ acc, int64_t n_vec) {
  constexpr int V = 16 / sizeof(T);
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n_vec) return;
  const uint4 g = __ldg(reinterpret_cast<const uint4*>(G) + i);
  const uint4 w = __ldg(reinterpret_cast<const uint4*>(W) + i);
  const T* ge = reinterpret_cast<const T*>(&g);
  const T* we = reinterpret_cast<const T*>(&w);
  float4* ap = reinterpret_cast<float4*>(acc + i * V);
#pragma unroll
  for (int q = 0; q < V / 4; ++q) {
    float4 a = ap[q];
    a.x += fabsf(to_f32<T>(ge[4 * q + 0]) * to_f32<T>(we[4 * q + 0]));
    a.y += fabsf(to_f32<T>(ge[4 * q + 1]) * to_f32<T>(we[4 * q + 1]));
    a.z += fabsf(to_f32<T>(ge[4 * q + 2]) * to_f32<T>(we[4 * q + 2]));
    a.w += fabsf(to_f32<T>(ge[4 * q + 3]) * to_f32<T>(we[4 * q + 3]));
    ap[q] = a;
  }
}

template <typename T>
__global__ void salience_tail_kernel(const T* __restrict__ G, const T* __restrict__ W,
                                     float* __restrict__ acc, int64_t start, int64_t n) {
  const int64_t i = start + int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  acc[i] += fabsf(to_f32<T>(G[i]) * to_f32<T>(W[i]));
}

__global__ void div_kernel(float* __restrict__ a, int64_t n, float d) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) a[i] = __fdiv_rn(a[i], d);
}

inline int64_t blocks_for(int64_t n) { return (n + kThreads - 1) / kThreads; }

template <typename T>
int launch_salience(const void* G, const void* W, float* acc, int64_t n, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = (reinterpret_cast<uintptr_t>(G) % 16 == 0) && (reinterpret_cast<uintptr_t>(W) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(acc) % 16 == 0);
  int64_t done = 0;
  if (vec) {
    const int64_t nv = n / V;
    if (nv) salience_kernel<T><<<blocks_for(nv), kThreads, 0, st>>>(
        reinterpret_cast<const T*>(G), reinterpret_cast<const T*>(W), acc, nv);
    done = nv * V;
  }
  if (done < n)
    salience_tail_kernel<T><<<blocks_for(n - done), kThreads, 0, st>>>(
        reinterpret_cast<const T*>(G), reinterpret_cast<const T*>(W), acc, done, n);
  return launch_status();
}

}  // namespace
}  // namespace csaq

using namespace csaq;

extern "C" int csaq_act_mask(const void* act, int dtype, int64_t n_tok, int64_t C, int64_t ld,
                             int mode, float thr, int64_t k, uint32_t* tok_thr, uint32_t* bits,
                             int64_t ld_bits, int64_t tok_offset, void* stream) {
  if (!act || !bits || n_tok < 0 || C <= 0 || ld < C || !dtype_size(dtype)) return CSAQ_ERR_ARG;
  if (mode != 0 && mode != 1) return CSAQ_ERR_ARG;
  if (tok_offset % 32 != 0 || ld_bits < (tok_offset + n_tok + 31) / 32) return CSAQ_ERR_ARG;
  if (mode == 1 && (!tok_thr || k < 1)) return CSAQ_ERR_ARG;
  if (n_tok == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  if (mode == 1) {
    if (k >= C) {
      mode = 0;  // every channel kept: k >= C gives an all-ones mask
      thr = -INFINITY;
    } else {
      switch (dtype) {
        case CSAQ_DT_F32: topk_threshold_kernel<float><<<n_tok, 512, 0, st>>>(reinterpret_cast<const float*>(act), C, ld, k, tok_thr); break;
        case CSAQ_DT_F16: topk_threshold_kernel<__half><<<n_tok, 512, 0, st>>>(reinterpret_cast<const __half*>(act), C, ld, k, tok_thr); break;
        default: topk_threshold_kernel<__nv_bfloat16><<<n_tok, 512, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(act), C, ld, k, tok_thr); break;
      }
      const int rc = launch_status();
      if (rc) return rc;
    }
  }
  const int64_t woff = tok_offset / 32;
  const int64_t n_words = (n_tok + 31) / 32;
  const int V = 16 / (int)dtype_size(dtype);
  if (C % V == 0 && ld % V == 0 && reinterpret_cast<uintptr_t>(act) % 16 == 0 && (n_words + 7) / 8 <= 65535) {
    const dim3 vgrid((unsigned)((C + 32 * V - 1) / (32 * V)), (unsigned)((n_words + 7) / 8));
    switch (dtype) {
      case CSAQ_DT_F32: mask_vec_kernel<float><<<vgrid, 256, 0, st>>>(reinterpret_cast<const float*>(act), n_tok, C, ld, mode, thr, tok_thr, bits, ld_bits, woff); break;
      case CSAQ_DT_F16: mask_vec_kernel<__half><<<vgrid, 256, 0, st>>>(reinterpret_cast<const __half*>(act), n_tok, C, ld, mode, thr, tok_thr, bits, ld_bits, woff); break;
      default: mask_vec_kernel<__nv_bfloat16><<<vgrid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(act), n_tok, C, ld, mode, thr, tok_thr, bits, ld_bits, woff); break;
    }
    return launch_status();
  }
  if (n_words > 65535) return CSAQ_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)((C + kThreads - 1) / kThreads), (unsigned)n_words);
  switch (dtype) {
    case CSAQ_DT_F32: mask_kernel<float><<<grid, kThreads, 0, st>>>(reinterpret_cast<const float*>(act), n_tok, C, ld, mode, thr, tok_thr, bits, ld_bits, woff); break;
    case CSAQ_DT_F16: mask_kernel<__half><<<grid, kThreads, 0, st>>>(reinterpret_cast<const __half*>(act), n_tok, C, ld, mode, thr, tok_thr, bits, ld_bits, woff); break;
    default: mask_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(act), n_tok, C, ld, mode, thr, tok_thr, bits, ld_bits, woff); break;
  }
  return launch_status();
}

extern "C" int csaq_coact_counts(const uint32_t* bits, int64_t C, int64_t n_words, int64_t ld_bits,
                                 int32_t* inter, int64_t ld_i, int32_t* f, void* stream) {
  if (!bits || !inter || C <= 0 || n_words < 0 || ld_bits < n_words || ld_i < C) return CSAQ_ERR_ARG;
  cudaStream_t st = as_stream(stream);
  const int n_tiles = (int)((C + kTile - 1) / kTile);
  const int64_t n_blocks = (int64_t)n_tiles * (n_tiles + 1) / 2;
  coact_kernel<<<n_blocks, 256, 0, st>>>(bits, C, n_words, ld_bits, inter, ld_i, n_tiles);
  int rc = launch_status();
  if (rc || !f) return rc;
  popc_rows_kernel<<<blocks_for(C * 32), kThreads, 0, st>>>(bits, C, n_words, ld_bits, f);
  return launch_status();
}

extern "C" int csaq_jaccard_bits(const int32_t* inter, int64_t ld_i, const int32_t* f, int64_t C,
                                 float threshold, uint32_t* adj, int64_t ld_adj, void* stream) {
  if (!inter || !f || !adj || C <= 0 || ld_i < C || ld_adj < (C + 31) / 32) return CSAQ_ERR_ARG;
  const int64_t warps = C * (((C + 31) / 32 + 7) / 8);
  jaccard_bits_kernel<<<blocks_for(warps * 32), kThreads, 0, as_stream(stream)>>>(
      inter, ld_i, f, C, threshold, adj, ld_adj);
  return launch_status();
}

extern "C" int csaq_greedy_cliques(const uint32_t* adj, int64_t ld_adj, int64_t C, int32_t* labels,
                                   int32_t* n_cliques, void* stream) {
  if (!adj || !labels || !n_cliques || C <= 0 || ld_adj < (C + 31) / 32) return CSAQ_ERR_ARG;
  const int64_t words = (C + 31) / 32;
  if (words * 4 > 200 * 1024) return CSAQ_ERR_UNSUPPORTED;  // the taken set lives in shared memory
  cudaStream_t st = as_stream(stream);
  row_tail_kernel<<<blocks_for(C * 32), kThreads, 0, st>>>(adj, ld_adj, C, labels);
  int rc = launch_status();
  if (rc) return rc;
  if (C <= kRunMaxChannels) {
    const size_t smem = (size_t)words * 8;
    if (smem > 48 * 1024) {
      if (cudaFuncSetAttribute(greedy_runs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
        return launch_status();
    }
    greedy_runs_kernel<<<1, 1024, smem, st>>>(adj, ld_adj, (int)C, labels, n_cliques);
    return launch_status();
  }
  const size_t smem = (size_t)words * 4;
  if (cudaFuncSetAttribute(greedy_seq_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return launch_status();
  greedy_seq_kernel<<<1, 32, smem, st>>>(adj, ld_adj, (int)C, labels, n_cliques);
  return launch_status();
}

extern "C" int csaq_salience_accum(const void* G, const void* W, int dtype, int64_t n, float* acc,
                                   void* stream) {
  if (!G || !W || !acc || n < 0 || !dtype_size(dtype)) return CSAQ_ERR_ARG;
  if (n == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case CSAQ_DT_F32: return launch_salience<float>(G, W, acc, n, st);
    case CSAQ_DT_F16: return launch_salience<__half>(G, W, acc, n, st);
    default: return launch_salience<__nv_bfloat16>(G, W, acc, n, st);
  }
}

extern "C" int csaq_salience_finalize(float* acc, int64_t n, int64_t n_batches, void* stream) {
  if (!acc || n < 0 || n_batches < 1) return CSAQ_ERR_ARG;
  if (n == 0) return CSAQ_OK;
  div_kernel<<<blocks_for(n), kThreads, 0, as_stream(stream)>>>(acc, n, (float)n_batches);
  return launch_status();
}
