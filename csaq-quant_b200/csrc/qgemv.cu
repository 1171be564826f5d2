// Mixed-precision quantised linear for decode / verify (small M).
//
// Two kernels share the csaq_tier descriptor:
//
// Tensor-core kernel (qgemv_mma_kernel), reading the GEMV block layout:
//   * A tier is repacked once (csaq_repack_tiles) into contiguous blocks, one
//     per (16-row tile, 128-column chunk): the codes of rows g and g+8 that
//     MMA lane (g, c) = (lane / 4, lane % 4) consumes (columns c*32..c*32+31),
//     stored lane by lane, then the 16 rows' scales and zero points.
//   * Persistent CTAs (8 warps), each serving tiles of one tier. The warps of a
//     CTA split a tile's chunks; each warp streams its blocks through a
//     cp.async ring in shared memory (several KB in flight per warp), and the
//     warps reduce their K slices through shared memory at the tile's end.
//   * Activations are staged once per CTA as fp16 MMA B-fragments ("records"),
//     scaled per token by a power of two (exact for bf16 / fp16 inputs).
//   * Codes become fp16 MMA operands with one LOP3 per register: OR-ing a
//     nibble into the mantissa of 1024.0 gives 1024 + f*q with f = 1, 4, 16
//     or 64 set by the nibble's bit position; the matching B entry is x / f,
//     so each product is (1024 / f + q) * x. Per (chunk, token) the staging
//     pass stores C = sum_k (1024 / f_k) x_k and S = sum_k x_k, and the chunk
//     adds s * (g - C - zp * S) to the row, with g the fp32 MMA sum.
//
// CUDA-core kernel (qgemv_simt_kernel), reading the reference layout: one warp
// per (row, 8-token block), exact fp32 (q - zp) * s per element; any K, any
// group size, fp32 activations too.

#include "common.cuh"

namespace csaq {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kTileRows = 16;

struct TierParams {
  csaq_tier t[CSAQ_MAX_TIERS];
  int tile_start[CSAQ_MAX_TIERS + 1];
  int n_tiers;
};

// ── PTX helpers ─────────────────────────────────────────────────────────────
__device__ __forceinline__ uint4 ld_cached_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t mask, uint32_t magic) {
  uint32_t r;  // (a & mask) | magic in one LOP3
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(magic));
  return r;
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// ── block geometry ──────────────────────────────────────────────────────────
// Block of one (tile, chunk): codes of 16 rows x 128 columns ordered
// [h (row g or g+8)][q (16-byte piece of the lane's columns)][lane][16 B]
// (2-bit: [h][lane][8 B]), then 16 fp32 scales and 16 uint8 zero points.
template <int BITS> struct Geo {
  static constexpr int kLaneBytes = 4 * BITS;               // per row, per lane
  static constexpr int kCodeBytes = 16 * 16 * BITS;         // 16 rows x 128 columns
  static constexpr int kMetaBytes = BITS == 16 ? 0 : 80;
  static constexpr int kBlockBytes = (kCodeBytes + kMetaBytes + 15) / 16 * 16;
};

__host__ __device__ __forceinline__ int block_bytes(int bits) {
  switch (bits) {
    case 2: return Geo<2>::kBlockBytes;
    case 4: return Geo<4>::kBlockBytes;
    case 8: return Geo<8>::kBlockBytes;
    default: return Geo<16>::kBlockBytes;
  }
}

// ── repack: reference layout -> GEMV blocks ─────────────────────────────────
// One thread per 16-byte (2-bit: 8-byte) code piece or per metadata entry.
__global__ void repack_codes_kernel(const csaq_tier T, int64_t n_chunks, int bits, int64_t n_tiles,
                                    uint8_t* __restrict__ blocks) {
  const int piece = bits == 2 ? 8 : 16;
  const int lane_bytes = 4 * bits;
  const int q_per_lane = lane_bytes / piece;               // pieces per lane per row
  const int64_t pieces_per_block = 2LL * q_per_lane * 32;  // both halves
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = n_tiles * n_chunks * pieces_per_block;
  if (idx >= total) return;
  const int64_t blk = idx / pieces_per_block;
  const int p = (int)(idx % pieces_per_block);
  const int lane = p % 32, hq = p / 32, q = hq % q_per_lane, h = hq / q_per_lane;
  const int64_t tile = blk / n_chunks, ch = blk % n_chunks;
  const int g = lane >> 2, c = lane & 3;
  const int64_t row = tile * kTileRows + g + 8 * h;
  uint8_t* dst = blocks + blk * block_bytes(bits) + (int64_t)p * piece;
  const int64_t col_byte = ch * (16 * bits) + c * lane_bytes + q * piece;
  if (row < T.n_rows) {
    const uint8_t* src = T.codes + row * T.row_bytes + col_byte;
    for (int i = 0; i < piece; ++i) dst[i] = src[i];
  } else {
    for (int i = 0; i < piece; ++i) dst[i] = 0;
  }
}

__global__ void repack_meta_kernel(const csaq_tier T, int64_t n_chunks, int bits, int64_t n_tiles,
                                   uint8_t* __restrict__ blocks) {
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n_tiles * n_chunks * kTileRows) return;
  const int r = (int)(idx % kTileRows);
  const int64_t blk = idx / kTileRows;
  const int64_t tile = blk / n_chunks, ch = blk % n_chunks;
  const int64_t row = tile * kTileRows + r;
  const int64_t gi = (T.n_groups > 1) ? (ch * 128) / T.group_size : 0;
  uint8_t* meta = blocks + blk * block_bytes(bits) + 16 * 16 * bits;
  float s = 0.0f;
  uint8_t z = 0;
  if (row < T.n_rows) {
    s = T.scales[row * T.n_groups + gi];
    z = T.zps[row * T.n_groups + gi];
  }
  reinterpret_cast<float*>(meta)[r] = s;
  meta[64 + r] = z;
}

// ── activation records ──────────────────────────────────────────────────────
// Per 32-column lane block, 8 records (b0, b1) of fp16 pairs:
//   4-bit, word m (cols 8m..8m+7): [2m] = ((x0,x4),(x1/16,x5/16)), [2m+1] = ((x2,x6),(x3/16,x7/16))
//   8-bit, word m (cols 4m..4m+3): [m]  = ((x0,x2),(x1,x3))
//   2-bit, word m (cols 16m..16m+15), t = 0..3:
//          [4m+t] = ((x_{2t}/f,x_{2t+8}/f),(x_{2t+1}/f',x_{2t+9}/f')), (f, f') = (1,4),(16,64),(1,4),(16,64)
//   16-bit: [s] = ((x_{4s},x_{4s+1}),(x_{4s+2},x_{4s+3}))
template <int BITS, typename ACT>
__device__ __forceinline__ void build_records(const ACT* __restrict__ xrow, float inv, uint2 (&rec)[8],
                                              float& C, float& S) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint4 q = ld_cached_v4(xrow + 8 * i);
    const ACT* e = reinterpret_cast<const ACT*>(&q);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[8 * i + j] = to_f32<ACT>(e[j]) * inv;  // exact power-of-two scaling
  }
  float s = 0.0f, c = 0.0f;
  if constexpr (BITS == 4) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const float* x = v + 8 * m;
      rec[2 * m] = make_uint2(pack_h2(x[0], x[4]), pack_h2(x[1] * 0.0625f, x[5] * 0.0625f));
      rec[2 * m + 1] = make_uint2(pack_h2(x[2], x[6]), pack_h2(x[3] * 0.0625f, x[7] * 0.0625f));
      c += 1024.0f * (x[0] + x[4] + x[2] + x[6]) + 64.0f * (x[1] + x[5] + x[3] + x[7]);
    }
  } else if constexpr (BITS == 8) {
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const float* x = v + 4 * m;
      rec[m] = make_uint2(pack_h2(x[0], x[2]), pack_h2(x[1], x[3]));
    }
  } else if constexpr (BITS == 2) {
    const float f[4] = {1.0f, 0.0625f, 1.0f, 0.0625f};
    const float f2[4] = {0.25f, 0.015625f, 0.25f, 0.015625f};
    const float cf[4] = {1024.0f, 64.0f, 1024.0f, 64.0f};
    const float cf2[4] = {256.0f, 16.0f, 256.0f, 16.0f};
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float* x = v + 16 * m;
        rec[4 * m + t] = make_uint2(pack_h2(x[2 * t] * f[t], x[2 * t + 8] * f[t]),
                                    pack_h2(x[2 * t + 1] * f2[t], x[2 * t + 9] * f2[t]));
        c += cf[t] * (x[2 * t] + x[2 * t + 8]) + cf2[t] * (x[2 * t + 1] + x[2 * t + 9]);
      }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      rec[j] = make_uint2(pack_h2(v[4 * j], v[4 * j + 1]), pack_h2(v[4 * j + 2], v[4 * j + 3]));
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) s += v[i];
  if constexpr (BITS == 8) c = 1024.0f * s;
  C = c;
  S = s;
}

// MMA over one chunk for the MT tiles of an item (rows g and g+8 of each):
// the tiles' MMAs are interleaved and each tile alternates between two
// accumulators, so 2*MT independent chains share the tensor pipe.
template <int BITS, int MT>
__device__ __forceinline__ void chunk_mma(const uint32_t (&cw)[MT][2][BITS], const uint2 (&rec)[8],
                                          float (&g)[MT][2][4]) {
  constexpr uint32_t M = 0x64006400u;  // fp16 1024.0 in both halves
  if constexpr (BITS == 4) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint32_t v[MT][2][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint32_t w = cw[mt][r][m], t = w >> 8;
          v[mt][r][0] = lop_and_or(w, 0x000F000Fu, M);  // 1024 + q   (cols 0, 4)
          v[mt][r][1] = lop_and_or(w, 0x00F000F0u, M);  // 1024 + 16q (cols 1, 5)
          v[mt][r][2] = lop_and_or(t, 0x000F000Fu, M);  //             (cols 2, 6)
          v[mt][r][3] = lop_and_or(t, 0x00F000F0u, M);  //             (cols 3, 7)
        }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        mma_f16(g[mt][0], v[mt][0][0], v[mt][1][0], v[mt][0][1], v[mt][1][1], rec[2 * m].x, rec[2 * m].y);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        mma_f16(g[mt][1], v[mt][0][2], v[mt][1][2], v[mt][0][3], v[mt][1][3], rec[2 * m + 1].x, rec[2 * m + 1].y);
    }
  } else if constexpr (BITS == 8) {
#pragma unroll
    for (int m = 0; m < 8; ++m) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint32_t a0 = prmt(cw[mt][0][m], 0x64646464u, 0x4240), a1 = prmt(cw[mt][1][m], 0x64646464u, 0x4240);
        const uint32_t a2 = prmt(cw[mt][0][m], 0x64646464u, 0x4341), a3 = prmt(cw[mt][1][m], 0x64646464u, 0x4341);
        mma_f16(g[mt][m & 1], a0, a1, a2, a3, rec[m].x, rec[m].y);
      }
    }
  } else if constexpr (BITS == 2) {
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      uint32_t v[MT][2][8];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const uint32_t w = cw[mt][r][m], t = w >> 8;
          v[mt][r][0] = lop_and_or(w, 0x00030003u, M);
          v[mt][r][1] = lop_and_or(w, 0x000C000Cu, M);
          v[mt][r][2] = lop_and_or(w, 0x00300030u, M);
          v[mt][r][3] = lop_and_or(w, 0x00C000C0u, M);
          v[mt][r][4] = lop_and_or(t, 0x00030003u, M);
          v[mt][r][5] = lop_and_or(t, 0x000C000Cu, M);
          v[mt][r][6] = lop_and_or(t, 0x00300030u, M);
          v[mt][r][7] = lop_and_or(t, 0x00C000C0u, M);
        }
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          mma_f16(g[mt][t & 1], v[mt][0][2 * t], v[mt][1][2 * t], v[mt][0][2 * t + 1], v[mt][1][2 * t + 1],
                  rec[4 * m + t].x, rec[4 * m + t].y);
    }
  } else {
#pragma unroll
    for (int s = 0; s < 8; ++s)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        mma_f16(g[mt][s & 1], cw[mt][0][2 * s], cw[mt][1][2 * s], cw[mt][0][2 * s + 1], cw[mt][1][2 * s + 1],
                rec[s].x, rec[s].y);
  }
}

struct LaunchCfg {
  int x_bytes;   // activation records: 2 * M * K
  int cs_bytes;  // (C, S) per (chunk, token)
  int ring_div;  // 1: full ring; 2: half ring (large activations)
  int smem_bytes;
};

struct KParams {
  TierParams tp;
  int cta_start[CSAQ_MAX_TIERS + 1];  // persistent CTAs per tier
};

// Tiles per work item: two 16-row tiles share each chunk's activation
// records and give two independent MMA chains; fp16 tiers keep one (their
// blocks are already 4 KB).
template <int BITS> struct Item {
  static constexpr int kTiles = BITS == 16 ? 1 : 2;
  static constexpr int kBytes = kTiles * Geo<BITS>::kBlockBytes;
  static constexpr int kDepth = BITS == 2 ? 8 : BITS == 4 ? 4 : 2;  // ring slots per warp
};

__host__ __device__ __forceinline__ int item_tiles(int bits) { return bits == 16 ? 1 : 2; }

template <typename ACT, int NT, int BITS>
__device__ __forceinline__ void run_tier(const csaq_tier& T, int cta_in_tier, int ctas_in_tier,
                                         int64_t K, const ACT* __restrict__ x, int M, int64_t ldx,
                                         uint8_t* smem, const LaunchCfg& cfg) {
  using G = Geo<BITS>;
  using I = Item<BITS>;
  constexpr int MT = I::kTiles;
  const int depth = I::kDepth / cfg.ring_div;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int n_chunks = (int)(K / 128);
  const int n_tiles = (T.n_rows + kTileRows - 1) / kTileRows;
  const int n_units = (n_tiles + MT - 1) / MT;
  const int my_units = cta_in_tier < n_units ? (n_units - 1 - cta_in_tier) / ctas_in_tier + 1 : 0;
  const int cpw = (n_chunks + kWarps - 1) / kWarps;  // items per warp per unit (uniform)
  const int total = my_units * cpw;
  constexpr int kRows = MT * kTileRows;

  uint2* xrec = reinterpret_cast<uint2*>(smem);                               // [ch][8][M][4]
  float2* xcs = reinterpret_cast<float2*>(smem + cfg.x_bytes);                // [ch][M] (C, S)
  float* xexp = reinterpret_cast<float*>(smem + cfg.x_bytes + cfg.cs_bytes);  // [16] 2^e per token
  float* red = xexp + 16;                                                     // [warps][kRows][NT*8]
  uint8_t* ring = reinterpret_cast<uint8_t*>(red + kWarps * 32 * NT * 8) +
                  (size_t)warp * depth * I::kBytes;

  // issue cursor: unit u covers tiles u*MT .. u*MT+MT-1; the warp's items are
  // chunks warp, warp+8, ... of each of its units
  int i_it = 0, i_j = 0, i_slot = 0, i_unit = cta_in_tier;
  auto issue = [&]() {
    if (i_it < total) {
      const int ch = warp + kWarps * i_j;
      if (ch < n_chunks) {
        uint8_t* slot = ring + i_slot * I::kBytes;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int tile = i_unit * MT + mt;
          if (tile < n_tiles) {
            const uint8_t* src = T.blocks + ((int64_t)tile * n_chunks + ch) * G::kBlockBytes;
            uint8_t* dst = slot + mt * G::kBlockBytes;
#pragma unroll
            for (int off = 0; off < G::kBlockBytes; off += 512)
              if (off + lane * 16 < G::kBlockBytes) cp_async16(dst + off + lane * 16, src + off + lane * 16);
          }
        }
      }
      ++i_it;
      i_slot = (i_slot + 1 == depth) ? 0 : i_slot + 1;
      if (++i_j == cpw) {
        i_j = 0;
        i_unit += ctas_in_tier;
      }
    }
    cp_async_commit();
  };

  // prologue: weights first (they do not depend on the activation)
  for (int it = 0; it < depth; ++it) issue();

  // token scales: e_t with max|x_t| * 2^-e_t in [2^14, 2^15)
  uint32_t* smax = reinterpret_cast<uint32_t*>(xexp);
  if (threadIdx.x < 16) smax[threadIdx.x] = 0u;
  __syncthreads();
  const int k8 = (int)(K / 8);
  for (int u = threadIdx.x; u < M * k8; u += blockDim.x) {
    const int tok = u / k8, kk = u - tok * k8;
    const uint4 q = ld_cached_v4(x + (int64_t)tok * ldx + 8 * kk);
    const ACT* e = reinterpret_cast<const ACT*>(&q);
    float mx = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(to_f32<ACT>(e[j])));
    atomicMax(&smax[tok], __float_as_uint(mx));
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    const uint32_t b = smax[threadIdx.x];
    const int E = (int)((b >> 23) & 0xFF) - 127;
    xexp[threadIdx.x] = ldexpf(1.0f, b == 0u ? 0 : E - 14);  // 2^e (the output factor)
  }
  __syncthreads();

  // stage activation records; whole warps iterate together (4-lane shuffles)
  const int n_st = M * n_chunks * 4;
  for (int base = 0; base < n_st; base += blockDim.x) {
    const int u = base + threadIdx.x;
    const bool live = u < n_st;
    const int cc = u & 3;
    const int rest = u >> 2;
    const int tok = live ? rest % M : 0, ch = live ? rest / M : 0;
    uint2 rec[8];
    float Cv = 0.0f, Sv = 0.0f;
    if (live) {
      const float inv = 1.0f / xexp[tok];  // exact: a power of two
      build_records<BITS, ACT>(x + (int64_t)tok * ldx + ch * 128 + cc * 32, inv, rec, Cv, Sv);
    }
    Cv += __shfl_xor_sync(0xffffffffu, Cv, 1);
    Cv += __shfl_xor_sync(0xffffffffu, Cv, 2);
    Sv += __shfl_xor_sync(0xffffffffu, Sv, 1);
    Sv += __shfl_xor_sync(0xffffffffu, Sv, 2);
    if (live) {
#pragma unroll
      for (int j = 0; j < 8; ++j) xrec[((ch * 8 + j) * M + tok) * 4 + cc] = rec[j];
      if (cc == 0) xcs[ch * M + tok] = make_float2(Cv, Sv);
    }
  }
  __syncthreads();

  float acc[MT][NT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.0f;

  int c_j = 0, c_slot = 0, c_unit = cta_in_tier;
  for (int it = 0; it < total; ++it) {
    const int ch = warp + kWarps * c_j;
    if constexpr (I::kDepth == 8) {
      if (cfg.ring_div == 1) cp_async_wait<7>(); else cp_async_wait<3>();
    } else if constexpr (I::kDepth == 4) {
      if (cfg.ring_div == 1) cp_async_wait<3>(); else cp_async_wait<1>();
    } else {
      if (cfg.ring_div == 1) cp_async_wait<1>(); else cp_async_wait<0>();
    }
    __syncwarp();
    if (ch < n_chunks) {
      const uint8_t* slot = ring + c_slot * I::kBytes;
      // activation records of this chunk, shared by the item's tiles
      const uint2* xr = xrec + (ch * 8 * M) * 4 + c;
      uint2 rec[NT][8];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int tok = nt * 8 + g;
#pragma unroll
        for (int q = 0; q < 8; ++q) rec[nt][q] = tok < M ? xr[(q * M + tok) * 4] : make_uint2(0u, 0u);
      }
      float2 cs[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int t0 = nt * 8 + 2 * c;
        cs[nt][0] = (BITS != 16 && t0 < M) ? xcs[ch * M + t0] : make_float2(0.0f, 0.0f);
        cs[nt][1] = (BITS != 16 && t0 + 1 < M) ? xcs[ch * M + t0 + 1] : make_float2(0.0f, 0.0f);
      }
      // codes and metadata of the item's tiles (a missing second tile reads a
      // stale slot; its rows lie past n_rows and are never stored)
      uint32_t cw[MT][2][BITS];
      float sm[MT][2], zm[MT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const uint8_t* blk = slot + mt * G::kBlockBytes;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if constexpr (BITS == 2) {
            const uint2 v = reinterpret_cast<const uint2*>(blk)[h * 32 + lane];
            cw[mt][h][0] = v.x; cw[mt][h][1] = v.y;
          } else {
#pragma unroll
            for (int q = 0; q < BITS / 4; ++q) {
              const uint4 v = reinterpret_cast<const uint4*>(blk)[(h * (BITS / 4) + q) * 32 + lane];
              cw[mt][h][4 * q] = v.x; cw[mt][h][4 * q + 1] = v.y; cw[mt][h][4 * q + 2] = v.z; cw[mt][h][4 * q + 3] = v.w;
            }
          }
        }
        sm[mt][0] = sm[mt][1] = 1.0f;
        zm[mt][0] = zm[mt][1] = 0.0f;
        if constexpr (BITS != 16) {
          const float* sc = reinterpret_cast<const float*>(blk + G::kCodeBytes);
          const uint8_t* zp = blk + G::kCodeBytes + 64;
          sm[mt][0] = sc[g]; sm[mt][1] = sc[g + 8];
          zm[mt][0] = (float)zp[g]; zm[mt][1] = (float)zp[g + 8];
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float gs[MT][2][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int a = 0; a < 2; ++a) gs[mt][a][0] = gs[mt][a][1] = gs[mt][a][2] = gs[mt][a][3] = 0.0f;
        chunk_mma<BITS, MT>(cw, rec[nt], gs);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const float g0 = gs[mt][0][0] + gs[mt][1][0], g1 = gs[mt][0][1] + gs[mt][1][1];
          const float g2 = gs[mt][0][2] + gs[mt][1][2], g3 = gs[mt][0][3] + gs[mt][1][3];
          if constexpr (BITS == 16) {
            acc[mt][nt][0] += g0; acc[mt][nt][1] += g1; acc[mt][nt][2] += g2; acc[mt][nt][3] += g3;
          } else {
            acc[mt][nt][0] = fmaf(sm[mt][0], fmaf(-zm[mt][0], cs[nt][0].y, g0 - cs[nt][0].x), acc[mt][nt][0]);
            acc[mt][nt][1] = fmaf(sm[mt][0], fmaf(-zm[mt][0], cs[nt][1].y, g1 - cs[nt][1].x), acc[mt][nt][1]);
            acc[mt][nt][2] = fmaf(sm[mt][1], fmaf(-zm[mt][1], cs[nt][0].y, g2 - cs[nt][0].x), acc[mt][nt][2]);
            acc[mt][nt][3] = fmaf(sm[mt][1], fmaf(-zm[mt][1], cs[nt][1].y, g3 - cs[nt][1].x), acc[mt][nt][3]);
          }
        }
      }
    }
    __syncwarp();
    issue();
    c_slot = (c_slot + 1 == depth) ? 0 : c_slot + 1;

    if (c_j == cpw - 1) {  // end of a unit: reduce the warps' K slices
      float* rw = red + warp * kRows * NT * 8;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int r0 = mt * kTileRows + g;
          rw[r0 * NT * 8 + nt * 8 + 2 * c] = acc[mt][nt][0];
          rw[r0 * NT * 8 + nt * 8 + 2 * c + 1] = acc[mt][nt][1];
          rw[(r0 + 8) * NT * 8 + nt * 8 + 2 * c] = acc[mt][nt][2];
          rw[(r0 + 8) * NT * 8 + nt * 8 + 2 * c + 1] = acc[mt][nt][3];
          acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.0f;
        }
      __syncthreads();
      for (int i = threadIdx.x; i < kRows * NT * 8; i += blockDim.x) {
        const int r = i / (NT * 8), tok = i % (NT * 8);
        const int row = c_unit * kRows + r;
        if (row >= T.n_rows || tok >= M) continue;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[w * kRows * NT * 8 + i];
        v *= xexp[tok];
        const int orow = T.out_rows[row];
        if (T.bias) v += to_f32<ACT>(reinterpret_cast<const ACT*>(T.bias)[orow]);
        if (T.residual) v += to_f32<ACT>(reinterpret_cast<const ACT*>(T.residual)[(int64_t)tok * T.ldr + orow]);
        reinterpret_cast<ACT*>(T.y)[(int64_t)tok * T.ldy + orow] = from_f32<ACT>(v);
      }
      __syncthreads();
      c_j = 0;
      c_unit += ctas_in_tier;
    } else {
      ++c_j;
    }
  }
  cp_async_wait<0>();
}

template <typename ACT, int NT>
__global__ void __launch_bounds__(kThreads) qgemv_mma_kernel(const __grid_constant__ KParams P,
                                                             int64_t K, const ACT* __restrict__ x,
                                                             int M, int64_t ldx, LaunchCfg cfg) {
  extern __shared__ __align__(16) uint8_t smem[];
  int ti = 0;
  while (ti + 1 < P.tp.n_tiers && (int)blockIdx.x >= P.cta_start[ti + 1]) ++ti;
  const csaq_tier& T = P.tp.t[ti];
  const int cta = blockIdx.x - P.cta_start[ti];
  const int nct = P.cta_start[ti + 1] - P.cta_start[ti];
  switch (T.bits) {
    case 4: run_tier<ACT, NT, 4>(T, cta, nct, K, x, M, ldx, smem, cfg); break;
    case 8: run_tier<ACT, NT, 8>(T, cta, nct, K, x, M, ldx, smem, cfg); break;
    case 2: run_tier<ACT, NT, 2>(T, cta, nct, K, x, M, ldx, smem, cfg); break;
    default: run_tier<ACT, NT, 16>(T, cta, nct, K, x, M, ldx, smem, cfg); break;
  }
}

// ── CUDA-core reference kernel ──────────────────────────────────────────────
__device__ __forceinline__ float weight_at(const csaq_tier& T, int row, int64_t col) {
  const uint8_t* rp = T.codes + (int64_t)row * T.row_bytes;
  if (T.bits == 16) return __half2float(reinterpret_cast<const __half*>(rp)[col]);
  int q;
  if (T.bits == 8) q = rp[col];
  else if (T.bits == 4) q = (rp[col >> 1] >> ((col & 1) * 4)) & 0xF;
  else q = (rp[col >> 2] >> ((col & 3) * 2)) & 0x3;
  const int64_t gi = (int64_t)row * T.n_groups + col / T.group_size;
  return dequant_one(q, (int32_t)T.zps[gi], T.scales[gi]);
}

template <typename ACT>
__global__ void qgemv_simt_kernel(const __grid_constant__ TierParams P, int64_t K,
                                  const ACT* __restrict__ x, int M, int64_t ldx, int row_blocks) {
  const int lane = threadIdx.x & 31;
  const int64_t wid = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int tok_blocks = (M + 7) / 8;
  const int64_t row_global = wid / tok_blocks;
  const int tb = (int)(wid % tok_blocks);
  if (row_global >= row_blocks) return;
  int ti = 0;
  int64_t rr = row_global;
  while (ti < P.n_tiers && rr >= P.t[ti].n_rows) { rr -= P.t[ti].n_rows; ++ti; }
  if (ti >= P.n_tiers) return;
  const csaq_tier& T = P.t[ti];
  const int row = (int)rr;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  for (int64_t k = lane; k < K; k += 32) {
    const float w = weight_at(T, row, k);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int tok = tb * 8 + j;
      if (tok < M) acc[j] = fmaf(w, to_f32<ACT>(x[(int64_t)tok * ldx + k]), acc[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
  if (lane < 8) {
    const int tok = tb * 8 + lane;
    float v = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) if (j == lane) v = acc[j];
    if (tok < M) {
      const int orow = T.out_rows[row];
      if (T.bias) v += to_f32<ACT>(reinterpret_cast<const ACT*>(T.bias)[orow]);
      if (T.residual) v += to_f32<ACT>(reinterpret_cast<const ACT*>(T.residual)[(int64_t)tok * T.ldr + orow]);
      reinterpret_cast<ACT*>(T.y)[(int64_t)tok * T.ldy + orow] = from_f32<ACT>(v);
    }
  }
}

// ── host side ───────────────────────────────────────────────────────────────
int build_params(const csaq_tier* tiers, int n_tiers, int64_t K, TierParams& P) {
  if (!tiers || n_tiers < 1 || n_tiers > CSAQ_MAX_TIERS || K <= 0) return CSAQ_ERR_ARG;
  P.n_tiers = n_tiers;
  int tiles = 0;
  for (int i = 0; i < n_tiers; ++i) {
    const csaq_tier& t = tiers[i];
    if (t.bits != 2 && t.bits != 4 && t.bits != 8 && t.bits != 16) return CSAQ_ERR_BITS;
    if (t.n_rows < 0 || !t.out_rows || !t.y) return CSAQ_ERR_ARG;
    if (t.n_rows > 0 && !t.codes && !t.blocks) return CSAQ_ERR_ARG;
    if (t.codes && t.row_bytes < packed_row_bytes(K, t.bits)) return CSAQ_ERR_ARG;
    if (t.bits != 16 && t.codes) {
      if (!t.scales || !t.zps || t.group_size <= 0 || t.n_groups < (K + t.group_size - 1) / t.group_size)
        return CSAQ_ERR_ARG;
    }
    P.t[i] = t;
    P.tile_start[i] = tiles;
    tiles += (t.n_rows + kTileRows - 1) / kTileRows;
  }
  P.tile_start[n_tiers] = tiles;
  return CSAQ_OK;
}

bool mma_eligible(const TierParams& P, int64_t K, const void* x, int64_t ldx) {
  if (K % 128 != 0 || ldx % 8 != 0 || reinterpret_cast<uintptr_t>(x) % 16 != 0) return false;
  for (int i = 0; i < P.n_tiers; ++i) {
    const csaq_tier& t = P.t[i];
    if (t.n_rows == 0) continue;
    if (!t.blocks || reinterpret_cast<uintptr_t>(t.blocks) % 16 != 0) return false;
  }
  return true;
}

bool simt_eligible(const TierParams& P) {
  for (int i = 0; i < P.n_tiers; ++i)
    if (P.t[i].n_rows > 0 && !P.t[i].codes) return false;
  return true;
}

int g_num_sms = 0;
int num_sms() {
  if (!g_num_sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

constexpr int kSmemBudget = 227 * 1024;

int ring_bytes(int div) {
  int m = 0;
  const int r[4] = {Item<2>::kDepth * Item<2>::kBytes, Item<4>::kDepth * Item<4>::kBytes,
                    Item<8>::kDepth * Item<8>::kBytes, Item<16>::kDepth * Item<16>::kBytes};
  for (int i = 0; i < 4; ++i) m = r[i] > m ? r[i] : m;
  return kWarps * m / div;
}

// Shared memory: activation records (2*M*K), (C, S) per (chunk, token), token
// scales, the reduction buffer and the per-warp cp.async rings.
bool plan(int64_t K, int M, int NT, LaunchCfg& cfg) {
  cfg.x_bytes = (int)(2 * M * K);
  cfg.cs_bytes = (int)(((K / 128) * M * 8 + 15) / 16 * 16);
  const int fixed = cfg.x_bytes + cfg.cs_bytes + 64 + kWarps * 32 * NT * 8 * 4;
  for (int div = 1; div <= 2; div *= 2) {
    cfg.ring_div = div;
    cfg.smem_bytes = fixed + ring_bytes(div);
    if (cfg.smem_bytes <= kSmemBudget) return true;
  }
  return false;
}

template <typename ACT, int NT>
int ctas_per_sm(int smem_bytes) {
  static int cached_smem[8] = {-1, -1, -1, -1, -1, -1, -1, -1};
  static int cached_val[8];
  static int next = 0;
  static bool attr_set = false;
  for (int i = 0; i < 8; ++i)
    if (cached_smem[i] == smem_bytes) return cached_val[i];
  if (!attr_set) {
    if (cudaFuncSetAttribute(qgemv_mma_kernel<ACT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBudget) != cudaSuccess)
      return -1;
    attr_set = true;
  }
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qgemv_mma_kernel<ACT, NT>, kThreads,
                                                    smem_bytes) != cudaSuccess)
    return -1;
  per_sm = per_sm < 1 ? 1 : per_sm;
  cached_smem[next] = smem_bytes;
  cached_val[next] = per_sm;
  next = (next + 1) % 8;
  return per_sm;
}

template <typename ACT, int NT>
int launch_mma_block(const TierParams& TP, int64_t K, const ACT* x, int M, int64_t ldx,
                     cudaStream_t st) {
  LaunchCfg cfg;
  if (!plan(K, M, NT, cfg)) return CSAQ_ERR_UNSUPPORTED;
  const int per_sm = ctas_per_sm<ACT, NT>(cfg.smem_bytes);
  if (per_sm < 0) return launch_status();
  const int max_ctas = num_sms() * per_sm;
  KParams P;
  P.tp = TP;
  // persistent CTAs per tier in proportion to the tier's bytes, at most one
  // per work unit (item_tiles tiles)
  double total_bytes = 0.0;
  int total_units = 0;
  for (int i = 0; i < TP.n_tiers; ++i) {
    const csaq_tier& t = TP.t[i];
    total_bytes += (double)t.n_rows * (double)block_bytes(t.bits);
    const int tiles = (t.n_rows + kTileRows - 1) / kTileRows;
    total_units += (tiles + item_tiles(t.bits) - 1) / item_tiles(t.bits);
  }
  if (total_units == 0) return CSAQ_OK;
  const int budget = total_units < max_ctas ? total_units : max_ctas;
  int ctas = 0;
  for (int i = 0; i < TP.n_tiers; ++i) {
    const csaq_tier& t = TP.t[i];
    const int tiles = (t.n_rows + kTileRows - 1) / kTileRows;
    const int units = (tiles + item_tiles(t.bits) - 1) / item_tiles(t.bits);
    int n = 0;
    if (units > 0) {
      n = (int)((double)budget * ((double)t.n_rows * (double)block_bytes(t.bits)) / total_bytes + 0.5);
      n = n < 1 ? 1 : (n > units ? units : n);
    }
    P.cta_start[i] = ctas;
    ctas += n;
  }
  P.cta_start[TP.n_tiers] = ctas;
  qgemv_mma_kernel<ACT, NT><<<ctas, kThreads, cfg.smem_bytes, st>>>(P, K, x, M, ldx, cfg);
  return launch_status();
}

template <typename ACT>
int launch_mma(const TierParams& P0, int64_t K, const void* x, int64_t M, int64_t ldx,
               cudaStream_t st) {
  if (P0.tile_start[P0.n_tiers] == 0) return CSAQ_OK;
  int64_t m0 = 0;
  while (m0 < M) {
    // as many tokens (<= 16) as the shared-memory plan allows
    int mb = (int)((M - m0) < 16 ? (M - m0) : 16);
    LaunchCfg probe;
    while (mb > 1 && !plan(K, mb, mb > 8 ? 2 : 1, probe)) --mb;
    TierParams P = P0;
    for (int i = 0; i < P.n_tiers; ++i) {
      P.t[i].y = reinterpret_cast<ACT*>(P.t[i].y) + m0 * P.t[i].ldy;
      if (P.t[i].residual)
        P.t[i].residual = reinterpret_cast<const ACT*>(P.t[i].residual) + m0 * P.t[i].ldr;
    }
    const ACT* xb = reinterpret_cast<const ACT*>(x) + m0 * ldx;
    const int rc = mb <= 8 ? launch_mma_block<ACT, 1>(P, K, xb, mb, ldx, st)
                           : launch_mma_block<ACT, 2>(P, K, xb, mb, ldx, st);
    if (rc) return rc;
    m0 += mb;
  }
  return CSAQ_OK;
}

template <typename ACT>
int launch_simt(const TierParams& P, int64_t K, const void* x, int64_t M, int64_t ldx,
                cudaStream_t st) {
  int rows = 0;
  for (int i = 0; i < P.n_tiers; ++i) rows += P.t[i].n_rows;
  if (rows == 0) return CSAQ_OK;
  const int64_t warps = (int64_t)rows * ((M + 7) / 8);
  const int64_t blocks = (warps * 32 + 255) / 256;
  qgemv_simt_kernel<ACT><<<blocks, 256, 0, st>>>(P, K, reinterpret_cast<const ACT*>(x), (int)M,
                                                ldx, rows);
  return launch_status();
}

}  // namespace
}  // namespace csaq

using namespace csaq;

extern "C" int64_t csaq_tile_blocks_bytes(int bits, int64_t n_rows, int64_t K) {
  if ((bits != 2 && bits != 4 && bits != 8 && bits != 16) || n_rows < 0 || K <= 0 || K % 128)
    return -1;
  const int64_t tiles = (n_rows + kTileRows - 1) / kTileRows;
  return tiles * (K / 128) * block_bytes(bits);
}

extern "C" int csaq_repack_tiles(const csaq_tier* tier, int64_t K, uint8_t* blocks, void* stream) {
  if (!tier || !blocks || K <= 0 || K % 128) return CSAQ_ERR_ARG;
  const csaq_tier& T = *tier;
  if (T.bits != 2 && T.bits != 4 && T.bits != 8 && T.bits != 16) return CSAQ_ERR_BITS;
  if (T.n_rows < 0 || (T.n_rows > 0 && !T.codes) || T.row_bytes < packed_row_bytes(K, T.bits))
    return CSAQ_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(blocks) % 16) return CSAQ_ERR_ARG;
  if (T.bits != 16) {
    if (!T.scales || !T.zps || T.group_size <= 0 || T.group_size % 128) return CSAQ_ERR_UNSUPPORTED;
    if (T.n_groups < (K + T.group_size - 1) / T.group_size) return CSAQ_ERR_ARG;
  }
  if (T.n_rows == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  const int64_t n_chunks = K / 128;
  const int64_t n_tiles = (T.n_rows + kTileRows - 1) / kTileRows;
  const int piece = T.bits == 2 ? 8 : 16;
  const int64_t pieces = n_tiles * n_chunks * 2 * (4 * T.bits / piece) * 32;
  repack_codes_kernel<<<(pieces + 255) / 256, 256, 0, st>>>(T, n_chunks, T.bits, n_tiles, blocks);
  int rc = launch_status();
  if (rc || T.bits == 16) return rc;
  const int64_t metas = n_tiles * n_chunks * kTileRows;
  repack_meta_kernel<<<(metas + 255) / 256, 256, 0, st>>>(T, n_chunks, T.bits, n_tiles, blocks);
  return launch_status();
}

extern "C" int csaq_qgemv(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x,
                          int x_dtype, int64_t M, int64_t ldx, void* stream) {
  TierParams P;
  int rc = build_params(tiers, n_tiers, K, P);
  if (rc) return rc;
  if (!x || M < 0 || ldx < K || !dtype_size(x_dtype)) return CSAQ_ERR_ARG;
  if (M == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  if (x_dtype != CSAQ_DT_F32 && mma_eligible(P, K, x, ldx)) {
    return x_dtype == CSAQ_DT_BF16 ? launch_mma<__nv_bfloat16>(P, K, x, M, ldx, st)
                                   : launch_mma<__half>(P, K, x, M, ldx, st);
  }
  if (!simt_eligible(P)) return CSAQ_ERR_UNSUPPORTED;
  if (x_dtype == CSAQ_DT_F32) return launch_simt<float>(P, K, x, M, ldx, st);
  return x_dtype == CSAQ_DT_BF16 ? launch_simt<__nv_bfloat16>(P, K, x, M, ldx, st)
                                 : launch_simt<__half>(P, K, x, M, ldx, st);
}

extern "C" int csaq_qgemv_simt(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x,
                               int x_dtype, int64_t M, int64_t ldx, void* stream) {
  TierParams P;
  int rc = build_params(tiers, n_tiers, K, P);
  if (rc) return rc;
  if (!x || M < 0 || ldx < K || !dtype_size(x_dtype)) return CSAQ_ERR_ARG;
  if (M == 0) return CSAQ_OK;
  if (!simt_eligible(P)) return CSAQ_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  if (x_dtype == CSAQ_DT_F32) return launch_simt<float>(P, K, x, M, ldx, st);
  return x_dtype == CSAQ_DT_BF16 ? launch_simt<__nv_bfloat16>(P, K, x, M, ldx, st)
                                 : launch_simt<__half>(P, K, x, M, ldx, st);
}
