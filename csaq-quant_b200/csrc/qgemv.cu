// Mixed-precision quantised linear for decode / verify (small M).
//
// Two kernels share the csaq_tier descriptor.
//
// Tensor-core kernel (qgemv_mma_kernel), reading the GEMV block layout
// (csaq_repack_tiles):
//   * A tier is cut into units of MT 16-row tiles (MT = 2 for 2/4-bit rows,
//     1 for 8/16-bit) and 128-column chunks. The block of one (unit, chunk) is
//     contiguous and holds, tile by tile, the codes that MMA lane
//     (g, c) = (lane / 4, lane % 4) consumes for rows g and g+8 and columns
//     c*32 .. c*32+31, followed by the tile's 16 fp32 scales and 16 uint8 zero
//     points. 8-bit rows are stored as two 4-bit planes (low and high nibbles);
//     fp16 rows are stored pre-arranged in the 4-bit column order (values in
//     "high" positions times 16, exact).
//   * Work = (unit, chunk) items of every tier of the launch, spread over the
//     warps of a one-CTA-per-SM grid of 2-CTA clusters: each cluster takes a
//     run of whole units, cut so the clusters carry equal cost (measured time
//     per item by bit-width), and
//     each of its 32 warps an equal-cost run of items (stream-K). Each warp
//     streams its blocks into a shared-memory ring by bulk copies. A unit
//     whose chunks all fall in one warp's range is finished in registers; a
//     unit cut between warps leaves one partial sum per warp in shared
//     memory, and after a cluster barrier the highest of those warps adds
//     them in warp order, reading the other CTA's through distributed shared
//     memory. The partition depends only on the tier shapes and the SM count,
//     so a token's result is bitwise independent of how many tokens share the
//     launch.
//   * Activations are staged once per CTA as fp16 MMA B-fragments ("records"),
//     scaled per (128-column chunk, token) by a power of two (exact for bf16 /
//     fp16 inputs; the factor is applied to the chunk's partial sum).
//   * Codes become fp16 MMA operands with one LOP3 per register: a nibble
//     OR-ed into the mantissa of 1024.0 gives 1024 + f*q (f = 1 or 16 by the
//     nibble's position; 2-bit codes: 1, 4, 16, 64); the matching record entry
//     is x / f, so each product is (1024 / f + q) * x. Per (chunk, token) the
//     staging pass stores C = sum_k (1024 / f_k) x_k and S = sum_k x_k; a
//     chunk adds s * (g - C - zp * S) to a row (8-bit:
//     s * ((g_lo - C) + 16 (g_hi - C) - zp * S)), g being the MMA sum.
//
// CUDA-core kernel (qgemv_simt_kernel), reading the reference layout: one warp
// per (row, 8-token block), exact fp32 (q - zp) * s per element; any K, any
// group size, fp32 activations too.

#include <algorithm>
#include <mutex>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "tile_blocks.cuh"

namespace csaq {
namespace {

constexpr int kWarps = 16;  // one CTA per SM
constexpr int kThreads = kWarps * 32;
constexpr int kRecStride = 288;  // bytes per (chunk, token) record block: 256 + 32 (bank spread)

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
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  return bits_of<__half>(__float2half_rn(a)) | (bits_of<__half>(__float2half_rn(b)) << 16);
}

// ── repack: reference layout -> GEMV blocks ─────────────────────────────────
// Block of (unit, chunk) at ((unit * n_chunks) + chunk) * chunk_bytes; inside,
// tile mt at mt * tile_block_bytes. Code pieces (16 B; 2-bit: 8 B) of a tile:
//   4-bit : [h][lane]         bytes of row g+8h, columns c*32..+32 (reference nibbles)
//   8-bit : [plane][h][lane]  nibble plane p (q >> 4p) & 15 of those columns
//   16-bit: [h][q][lane]      fp16 of columns c*32+8q..+8 as (w0,w4),(16w1,16w5),(w2,w6),(16w3,16w7)
//   2-bit : [h][lane]         reference bytes (8 B = 32 codes)
__global__ void repack_codes_kernel(const csaq_tier T, int64_t n_chunks, int64_t n_units,
                                    uint8_t* __restrict__ blocks) {
  const int bits = T.bits;
  const int piece = bits == 2 ? 8 : 16;
  const int pieces_per_tile = code_bytes(bits) / piece;
  const int mt_n = unit_tiles(bits);
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t total = n_units * n_chunks * mt_n * pieces_per_tile;
  if (idx >= total) return;
  const int p = (int)(idx % pieces_per_tile);
  int64_t rest = idx / pieces_per_tile;
  const int mt = (int)(rest % mt_n);
  rest /= mt_n;
  const int64_t ch = rest % n_chunks, unit = rest / n_chunks;
  const int lane = p % 32;
  const int g = lane >> 2, c = lane & 3;
  int h, q = 0, plane = 0;
  if (bits == 8) { plane = p / 64; h = (p / 32) % 2; }
  else if (bits == 16) { h = p / 128; q = (p / 32) % 4; }
  else { h = p / 32; }
  const int64_t tile = unit * mt_n + mt;
  const int64_t row = tile * kTileRows + g + 8 * h;
  uint8_t* dst = blocks + (unit * n_chunks + ch) * chunk_bytes(bits) + mt * tile_block_bytes(bits) +
                 (int64_t)p * piece;
  const bool live = row < T.n_rows;
  const int64_t col0 = ch * 128 + c * 32;  // first column of the lane's block
  if (bits == 4 || bits == 2) {
    const uint8_t* src = T.codes + row * T.row_bytes + (ch * 16 * bits) + c * (4 * bits);
    for (int i = 0; i < piece; ++i) dst[i] = live ? src[i] : 0;
  } else if (bits == 8) {
    const uint8_t* src = T.codes + row * T.row_bytes + col0;
    for (int j = 0; j < 16; ++j) {
      uint32_t b = 0;
      if (live) {
        const uint32_t q0 = src[2 * j], q1 = src[2 * j + 1];
        b = ((q0 >> (4 * plane)) & 15u) | (((q1 >> (4 * plane)) & 15u) << 4);
      }
      dst[j] = (uint8_t)b;
    }
  } else {
    const __half* src = reinterpret_cast<const __half*>(T.codes + row * T.row_bytes) + col0 + 8 * q;
    uint16_t* d16 = reinterpret_cast<uint16_t*>(dst);  // 16-byte aligned piece
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = (j >> 1) + 4 * (j & 1);  // column order 0, 4, 1, 5, 2, 6, 3, 7
      float v = live ? __half2float(src[k]) : 0.0f;
      if (k & 1) v = fminf(fmaxf(v * 16.0f, -65504.0f), 65504.0f);  // "high" positions: x16 (exact)
      d16[j] = __half_as_ushort(__float2half_rn(v));
    }
  }
}

__global__ void repack_meta_kernel(const csaq_tier T, int64_t n_chunks, int64_t n_units,
                                   uint8_t* __restrict__ blocks) {
  const int bits = T.bits;
  const int mt_n = unit_tiles(bits);
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n_units * n_chunks * mt_n * kTileRows) return;
  const int r = (int)(idx % kTileRows);
  int64_t rest = idx / kTileRows;
  const int mt = (int)(rest % mt_n);
  rest /= mt_n;
  const int64_t ch = rest % n_chunks, unit = rest / n_chunks;
  const int64_t row = (unit * mt_n + mt) * kTileRows + r;
  const int64_t gi = (T.n_groups > 1) ? (ch * 128) / T.group_size : 0;
  uint8_t* meta = blocks + (unit * n_chunks + ch) * chunk_bytes(bits) + mt * tile_block_bytes(bits) +
                  code_bytes(bits);
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
// R4 (4/8/16-bit tiers), per 32-column lane block, word m = cols 8m..8m+7:
//   [2m] = ((x0,x4),(x1/16,x5/16)), [2m+1] = ((x2,x6),(x3/16,x7/16))
//   C4 = 1024 (x0+x4+x2+x6) + 64 (x1+x5+x3+x7) summed over the chunk
// R2 (2-bit tiers), word m = cols 16m..16m+15, t = 0..3:
//   [4m+t] = ((x_{2t}/f,x_{2t+8}/f),(x_{2t+1}/f',x_{2t+9}/f')), (f,f') = (1,4),(16,64),(1,4),(16,64)
//   C2 = sum (1024 / f) x
__device__ __forceinline__ void build_records(const float (&xv)[32], float inv, bool want2, uint2 (&r4)[8],
                                              uint2 (&r2)[8], float& C4, float& C2, float& S) {
  float v[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = xv[i] * inv;  // exact power-of-two scaling
  float c4 = 0.0f, s = 0.0f;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const float* x = v + 8 * m;
    r4[2 * m] = make_uint2(pack_h2(x[0], x[4]), pack_h2(x[1] * 0.0625f, x[5] * 0.0625f));
    r4[2 * m + 1] = make_uint2(pack_h2(x[2], x[6]), pack_h2(x[3] * 0.0625f, x[7] * 0.0625f));
    c4 += 1024.0f * (x[0] + x[4] + x[2] + x[6]) + 64.0f * (x[1] + x[5] + x[3] + x[7]);
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) s += v[i];
  float c2 = 0.0f;
  if (want2) {
    const float f[4] = {1.0f, 0.0625f, 1.0f, 0.0625f};
    const float f2[4] = {0.25f, 0.015625f, 0.25f, 0.015625f};
    const float cf[4] = {1024.0f, 64.0f, 1024.0f, 64.0f};
    const float cf2[4] = {256.0f, 16.0f, 256.0f, 16.0f};
#pragma unroll
    for (int m = 0; m < 2; ++m)
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float* x = v + 16 * m;
        r2[4 * m + t] = make_uint2(pack_h2(x[2 * t] * f[t], x[2 * t + 8] * f[t]),
                                   pack_h2(x[2 * t + 1] * f2[t], x[2 * t + 9] * f2[t]));
        c2 += cf[t] * (x[2 * t] + x[2 * t + 8]) + cf2[t] * (x[2 * t + 1] + x[2 * t + 9]);
      }
  }
  C4 = c4;
  C2 = c2;
  S = s;
}

// ── MMA over one chunk ──────────────────────────────────────────────────────
constexpr uint32_t kMagic = 0x64006400u;  // fp16 1024.0 in both halves

// 4-bit (or two 8-bit nibble planes) for two tiles: g[tile][acc], the two
// accumulators of a tile alternate k-steps
__device__ __forceinline__ void mma4(const uint32_t (&cw)[2][2][4], const uint2 (&rec)[8],
                                     float (&g)[2][2][4]) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    uint32_t v[2][2][4];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint32_t w = cw[mt][r][m], t = w >> 8;
        v[mt][r][0] = lop_and_or(w, 0x000F000Fu, kMagic);  // 1024 + q   (cols 0, 4)
        v[mt][r][1] = lop_and_or(w, 0x00F000F0u, kMagic);  // 1024 + 16q (cols 1, 5)
        v[mt][r][2] = lop_and_or(t, 0x000F000Fu, kMagic);  //             (cols 2, 6)
        v[mt][r][3] = lop_and_or(t, 0x00F000F0u, kMagic);  //             (cols 3, 7)
      }
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
      mma_f16(g[mt][0], v[mt][0][0], v[mt][1][0], v[mt][0][1], v[mt][1][1], rec[2 * m].x, rec[2 * m].y);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
      mma_f16(g[mt][1], v[mt][0][2], v[mt][1][2], v[mt][0][3], v[mt][1][3], rec[2 * m + 1].x, rec[2 * m + 1].y);
  }
}

// 2-bit, two tiles
__device__ __forceinline__ void mma2(const uint32_t (&cw)[2][2][2], const uint2 (&rec)[8],
                                     float (&g)[2][2][4]) {
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    uint32_t v[2][2][8];
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint32_t w = cw[mt][r][m], t = w >> 8;
        v[mt][r][0] = lop_and_or(w, 0x00030003u, kMagic);
        v[mt][r][1] = lop_and_or(w, 0x000C000Cu, kMagic);
        v[mt][r][2] = lop_and_or(w, 0x00300030u, kMagic);
        v[mt][r][3] = lop_and_or(w, 0x00C000C0u, kMagic);
        v[mt][r][4] = lop_and_or(t, 0x00030003u, kMagic);
        v[mt][r][5] = lop_and_or(t, 0x000C000Cu, kMagic);
        v[mt][r][6] = lop_and_or(t, 0x00300030u, kMagic);
        v[mt][r][7] = lop_and_or(t, 0x00C000C0u, kMagic);
      }
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
        mma_f16(g[mt][t & 1], v[mt][0][2 * t], v[mt][1][2 * t], v[mt][0][2 * t + 1], v[mt][1][2 * t + 1],
                rec[4 * m + t].x, rec[4 * m + t].y);
  }
}

// 16-bit (pre-arranged fp16): words [4m], [4m+1] with rec[2m]; [4m+2], [4m+3] with rec[2m+1]
__device__ __forceinline__ void mma16(const uint32_t (&cw)[2][16], const uint2 (&rec)[8], float (&g)[2][4]) {
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    mma_f16(g[0], cw[0][4 * m], cw[1][4 * m], cw[0][4 * m + 1], cw[1][4 * m + 1], rec[2 * m].x, rec[2 * m].y);
    mma_f16(g[1], cw[0][4 * m + 2], cw[1][4 * m + 2], cw[0][4 * m + 3], cw[1][4 * m + 3], rec[2 * m + 1].x,
            rec[2 * m + 1].y);
  }
}

// ── kernel parameters ───────────────────────────────────────────────────────
// Work items are (unit, chunk) pairs, numbered tier by tier and unit-major, so
// a run of items is a run of consecutive GEMV blocks. Warp w owns items
// [begin[w], begin[w + 1]); the host cuts the items into runs of equal block
// bytes. The cut depends only on the tier shapes and the SM count, never on
// M, so neither does any partial sum.
constexpr int kMaxCtas = 160;
constexpr int kMaxWarps = kMaxCtas * 16;

struct TierWork {
  int bits, mt, n_units;
  int item0;    // first item of the tier
  int n_items;  // n_units * n_chunks
};

struct KParams {
  TierParams tp;
  TierWork w[CSAQ_MAX_TIERS];
  int n_items_total;
  int n_warps;     // W = gridDim.x * kWarps
  int slot_bytes;  // ring slot: the largest chunk_bytes of the launch
  int depth;       // ring slots per warp
  int want2;       // any 2-bit tier (stage R2 records)
  int x_bytes;     // R4 records: n_rec * M * kRecStride (R2 the same again when want2)
  int split;       // records split by chunk between the cluster's CTAs (they do not fit one)
  int ch_half;     // split: CTA rank 0 holds chunks [0, ch_half), rank 1 the rest
  uint32_t silu_tiers;  // bit i: tier i stores dtype(silu(y))
  const void* x_mul;   // nullable: the input is dtype(x * x_mul), rows ldx apart
  int begin[kMaxWarps + 1];
};

__device__ __forceinline__ int tier_of_item(const KParams& P, int item) {
  int t = 0;
  while (t + 1 < P.tp.n_tiers && item >= P.w[t + 1].item0) ++t;
  return t;
}

// a value the compiler must have in a register at this point of the program
// (so a load is issued here, not sunk past the barriers that follow)
template <typename V>
__device__ __forceinline__ V pin(V v) {
  static_assert(sizeof(V) == 4 || sizeof(V) == 8, "pin: 4 or 8 bytes");
  if constexpr (sizeof(V) == 8) {
    uint64_t u;
    memcpy(&u, &v, 8);
    asm volatile("mov.b64 %0, %0;" : "+l"(u));
    memcpy(&v, &u, 8);
  } else {
    uint32_t u;
    memcpy(&u, &v, 4);
    asm volatile("mov.b32 %0, %0;" : "+r"(u));
    memcpy(&v, &u, 4);
  }
  return v;
}

// the fields of a tier that writing y needs
struct OutDesc {
  const int32_t* out_rows;
  const void* bias;
  const void* residual;
  void* y;
  int64_t ldy, ldr;
  int n_rows;
};

CSAQ_GUARD_RECORD()

// The stored value: dtype(v), or for a gate tier the SiLU of it as the
// separate gate kernel computes it, g = float(dtype(v)), dtype(g / (1 +
// exp(-g))) (silu_mul_kernel, runtime.cu).
template <typename ACT>
__device__ __forceinline__ ACT out_value(float v, bool silu) {
  if (silu) {
    const float g = to_f32<ACT>(from_f32<ACT>(v));
    v = g / (1.0f + __expf(-g));
  }
  return from_f32<ACT>(v);
}

template <typename ACT, typename TD>
__device__ __forceinline__ void store_out(const TD& T, int row, int tok, float v, float xe, bool silu) {
  v = __fmul_rn(v, xe);
  const int orow = T.out_rows[row];
  if (!CSAQ_GUARD(orow >= 0 && orow < T.ldy && (!T.residual || orow < T.ldr), CSAQ_GUARD_GEMV_OUT_ROW, orow,
                  T.ldy))
    return;
  if (T.bias) v = __fadd_rn(v, to_f32<ACT>(reinterpret_cast<const ACT*>(T.bias)[orow]));
  if (T.residual)
    v = __fadd_rn(v, to_f32<ACT>(reinterpret_cast<const ACT*>(T.residual)[(int64_t)tok * T.ldr + orow]));
  reinterpret_cast<ACT*>(T.y)[(int64_t)tok * T.ldy + orow] = out_value<ACT>(v, silu);
}

// ── bulk copies into the per-warp ring (one elected lane; no multicast) ────
constexpr int kWaitLimit = 1 << 20;  // try_wait rounds before a wait is abandoned
__device__ unsigned int g_wait_timeouts;

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n\tfence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait for the phase with the given parity; false when abandoned
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// ── thread-block cluster helpers (distributed shared memory) ────────────────
constexpr int kCluster = 2;  // CTAs per cluster: a unit's partial sums never leave its cluster

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the two halves of cluster_sync; `dep` is an unused operand that orders the
// arrive after the computation of its value
__device__ __forceinline__ void cluster_arrive_after(float dep) {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::"f"(dep) : "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the shared::cluster address of `saddr` (a local shared address) in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t saddr, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// A load of data that no thread writes any more (after a cluster barrier):
// not volatile, so that independent loads are issued back to back. It stays
// after the barrier because its address comes from mapa, which is volatile.
__device__ __forceinline__ float ld_dsmem_f32_after_sync(uint32_t addr) {
  float v;
  asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

// One 128-column chunk of one unit: acc[tile][n-tile][fragment] += the chunk's
// contribution (see the header comment for the algebra).
// DS: the chunk's records and (C, S) live in the other CTA of the cluster
// (or this one) and are read through distributed shared memory at the
// shared::cluster addresses rb_cl and xcs_cl; otherwise at rbase and xcs_ch.
template <int BITS, int NT, bool DS>
__device__ __forceinline__ void chunk_math(const uint8_t* slot, const uint8_t* rbase,
                                           const float4* xcs_ch, uint32_t rb_cl, uint32_t xcs_cl, int M,
                                           int lane, float (&acc)[2][NT][4]) {
  constexpr int bits = BITS;
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int tok = nt * 8 + g;
    uint2 rec[8];
    if (tok < M) {
      if constexpr (DS) {
        const uint32_t ra = rb_cl + (uint32_t)(tok * kRecStride + 8 * c);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          asm volatile("ld.shared::cluster.v2.u32 {%0, %1}, [%2];"
                       : "=r"(rec[q].x), "=r"(rec[q].y)
                       : "r"(ra + 32u * q));
      } else {
        const uint2* rp = reinterpret_cast<const uint2*>(rbase + tok * kRecStride) + c;
#pragma unroll
        for (int q = 0; q < 8; ++q) rec[q] = rp[4 * q];
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) rec[q] = make_uint2(0u, 0u);
    }
    const int t0 = nt * 8 + 2 * c;
    float4 cs0 = make_float4(0.f, 0.f, 0.f, 0.f), cs1 = make_float4(0.f, 0.f, 0.f, 0.f);
    if constexpr (DS) {
      if (t0 < M)
        asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(cs0.x), "=f"(cs0.y), "=f"(cs0.z), "=f"(cs0.w)
                     : "r"(xcs_cl + 16u * t0));
      if (t0 + 1 < M)
        asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(cs1.x), "=f"(cs1.y), "=f"(cs1.z), "=f"(cs1.w)
                     : "r"(xcs_cl + 16u * (t0 + 1)));
    } else {
      if (t0 < M) cs0 = xcs_ch[t0];
      if (t0 + 1 < M) cs1 = xcs_ch[t0 + 1];
    }
    if constexpr (bits == 4 || bits == 8) {
      // 4-bit: [tile][h][word]; 8-bit: [nibble plane][h][word] of one tile
      uint32_t cw[2][2][4];
      float gg[2][2][4];
      const int sub = bits == 4 ? tile_block_bytes(4) : 1024;
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint4* cp = reinterpret_cast<const uint4*>(slot + mt * sub);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint4 v = cp[h * 32 + lane];
          cw[mt][h][0] = v.x; cw[mt][h][1] = v.y; cw[mt][h][2] = v.z; cw[mt][h][3] = v.w;
        }
#pragma unroll
        for (int a = 0; a < 2; ++a) gg[mt][a][0] = gg[mt][a][1] = gg[mt][a][2] = gg[mt][a][3] = 0.0f;
      }
      mma4(cw, rec, gg);
      if constexpr (bits == 4) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          const uint8_t* meta = slot + mt * tile_block_bytes(4) + code_bytes(4);
          const float s0 = reinterpret_cast<const float*>(meta)[g], s1 = reinterpret_cast<const float*>(meta)[g + 8];
          const float z0 = (float)meta[64 + g], z1 = (float)meta[64 + g + 8];
          const float d0 = gg[mt][0][0] + gg[mt][1][0], d1 = gg[mt][0][1] + gg[mt][1][1];
          const float d2 = gg[mt][0][2] + gg[mt][1][2], d3 = gg[mt][0][3] + gg[mt][1][3];
          acc[mt][nt][0] = fmaf(s0 * cs0.w, fmaf(-z0, cs0.y, d0 - cs0.x), acc[mt][nt][0]);
          acc[mt][nt][1] = fmaf(s0 * cs1.w, fmaf(-z0, cs1.y, d1 - cs1.x), acc[mt][nt][1]);
          acc[mt][nt][2] = fmaf(s1 * cs0.w, fmaf(-z1, cs0.y, d2 - cs0.x), acc[mt][nt][2]);
          acc[mt][nt][3] = fmaf(s1 * cs1.w, fmaf(-z1, cs1.y, d3 - cs1.x), acc[mt][nt][3]);
        }
      } else {
        const uint8_t* meta = slot + code_bytes(8);
        const float s0 = reinterpret_cast<const float*>(meta)[g], s1 = reinterpret_cast<const float*>(meta)[g + 8];
        const float z0 = (float)meta[64 + g], z1 = (float)meta[64 + g + 8];
        float d[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = gg[0][0][e] + gg[0][1][e], hi = gg[1][0][e] + gg[1][1][e];
          const float C = (e & 1) ? cs1.x : cs0.x;
          d[e] = fmaf(16.0f, hi - C, lo - C);
        }
        acc[0][nt][0] = fmaf(s0 * cs0.w, fmaf(-z0, cs0.y, d[0]), acc[0][nt][0]);
        acc[0][nt][1] = fmaf(s0 * cs1.w, fmaf(-z0, cs1.y, d[1]), acc[0][nt][1]);
        acc[0][nt][2] = fmaf(s1 * cs0.w, fmaf(-z1, cs0.y, d[2]), acc[0][nt][2]);
        acc[0][nt][3] = fmaf(s1 * cs1.w, fmaf(-z1, cs1.y, d[3]), acc[0][nt][3]);
      }
    } else if constexpr (bits == 16) {
      uint32_t cw[2][16];
      float gg[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const uint4* cp = reinterpret_cast<const uint4*>(slot);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 v = cp[(h * 4 + q) * 32 + lane];
          cw[h][4 * q] = v.x; cw[h][4 * q + 1] = v.y; cw[h][4 * q + 2] = v.z; cw[h][4 * q + 3] = v.w;
        }
      mma16(cw, rec, gg);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[0][nt][e] = fmaf(gg[0][e] + gg[1][e], (e & 1) ? cs1.w : cs0.w, acc[0][nt][e]);
    } else {  // 2-bit
      uint32_t cw[2][2][2];
      float gg[2][2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint2* cp = reinterpret_cast<const uint2*>(slot + mt * tile_block_bytes(2));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint2 v = cp[h * 32 + lane];
          cw[mt][h][0] = v.x; cw[mt][h][1] = v.y;
        }
#pragma unroll
        for (int a = 0; a < 2; ++a) gg[mt][a][0] = gg[mt][a][1] = gg[mt][a][2] = gg[mt][a][3] = 0.0f;
      }
      mma2(cw, rec, gg);
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        const uint8_t* meta = slot + mt * tile_block_bytes(2) + code_bytes(2);
        const float s0 = reinterpret_cast<const float*>(meta)[g], s1 = reinterpret_cast<const float*>(meta)[g + 8];
        const float z0 = (float)meta[64 + g], z1 = (float)meta[64 + g + 8];
        const float d0 = gg[mt][0][0] + gg[mt][1][0], d1 = gg[mt][0][1] + gg[mt][1][1];
        const float d2 = gg[mt][0][2] + gg[mt][1][2], d3 = gg[mt][0][3] + gg[mt][1][3];
        acc[mt][nt][0] = fmaf(s0 * cs0.w, fmaf(-z0, cs0.y, d0 - cs0.z), acc[mt][nt][0]);
        acc[mt][nt][1] = fmaf(s0 * cs1.w, fmaf(-z0, cs1.y, d1 - cs1.z), acc[mt][nt][1]);
        acc[mt][nt][2] = fmaf(s1 * cs0.w, fmaf(-z1, cs0.y, d2 - cs0.z), acc[mt][nt][2]);
        acc[mt][nt][3] = fmaf(s1 * cs1.w, fmaf(-z1, cs1.y, d3 - cs1.z), acc[mt][nt][3]);
      }
    }
  }
}

// fragment (tile mt, n-tile nt, element e) -> (row in unit, token)
__device__ __forceinline__ int frag_row(int mt, int e, int lane) { return mt * kTileRows + (lane >> 2) + ((e >> 1) << 3); }
__device__ __forceinline__ int frag_tok(int nt, int e, int lane) { return nt * 8 + 2 * (lane & 3) + (e & 1); }

// a unit of the launch, addressed by tier and index within the tier
struct UnitRef {
  int t, unit, start, end;  // items [start, end)
};

template <typename ACT, int NT, bool SPLIT>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads, 1)
    qgemv_mma_kernel(const __grid_constant__ KParams P,
                                                                int64_t K, const ACT* __restrict__ x,
                                                                int M, int64_t ldx) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_chunks = (int)(K / 128);

  uint8_t* rec4 = smem;                                          // [ch][tok] x kRecStride
  uint8_t* rec2 = smem + P.x_bytes;                              // same layout, 2-bit records
  float4* xcs = reinterpret_cast<float4*>(smem + (P.want2 ? 2 : 1) * P.x_bytes);  // [ch][tok] (C4, S, C2, -)
  const int n_rec = SPLIT ? P.ch_half : n_chunks;                // chunks of records held here
  float* xexp = reinterpret_cast<float*>(xcs + n_rec * M);       // [16] 2^e per token
  uint64_t* bars = reinterpret_cast<uint64_t*>(xexp + 16) + warp * 8;  // [warp][8] ring barriers
  uint8_t* ring_all = reinterpret_cast<uint8_t*>(xexp + 16) + kWarps * 8 * sizeof(uint64_t);
  uint8_t* ring = ring_all + (size_t)warp * P.depth * P.slot_bytes;

  const int wg = blockIdx.x * kWarps + warp;
  const int it_begin = P.begin[wg];
  const int it_end = P.begin[wg + 1];

  pdl_trigger();
  if (lane == 0) {
    for (int s = 0; s < P.depth; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
  }
  __syncwarp();

  // issue cursor: walks the warp's items (consecutive blocks of each tier)
  int i_left = it_end - it_begin, i_local = 0;
  int i_t = 0, i_slot = 0;
  // the current tier's fields, reloaded from the kernel parameters only when
  // the cursor enters another tier (indexed parameter loads miss the constant cache)
  const uint8_t* i_blocks = nullptr;
  int i_cb = 0, i_n = 0;
  auto enter_tier = [&]() {
    i_blocks = P.tp.t[i_t].blocks;
    i_cb = chunk_bytes(P.w[i_t].bits);
    i_n = P.w[i_t].n_items;
  };
  const int slot_bytes = P.slot_bytes, depth = P.depth;
  if (i_left > 0) {
    i_t = tier_of_item(P, it_begin);
    i_local = it_begin - P.w[i_t].item0;
    enter_tier();
  }
  auto issue = [&]() {
    if (i_left > 0) {
      if (lane == 0) {
        mbar_expect_tx(&bars[i_slot], (uint32_t)i_cb);
        bulk_load(ring + i_slot * slot_bytes, i_blocks + (int64_t)i_local * i_cb, (uint32_t)i_cb, &bars[i_slot]);
      }
      --i_left;
      if (++i_local == i_n) {
        i_local = 0;
        do { ++i_t; } while (i_left > 0 && P.w[i_t].n_items == 0);
        if (i_left > 0) enter_tier();
      }
      i_slot = (i_slot + 1 == depth) ? 0 : i_slot + 1;
    }
  };
  for (int d = 0; d < P.depth; ++d) issue();  // weights first: no kernel writes them
  pdl_wait();  // x (and y, bias, residual) may come from the previous kernel of the stream

  // the power-of-two scales are per (chunk, token): no pass over x before
  // the records; the output factor is applied per chunk in the main loop
  if (threadIdx.x < 16) xexp[threadIdx.x] = 1.0f;

  // activation records (whole warps iterate: 4-lane shuffles); split: this
  // CTA builds and holds the records of its own chunk half only
  const int rank = (int)(blockIdx.x % kCluster);
  const int c_lo = SPLIT ? rank * P.ch_half : 0;
  const int n_loc = SPLIT ? (rank == 0 ? P.ch_half : n_chunks - P.ch_half) : n_chunks;
  const int n_st = M * n_loc * 4;
  const bool gated = P.x_mul != nullptr;
  for (int base = 0; base < n_st; base += blockDim.x) {
    const int u = base + threadIdx.x;
    const bool live = u < n_st;
    const int cc = u & 3, rest = u >> 2;
    const int tok = live ? rest % M : 0, li = live ? rest / M : 0, ch = c_lo + li;
    uint2 r4[8], r2[8];
    float C4 = 0.0f, C2 = 0.0f, S = 0.0f;
    // this lane's 32 columns, then the chunk's scale 2^e (max|x| * 2^-e in
    // [2^14, 2^15), exact for bf16/fp16) from the 4 lanes of the (chunk, token)
    float xv[32];
    float mx = 0.0f;
    const int64_t xo = (int64_t)tok * ldx + ch * 128 + cc * 32;
    uint4 q[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) q[i] = live ? ld_cached_v4(x + xo + 8 * i) : make_uint4(0u, 0u, 0u, 0u);
    if (gated) {  // h = dtype(g' * u), as silu_mul_kernel stores it
      const ACT* xm = reinterpret_cast<const ACT*>(P.x_mul);
      uint4 q2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) q2[i] = live ? ld_cached_v4(xm + xo + 8 * i) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ACT* e = reinterpret_cast<ACT*>(&q[i]);
        const ACT* e2 = reinterpret_cast<const ACT*>(&q2[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = from_f32<ACT>(to_f32<ACT>(e[j]) * to_f32<ACT>(e2[j]));
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const ACT* e = reinterpret_cast<const ACT*>(&q[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        xv[8 * i + j] = to_f32<ACT>(e[j]);
        mx = fmaxf(mx, fabsf(xv[8 * i + j]));
      }
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const uint32_t mb = __float_as_uint(mx);
    const int E = mb == 0u ? 14 : (int)((mb >> 23) & 0xFF) - 127;
    const float fac = ldexpf(1.0f, E - 14);
    if (live) build_records(xv, 1.0f / fac, P.want2 != 0, r4, r2, C4, C2, S);
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      C4 += __shfl_xor_sync(0xffffffffu, C4, o);
      C2 += __shfl_xor_sync(0xffffffffu, C2, o);
      S += __shfl_xor_sync(0xffffffffu, S, o);
    }
    if (live) {
      uint2* d4 = reinterpret_cast<uint2*>(rec4 + ((int64_t)li * M + tok) * kRecStride) + cc;
#pragma unroll
      for (int j = 0; j < 8; ++j) d4[4 * j] = r4[j];
      if (P.want2) {
        uint2* d2 = reinterpret_cast<uint2*>(rec2 + ((int64_t)li * M + tok) * kRecStride) + cc;
#pragma unroll
        for (int j = 0; j < 8; ++j) d2[4 * j] = r2[j];
      }
      if (cc == 0) xcs[li * M + tok] = make_float4(C4, S, C2, fac);
    }
  }
  if constexpr (SPLIT)
    cluster_sync();  // both halves of the records are written and visible
  else
    __syncthreads();

  // ── main loop over the warp's units ──────────────────────────────────────
  float acc[2][NT][4], fst[2][NT][4];
  // cut units of this warp: [0] its first unit, [1] its last one (tier -1: none)
  int cut_t0 = -1, cut_u0 = 0, cut_s0 = 0, cut_t1 = -1, cut_u1 = 0, cut_s1 = 0;
  uint32_t phase = 0;                                  // parity bit per ring slot
  uint32_t late = 0, late_parity = 0;                 // slots whose wait was abandoned
  int c_slot = 0;
  int item = it_begin, local = 0, t = 0;
  if (item < it_end) {
    t = tier_of_item(P, item);
    local = item - P.w[t].item0;
  }
  auto chunks = [&](auto bits_c, int ch_first, int ch_last) {
    constexpr int B = decltype(bits_c)::value;
    for (int ch = ch_first; ch < ch_last; ++ch) {
      if (!mbar_wait(&bars[c_slot], (phase >> c_slot) & 1u)) {
        late |= 1u << c_slot;
        late_parity = (late_parity & ~(1u << c_slot)) | (phase & (1u << c_slot));
      }
      phase ^= 1u << c_slot;
      if constexpr (SPLIT) {
        const int r = ch >= P.ch_half ? 1 : 0, li = ch - r * P.ch_half;
        const uint32_t rb = dsmem_addr(smem_u32((B == 2 ? rec2 : rec4) + (int64_t)li * M * kRecStride), r);
        const uint32_t xb = dsmem_addr(smem_u32(xcs + li * M), r);
        chunk_math<B, NT, true>(ring + c_slot * P.slot_bytes, nullptr, nullptr, rb, xb, M, lane, acc);
      } else {
        chunk_math<B, NT, false>(ring + c_slot * P.slot_bytes, (B == 2 ? rec2 : rec4) + (int64_t)ch * M * kRecStride,
                                 xcs + ch * M, 0u, 0u, M, lane, acc);
      }
      __syncwarp();
      issue();
      c_slot = (c_slot + 1 == P.depth) ? 0 : c_slot + 1;
    }
  };
  // the current tier's work fields, reloaded only at tier boundaries
  int c_bits = 0, c_mt = 0, c_item0 = 0, c_n = 0;
  auto enter_ctier = [&]() {
    c_bits = P.w[t].bits;
    c_mt = P.w[t].mt;
    c_item0 = P.w[t].item0;
    c_n = P.w[t].n_items;
  };
  if (item < it_end) enter_ctier();
  while (item < it_end) {
    const int unit = local / n_chunks;
    const int ch_first = local - unit * n_chunks;
    const int room = it_end - item;
    const int ch_last = room < n_chunks - ch_first ? ch_first + room : n_chunks;
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[a][nt][0] = acc[a][nt][1] = acc[a][nt][2] = acc[a][nt][3] = 0.0f;
    switch (c_bits) {
      case 4: chunks(std::integral_constant<int, 4>(), ch_first, ch_last); break;
      case 8: chunks(std::integral_constant<int, 8>(), ch_first, ch_last); break;
      case 16: chunks(std::integral_constant<int, 16>(), ch_first, ch_last); break;
      default: chunks(std::integral_constant<int, 2>(), ch_first, ch_last); break;
    }

    const int u_start = c_item0 + unit * n_chunks;
    if (ch_first == 0 && ch_last == n_chunks) {
      // the whole unit is in this warp: write y from the fragments
      const csaq_tier& T = P.tp.t[t];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int row = unit * c_mt * kTileRows + frag_row(mt, e, lane), tok = frag_tok(nt, e, lane);
            if (mt < c_mt && tok < M && row < T.n_rows) store_out<ACT>(T, row, tok, acc[mt][nt][e], xexp[tok], (P.silu_tiers >> t) & 1u);
          }
    } else if (item == it_begin) {
      cut_t0 = t; cut_u0 = unit; cut_s0 = u_start;
#pragma unroll
      for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) fst[a][nt][e] = acc[a][nt][e];
    } else {
      cut_t1 = t; cut_u1 = unit; cut_s1 = u_start;  // the last unit: stays in acc
    }

    item += ch_last - ch_first;
    local += ch_last - ch_first;
    if (local == c_n) {
      local = 0;
      do { ++t; } while (item < it_end && P.w[t].n_items == 0);
      if (item < it_end) enter_ctier();
    }
  }
  // What the tail needs from the kernel parameters, read now (loads with a
  // warp-dependent index miss the constant cache; their latency overlaps the
  // barriers below instead of following them): the cluster's range starts
  // and the output description of the warp's first unit.
  const int cl_base = wg - (wg & 31);
  const int b_lane = pin(P.begin[cl_base + lane]), b_end = pin(P.begin[cl_base + 32]);
  const int t_own = cut_t0 >= 0 ? cut_t0 : 0;
  const int own_rows = pin(P.w[t_own].mt) * kTileRows;
  const bool own_silu = (P.silu_tiers >> t_own) & 1u;
  OutDesc od;
  od.out_rows = pin(P.tp.t[t_own].out_rows);
  od.bias = pin(P.tp.t[t_own].bias);
  od.residual = pin(P.tp.t[t_own].residual);
  od.y = pin(P.tp.t[t_own].y);
  od.ldy = pin(P.tp.t[t_own].ldy);
  od.ldr = pin(P.tp.t[t_own].ldr);
  od.n_rows = pin(P.tp.t[t_own].n_rows);
  if (late) {
    if (lane == 0) atomicAdd(&g_wait_timeouts, 1u);
    // let the abandoned copies land (again bounded) before shared memory is reused
    for (int s = 0; s < P.depth; ++s)
      if (late & (1u << s)) mbar_wait(&bars[s], (late_parity >> s) & 1u);
  }

  // ── cut units: partials of the cluster's warps meet in distributed shared memory
  __syncthreads();  // every ring of this CTA is drained
  float* part = reinterpret_cast<float*>(ring_all);  // [warp][2][32 rows][M]
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int ct = s == 0 ? cut_t0 : cut_t1;
    if (ct < 0) continue;
    float* dst = part + (warp * 2 + s) * 32 * M;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = frag_tok(nt, e, lane);
          if (mt < P.w[ct].mt && tok < M)
            dst[frag_row(mt, e, lane) * M + tok] = s == 0 ? fst[mt][nt][e] : acc[mt][nt][e];
        }
  }
  cluster_sync();  // partials of both CTAs written and visible

  const uint32_t part_sa = smem_u32(part);
  // the range starts of this cluster's 32 warps, lane l holding warp
  // cl_base + l's (kernel-parameter loads with a varying index are slow):
  // begin[w] of any warp of the cluster is one shuffle away
  static_assert(kWarps * kCluster == 32, "one lane per warp of a cluster");
  auto begin_of = [&](int w) {  // w in [cl_base, cl_base + 32]
    const int v = __shfl_sync(0xffffffffu, b_lane, (w - cl_base) & 31);
    return w - cl_base == 32 ? b_end : v;
  };
  // Only a warp's first unit can be one it finishes: its last unit, when cut,
  // continues in a higher warp. The finishing (highest) warp of a cut unit
  // adds the partials in warp order and writes y.
  const int u_start = cut_s0, u_end = cut_s0 + n_chunks;
  const bool own = cut_t0 >= 0 && begin_of(wg + 1) >= u_end;  // units never cross a cluster boundary
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = 0.0f;
  int nv = 0, n_val = 0, rows = 0;
  if (own) {
    rows = own_rows;
    n_val = rows * M;
    nv = (n_val + 31) >> 5;  // values per lane: e = lane + 32 j
    // first warp holding part of the unit: the last of the cluster with begin <= u_start
    const int w_first = cl_base + 31 - __clz(__ballot_sync(0xffffffffu, b_lane <= u_start));
    // eight warps' partials at a time: their loads are issued together and
    // added in warp order afterwards
    for (int w0 = w_first; w0 <= wg; w0 += 8) {
      uint32_t src[8];
      bool ok[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int w = w0 + q;
        const int bw = begin_of(w <= wg ? w : wg), bw1 = begin_of(w <= wg ? w + 1 : wg + 1);
        ok[q] = w <= wg && bw != bw1;  // skip empty ranges
        const uint32_t off = ok[q] ? (uint32_t)((((w % kWarps) * 2 + (bw >= u_start ? 0 : 1)) * 32 * M) * 4) : 0u;
        src[q] = ok[q] ? dsmem_addr(part_sa + off, (w / kWarps) % kCluster) : 0u;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j >= nv) break;
        const int e = lane + 32 * j;
        if (e >= n_val) continue;
        float a[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) a[q] = ok[q] ? ld_dsmem_f32_after_sync(src[q] + 4u * (uint32_t)e) : 0.0f;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          if (ok[q]) v[j] += a[q];
      }
    }
  }
  // This warp reads no more of the peer's shared memory: arrive now and wait
  // only before leaving, so the stores below overlap the barrier. The sum of
  // the partials is an operand of the arrive, which keeps every load before it.
  float dep = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) dep += v[j];
  cluster_arrive_after(dep);
  if (own) {
    const int unit = cut_u0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (j >= nv) break;
      const int e = lane + 32 * j, r = e / M, tok = e - r * M, row = unit * rows + r;
      if (e < n_val && row < od.n_rows) store_out<ACT>(od, row, tok, v[j], xexp[tok], own_silu);
    }
  }
  cluster_wait();  // no CTA leaves while the other may still read its partials
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
  pdl_wait();
  pdl_trigger();
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
    const int orow = tok < M ? T.out_rows[row] : 0;
    if (tok < M && CSAQ_GUARD(orow >= 0 && orow < T.ldy && (!T.residual || orow < T.ldr), CSAQ_GUARD_GEMV_OUT_ROW,
                              orow, T.ldy)) {
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
constexpr int kRingBudget = 12 * 1024;  // bytes of weights in flight per warp (target)

// CTAs of the grid at most: the SM count, capped, a multiple of the cluster size
int grid_ctas_max() {
  const int n = num_sms() < kMaxCtas ? num_sms() : kMaxCtas;
  return n / kCluster * kCluster > 0 ? n / kCluster * kCluster : kCluster;
}

// Fill the per-tier work table; -1 when the launch has more work items than
// the kernel indexes.
int64_t work_table(const TierParams& TP, int64_t K, TierWork* w) {
  const int64_t n_chunks = K / 128;
  int64_t items = 0;
  for (int i = 0; i < TP.n_tiers; ++i) {
    const csaq_tier& t = TP.t[i];
    const int mt = unit_tiles(t.bits);
    const int64_t tiles = ((int64_t)t.n_rows + kTileRows - 1) / kTileRows;
    const int64_t units = (tiles + mt - 1) / mt;
    w[i].bits = t.bits;
    w[i].mt = mt;
    w[i].n_units = (int)units;
    w[i].item0 = (int)items;
    w[i].n_items = (int)(units * n_chunks);
    items += units * n_chunks;
  }
  return items >= (int64_t)1 << 30 ? -1 : items;
}

// The partition, cached per shape. Cluster j (kCluster CTAs) takes the units
// between two unit boundaries, chosen nearest to the cost targets C j / G, so
// that no unit leaves its cluster; inside a cluster its kCluster * kWarps
// warps take runs of equal cost, cut at chunk granularity (item start cost >=
// the warp's target). Costs are item_cost() per item.
struct PartitionCache {
  struct Entry {
    std::vector<int> key;
    std::vector<int> begin;
  };
  std::mutex mu;
  std::vector<Entry> entries;
  size_t next = 0;
};

// Relative time of one item (a unit's 128-column chunk) by bit-width, as
// measured on B200 with every warp streaming: a 16-bit item (16 rows, 4 KB)
// takes about 0.8 of a 4-bit item (32 rows, 2.2 KB), an 8-bit one (16 rows as
// two nibble planes) about as long as a 4-bit one. Warps streaming fp16 rows
// finish early when items are costed by bytes.
int64_t item_cost(int bits) { return bits == 16 ? 82 : (bits == 8 ? 100 : 100); }

bool partition(const TierParams& TP, const TierWork* w, int64_t K, int n_warps, int* begin) {
  static PartitionCache cache;
  std::vector<int> key;
  key.reserve(4 + 2 * TP.n_tiers);
  key.push_back((int)(K / 128));
  key.push_back(n_warps);
  key.push_back(TP.n_tiers);
  for (int i = 0; i < TP.n_tiers; ++i) {
    key.push_back(TP.t[i].bits);
    key.push_back(TP.t[i].n_rows);
  }
  std::lock_guard<std::mutex> lock(cache.mu);
  for (const auto& e : cache.entries)
    if (e.key == key) {
      std::copy(e.begin.begin(), e.begin.end(), begin);
      return true;
    }
  const int n_tiers = TP.n_tiers;
  const int64_t n_chunks = K / 128;
  std::vector<int64_t> ic(n_tiers), cost0(n_tiers + 1);
  cost0[0] = 0;
  for (int i = 0; i < n_tiers; ++i) {
    ic[i] = item_cost(w[i].bits);
    cost0[i + 1] = cost0[i] + ic[i] * w[i].n_items;
  }
  const int64_t total = cost0[n_tiers];
  const int n_items = w[n_tiers - 1].item0 + w[n_tiers - 1].n_items;
  auto cost_at = [&](int item) -> int64_t {  // start cost of an item (or the end)
    int t = 0;
    while (t + 1 < n_tiers && item >= w[t + 1].item0) ++t;
    return cost0[t] + ic[t] * (item - w[t].item0);
  };
  // first item whose start cost is >= target, within [lo, hi]
  auto first_at = [&](int64_t target, int lo, int hi) -> int {
    while (lo < hi) {
      const int mid = lo + (hi - lo) / 2;
      if (cost_at(mid) >= target) hi = mid; else lo = mid + 1;
    }
    return lo;
  };
  const int n_clusters = n_warps / (kWarps * kCluster);
  const int per_cluster = kWarps * kCluster;
  std::vector<int> cb(n_clusters + 1);
  cb[0] = 0;
  cb[n_clusters] = n_items;
  for (int j = 1; j < n_clusters; ++j) {
    const int64_t target = total * j / n_clusters;
    int t = 0;
    while (t + 1 < n_tiers && target >= cost0[t + 1]) ++t;
    const int64_t unit_cost = ic[t] * n_chunks;
    int64_t u = unit_cost > 0 ? (target - cost0[t] + unit_cost / 2) / unit_cost : 0;
    if (u > w[t].n_units) u = w[t].n_units;
    int item = w[t].item0 + (int)(u * n_chunks);
    if (item < cb[j - 1]) item = cb[j - 1];
    if (item > n_items) item = n_items;
    cb[j] = item;
  }
  std::vector<int> b(n_warps + 1);
  for (int j = 0; j < n_clusters; ++j) {
    const int64_t c0 = cost_at(cb[j]), c1 = cost_at(cb[j + 1]);
    for (int k = 0; k < per_cluster; ++k)
      b[j * per_cluster + k] = k == 0 ? cb[j] : first_at(c0 + (c1 - c0) * k / per_cluster, cb[j], cb[j + 1]);
  }
  b[n_warps] = n_items;
  std::copy(b.begin(), b.end(), begin);
  if (cache.entries.size() < 64) {
    cache.entries.push_back({key, b});
  } else {
    cache.entries[cache.next] = {key, b};
    cache.next = (cache.next + 1) % cache.entries.size();
  }
  return true;
}

struct Plan {
  int x_bytes, smem_bytes, depth, slot_bytes, want2, split, ch_half;
};

bool make_plan(const TierParams& TP, int64_t K, int M, Plan& p) {
  const int n_chunks = (int)(K / 128);
  p.slot_bytes = 0;
  p.want2 = 0;
  for (int i = 0; i < TP.n_tiers; ++i) {
    if (TP.t[i].n_rows == 0) continue;
    const int cb = chunk_bytes(TP.t[i].bits);
    p.slot_bytes = cb > p.slot_bytes ? cb : p.slot_bytes;
    if (TP.t[i].bits == 2) p.want2 = 1;
  }
  if (p.slot_bytes == 0) p.slot_bytes = 16;
  const int part_bytes = kWarps * 2 * 32 * M * 4;  // reuses the rings after the main loop
  auto ring_bytes = [&](int d) { return kWarps * d * p.slot_bytes > part_bytes ? kWarps * d * p.slot_bytes : part_bytes; };
  // whole records first; when they do not fit beside a 2-deep ring, each CTA
  // of a cluster holds half of the chunks and reads the other half from its peer
  for (int split = 0; split < 2; ++split) {
    p.split = split;
    p.ch_half = split ? (n_chunks + 1) / 2 : n_chunks;
    const int n_rec = p.ch_half;
    p.x_bytes = n_rec * M * kRecStride;
    // records, (C, S) per chunk and token, 2^e per token, ring barriers
    const int fixed = (p.want2 ? 2 : 1) * p.x_bytes + n_rec * M * 16 + 64 + kWarps * 8 * 8;
    int depth = kRingBudget / p.slot_bytes;
    depth = depth < 2 ? 2 : (depth > 8 ? 8 : depth);
    while (depth > 2 && fixed + ring_bytes(depth) > kSmemBudget) --depth;
    p.depth = depth;
    p.smem_bytes = fixed + ring_bytes(depth);
    if (p.smem_bytes <= kSmemBudget) return true;
  }
  return false;
}

template <typename ACT, int NT, bool SPLIT>
int set_smem_attr() {
  static bool done = false;
  if (!done) {
    if (cudaFuncSetAttribute(qgemv_mma_kernel<ACT, NT, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemBudget) != cudaSuccess)
      return launch_status();
    done = true;
  }
  return CSAQ_OK;
}

template <typename ACT, int NT>
int launch_mma_block(const TierParams& TP, int64_t K, const ACT* x, int M, int64_t ldx, const csaq_gemv_ext& ext,
                     const ACT* x_mul, cudaStream_t st) {
  Plan pl;
  if (!make_plan(TP, K, M, pl)) return CSAQ_ERR_UNSUPPORTED;
  int rc = pl.split ? set_smem_attr<ACT, NT, true>() : set_smem_attr<ACT, NT, false>();
  if (rc) return rc;
  static thread_local KParams P;  // about 12 KB: kept off the stack
  P.tp = TP;
  if (work_table(TP, K, P.w) < 0) return CSAQ_ERR_UNSUPPORTED;
  const int items = P.w[TP.n_tiers - 1].item0 + P.w[TP.n_tiers - 1].n_items;
  if (items == 0) return CSAQ_OK;
  P.n_items_total = items;
  P.slot_bytes = pl.slot_bytes;
  P.depth = pl.depth;
  P.want2 = pl.want2;
  P.x_bytes = pl.x_bytes;
  P.split = pl.split;
  P.ch_half = pl.ch_half;
  P.silu_tiers = ext.silu_tiers;
  P.x_mul = x_mul;
  // the grid depends on the shapes and the SM count only (never on M)
  int ctas = (items + kWarps - 1) / kWarps;
  ctas = (ctas + kCluster - 1) / kCluster * kCluster;
  ctas = ctas < grid_ctas_max() ? ctas : grid_ctas_max();
  P.n_warps = ctas * kWarps;
  partition(TP, P.w, K, P.n_warps, P.begin);
  if (pl.split)
    return launch_pdl(qgemv_mma_kernel<ACT, NT, true>, dim3((unsigned)ctas), dim3(kThreads), (size_t)pl.smem_bytes,
                      st, P, K, x, M, ldx);
  return launch_pdl(qgemv_mma_kernel<ACT, NT, false>, dim3((unsigned)ctas), dim3(kThreads), (size_t)pl.smem_bytes, st,
                    P, K, x, M, ldx);
}

template <typename ACT>
int launch_mma(const TierParams& P0, int64_t K, const void* x, int64_t M, int64_t ldx, cudaStream_t st,
               const csaq_gemv_ext* ext_in = nullptr) {
  const csaq_gemv_ext ext = ext_in ? *ext_in : csaq_gemv_ext{0u, nullptr};
  if (P0.tile_start[P0.n_tiers] == 0) return CSAQ_OK;
  int64_t m0 = 0;
  while (m0 < M) {
    int mb = (int)((M - m0) < 16 ? (M - m0) : 16);
    Plan probe;
    while (mb > 1 && !make_plan(P0, K, mb, probe)) --mb;
    TierParams P = P0;
    for (int i = 0; i < P.n_tiers; ++i) {
      P.t[i].y = reinterpret_cast<ACT*>(P.t[i].y) + m0 * P.t[i].ldy;
      if (P.t[i].residual)
        P.t[i].residual = reinterpret_cast<const ACT*>(P.t[i].residual) + m0 * P.t[i].ldr;
    }
    const ACT* xb = reinterpret_cast<const ACT*>(x) + m0 * ldx;
    const ACT* xm = ext.x_mul ? reinterpret_cast<const ACT*>(ext.x_mul) + m0 * ldx : nullptr;
    const int rc = mb <= 8 ? launch_mma_block<ACT, 1>(P, K, xb, mb, ldx, ext, xm, st)
                           : launch_mma_block<ACT, 2>(P, K, xb, mb, ldx, ext, xm, st);
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
  return launch_pdl(qgemv_simt_kernel<ACT>, dim3((unsigned)blocks), dim3(256), 0, st, P, K,
                    reinterpret_cast<const ACT*>(x), (int)M, ldx, rows);
}

}  // namespace
}  // namespace csaq

using namespace csaq;

extern "C" int64_t csaq_tile_blocks_bytes(int bits, int64_t n_rows, int64_t K) {
  if ((bits != 2 && bits != 4 && bits != 8 && bits != 16) || n_rows < 0 || K <= 0 || K % 128)
    return -1;
  const int64_t tiles = (n_rows + kTileRows - 1) / kTileRows;
  const int64_t units = (tiles + unit_tiles(bits) - 1) / unit_tiles(bits);
  return units * (K / 128) * chunk_bytes(bits);
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
  const int64_t tiles = (T.n_rows + kTileRows - 1) / kTileRows;
  const int64_t units = (tiles + unit_tiles(T.bits) - 1) / unit_tiles(T.bits);
  const int piece = T.bits == 2 ? 8 : 16;
  const int64_t pieces = units * n_chunks * unit_tiles(T.bits) * (code_bytes(T.bits) / piece);
  repack_codes_kernel<<<(pieces + 255) / 256, 256, 0, st>>>(T, n_chunks, units, blocks);
  int rc = launch_status();
  if (rc || T.bits == 16) return rc;
  const int64_t metas = units * n_chunks * unit_tiles(T.bits) * kTileRows;
  repack_meta_kernel<<<(metas + 255) / 256, 256, 0, st>>>(T, n_chunks, units, blocks);
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

extern "C" int csaq_qgemv_ext(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x, int x_dtype,
                              int64_t M, int64_t ldx, const csaq_gemv_ext* ext, void* stream) {
  TierParams P;
  int rc = build_params(tiers, n_tiers, K, P);
  if (rc) return rc;
  if (!x || !ext || M < 0 || ldx < K || !dtype_size(x_dtype)) return CSAQ_ERR_ARG;
  if ((ext->silu_tiers >> n_tiers) != 0u) return CSAQ_ERR_ARG;  // n_tiers <= CSAQ_MAX_TIERS (build_params)
  if (x_dtype == CSAQ_DT_F32 || !mma_eligible(P, K, x, ldx)) return CSAQ_ERR_UNSUPPORTED;
  if (ext->x_mul && reinterpret_cast<uintptr_t>(ext->x_mul) % 16) return CSAQ_ERR_UNSUPPORTED;
  if (M == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  return x_dtype == CSAQ_DT_BF16 ? launch_mma<__nv_bfloat16>(P, K, x, M, ldx, st, ext)
                                 : launch_mma<__half>(P, K, x, M, ldx, st, ext);
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

extern "C" int csaq_qgemv_wait_timeouts(int64_t* count) {
  if (!count) return CSAQ_ERR_ARG;
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess) return launch_status();
  *count = v;
  return CSAQ_OK;
}
