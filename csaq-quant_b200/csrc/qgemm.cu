// Mixed-precision quantised linear for many tokens (prefill / verify): a
// dequantise-to-bf16 GEMM on the 5th-generation tensor cores.
//
// Y[m, out_rows[i]] = residual + sum_k X[m, k] * bf16(W[i, k]) + bias, where
// bf16(W) is the reference's weight as F.linear sees it: the fp32 dequantised
// value (q - zp) * s rounded to the activation dtype (csaq/kernels.py:450-475).
//
// One CTA computes a 256-token x 256-row tile of one tier, K in steps of 64,
// with warp-specialised roles joined by mbarriers:
//   * warp 0, one thread: TMA loads of the activation tile A (256 tokens x 64
//     columns, 128-byte swizzle: exactly the layout the tensor core reads) and
//     of the raw packed codes of the weight tile (256 rows x 64 codes, 16 to
//     128 bytes a row, swizzled by the row width so that the dequantising
//     threads read it without bank conflicts) into a ring of 2-4 stages;
//   * warps 2-9, one weight row a thread: dequantise the row's 64 codes of the
//     step from shared memory into the weight tile B (256 x 64, activation
//     dtype, 128-byte swizzle: 16-byte chunk c of row r at chunk c ^ (r % 8),
//     8-row groups 1024 bytes apart), double-buffered. A code q becomes the
//     fp32 value 2^23 + q by one byte permute into the mantissa of 2^23, so
//     q - zp is one exact subtraction of 2^23 + zp;
//   * warp 1, one thread: per step 4 x 2 tcgen05.mma (M=128, N=256, K=16) into
//     two 128 x 256 fp32 accumulators in tensor memory (tokens 0-127 at
//     columns 0-255, tokens 128-255 at columns 256-511); each step's commit
//     frees its load stage and its B buffer;
//   * after the last step warps 2-9 read the accumulators with tcgen05.ld
//     (a warp reads the 32 lanes its rank allows), turn each 32 x 32 block
//     around in shared memory, add bias and residual and store the rows to
//     their output columns, one token per store instruction.
// Tiles are visited in groups of 8 token tiles, so the CTAs running at once
// share their activation and weight tiles through L2. Tokens beyond M and
// rows beyond the tier read as zeros. Every wait is bounded; a CTA whose wait
// gives up raises a CTA-wide abort, stops issuing, lets its copies and MMAs in
// flight land, counts itself in g_qgemm_timeouts and ends without storing.

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "tile_blocks.cuh"

namespace csaq {
namespace {

CSAQ_GUARD_RECORD()

constexpr int kBM = 256;                   // tokens per tile (two MMAs of M = 128)
constexpr int kBN = 256;                   // weight rows per tile (MMA N)
constexpr int kBK = 64;                    // columns per step (one 128-byte swizzle row of bf16)
constexpr int kDqWarps = 16;               // two threads a weight row
constexpr int kThreads = 64 + 32 * kDqWarps;  // warp 0 TMA, warp 1 MMA, warps 2-17 dequantise + epilogue
constexpr int kATile = kBM * kBK * 2;      // 32 KB
constexpr int kBTile = kBN * kBK * 2;      // 32 KB
constexpr int kBBufs = 2;
constexpr int kMaxSmem = 232448;           // dynamic shared memory a CTA may opt into
constexpr int kEpiBytes = kDqWarps * 32 * 33 * 4;  // epilogue transpose blocks (in the rings)
constexpr int kGroupM = 8;                 // token tiles per raster group
constexpr int kWait = 1 << 22;             // polls of an mbarrier before a wait gives up

// raw code bytes of one weight row per step, and the load-ring depth for it
__host__ __device__ constexpr int raw_row_bytes(int bits) { return kBK * bits / 8; }
__host__ __device__ constexpr int load_stages(int bits) { return bits == 16 ? 2 : (bits == 8 ? 3 : 4); }
__host__ __device__ constexpr int smem_bytes(int bits) {
  return load_stages(bits) * (kATile + kBN * raw_row_bytes(bits)) + kBBufs * kBTile + 1024 + 256;
}
static_assert(smem_bytes(2) <= kMaxSmem && smem_bytes(4) <= kMaxSmem && smem_bytes(8) <= kMaxSmem &&
                  smem_bytes(16) <= kMaxSmem,
              "stage ring exceeds shared memory");
static_assert(2 * (kATile + kBN * raw_row_bytes(16)) >= kEpiBytes && 3 * (kATile + kBN * raw_row_bytes(8)) >= kEpiBytes &&
                  4 * (kATile + kBN * raw_row_bytes(2)) >= kEpiBytes,
              "epilogue blocks exceed the rings");

__device__ unsigned int g_qgemm_timeouts;

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// Wait for the phase of parity `parity` to complete. Gives up (false) after
// kWait polls, raising the CTA's abort flag, or as soon as another thread has
// raised it.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  for (int i = 0; i < kWait; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((i & 63) == 63 && *abort_flag) return false;
  }
  *abort_flag = 1;
  return false;
}

// 2-D TMA tile load into this CTA's shared memory, completing on `bar`
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// K-major, 128-byte swizzle, 8-row groups 1024 bytes apart (tcgen05 shared
// memory descriptor: start >> 4, leading offset 1 (unused when swizzled),
// stride offset 1024 >> 4, version 1, layout type 2 = 128-byte swizzle)
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// instruction descriptor: fp32 accumulator, bf16 (or fp16) A and B, both
// K-major, N = kBN, M = 128
template <typename ACT>
__device__ __forceinline__ uint32_t instr_desc() {
  const uint32_t fmt = std::is_same<ACT, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t ad, uint64_t bd, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem), "l"(ad), "l"(bd), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// byte offset of logical 16-byte chunk i of row r in a raw-code tile whose
// rows are rb bytes, as the TMA swizzle for that width places it (16: none;
// 32: chunk bit 0 ^= address bit 7; 64: chunk bits 0-1 ^= address bits 7-8;
// 128: chunk bits 0-2 ^= address bits 7-9)
__device__ __forceinline__ uint32_t raw_off(int rb, int r, int i) {
  const uint32_t a = (uint32_t)(r * rb + 16 * i);
  const uint32_t mask = rb == 128 ? 7u : (rb == 64 ? 3u : (rb == 32 ? 1u : 0u));
  return a ^ (((a >> 7) & mask) << 4);
}

// a and b rounded to the activation dtype, a in the low half
template <typename ACT>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  uint32_t d;
  if (std::is_same<ACT, __nv_bfloat16>::value)
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
  else
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
  return d;
}

// 2^23 + (byte `byte` of w), exactly, as fp32
__device__ __forceinline__ float magic(uint32_t w, uint32_t byte) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440u | byte));
}

// one packed pair (q_a - zp) * s, (q_b - zp) * s from the codes in byte
// `byte` of wa and of wb; nc = -(2^23 + zp) and ss = s in both lanes (the
// packed fp32 add and multiply round each lane like the scalar ops)
template <typename ACT>
__device__ __forceinline__ uint32_t dq2(uint32_t wa, uint32_t wb, uint32_t byte, float2 nc, float2 ss) {
  const float2 d = __fmul2_rn(__fadd2_rn(make_float2(magic(wa, byte), magic(wb, byte)), nc), ss);
  return pack2<ACT>(d.x, d.y);
}

// the four codes in the bytes of w (code j in byte j) as two packed pairs
template <typename ACT>
__device__ __forceinline__ uint2 dq4(uint32_t w, float2 nc, float2 ss) {
  const float2 d0 = __fmul2_rn(__fadd2_rn(make_float2(magic(w, 0), magic(w, 1)), nc), ss);
  const float2 d1 = __fmul2_rn(__fadd2_rn(make_float2(magic(w, 2), magic(w, 3)), nc), ss);
  return make_uint2(pack2<ACT>(d0.x, d0.y), pack2<ACT>(d1.x, d1.y));
}

// Dequantise half h (columns 32h .. 32h+31) of weight row r of a step from
// the raw tile and store it as chunks 4h .. 4h+3 of B row r (at brow).
template <typename ACT, int BITS>
__device__ __forceinline__ void dequant_half(const uint8_t* tile, int r, int h, float c, float s, uint8_t* brow,
                                             bool live) {
  constexpr int rb = raw_row_bytes(BITS);
  const float2 nc = make_float2(-c, -c), ss = make_float2(s, s);
  uint4 out[4];
  if (!live) {
#pragma unroll
    for (int k = 0; k < 4; ++k) out[k] = make_uint4(0u, 0u, 0u, 0u);
  } else if (BITS == 8) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {  // chunk 2h + i: 16 codes, output chunks 2i, 2i + 1 of the half
      const uint4 q = *reinterpret_cast<const uint4*>(tile + raw_off(rb, r, 2 * h + i));
      const uint2 a = dq4<ACT>(q.x, nc, ss), b = dq4<ACT>(q.y, nc, ss), e = dq4<ACT>(q.z, nc, ss),
                  f = dq4<ACT>(q.w, nc, ss);
      out[2 * i] = make_uint4(a.x, a.y, b.x, b.y);
      out[2 * i + 1] = make_uint4(e.x, e.y, f.x, f.y);
    }
  } else if (BITS == 4) {
    const uint4 q = *reinterpret_cast<const uint4*>(tile + raw_off(rb, r, h));  // 32 codes
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // word j: code 2t + n of its 8 in nibble n of byte t
      const uint32_t lo = w[j] & 0x0F0F0F0Fu, hi = (w[j] >> 4) & 0x0F0F0F0Fu;
      out[j] = make_uint4(dq2<ACT>(lo, hi, 0, nc, ss), dq2<ACT>(lo, hi, 1, nc, ss), dq2<ACT>(lo, hi, 2, nc, ss),
                          dq2<ACT>(lo, hi, 3, nc, ss));
    }
  } else if (BITS == 2) {
    const uint2 q = *reinterpret_cast<const uint2*>(tile + raw_off(rb, r, 0) + 8 * h);  // 32 codes
    const uint32_t w[2] = {q.x, q.y};
#pragma unroll
    for (int j = 0; j < 2; ++j) {  // word j: code 4t + n of its 16 in bits 2n of byte t
      const uint32_t m0 = w[j] & 0x03030303u, m1 = (w[j] >> 2) & 0x03030303u, m2 = (w[j] >> 4) & 0x03030303u,
                     m3 = (w[j] >> 6) & 0x03030303u;
      out[2 * j] = make_uint4(dq2<ACT>(m0, m1, 0, nc, ss), dq2<ACT>(m2, m3, 0, nc, ss), dq2<ACT>(m0, m1, 1, nc, ss),
                              dq2<ACT>(m2, m3, 1, nc, ss));
      out[2 * j + 1] = make_uint4(dq2<ACT>(m0, m1, 2, nc, ss), dq2<ACT>(m2, m3, 2, nc, ss),
                                  dq2<ACT>(m0, m1, 3, nc, ss), dq2<ACT>(m2, m3, 3, nc, ss));
    }
  } else {  // fp16 rows: chunk 4h + i holds 8 values
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 q = *reinterpret_cast<const uint4*>(tile + raw_off(rb, r, 4 * h + i));
      if (std::is_same<ACT, __half>::value) {
        out[i] = q;
      } else {
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = pack2<ACT>(__half2float(__ushort_as_half((unsigned short)(w[j] & 0xFFFFu))),
                            __half2float(__ushort_as_half((unsigned short)(w[j] >> 16))));
        out[i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) *reinterpret_cast<uint4*>(brow + (((4 * h + k) ^ (r & 7)) << 4)) = out[k];
}

template <typename ACT, int BITS>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                 const csaq_tier T, int64_t K, int64_t M, int use_meta) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int n_ls = load_stages(BITS);
  constexpr int rb = raw_row_bytes(BITS);
  constexpr int w_tile = kBN * rb;

  // grouped raster: kGroupM token tiles x every row tile, token tile fastest
  const int n_m = (int)((M + kBM - 1) / kBM), n_n = (T.n_rows + kBN - 1) / kBN;
  const int span = kGroupM * n_n, bid = blockIdx.x;
  const int first_m = (bid / span) * kGroupM;
  const int gm = min(n_m - first_m, kGroupM);
  const int mt = first_m + (bid % span) % gm, nt = (bid % span) / gm;
  const int64_t tok0 = (int64_t)mt * kBM;
  const int row0 = nt * kBN;
  const bool two = tok0 + 128 < M;  // the second accumulator has live tokens

  // layout: A ring, raw-code ring, B buffers (all 1024-aligned), barriers, flags
  const uint32_t raw_s = saddr(smem_raw);
  const uint32_t base = (raw_s + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw_s);
  const uint32_t a_ring = base, w_ring = base + n_ls * kATile, b_ring = w_ring + n_ls * w_tile;
  const uint32_t bars = b_ring + kBBufs * kBTile;
  const uint32_t full = bars, empty = bars + 8 * 4, bfull = bars + 8 * 8, bempty = bars + 8 * 10,
                 accfull = bars + 8 * 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bars - base) + 8 * 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + (bars - base) + 8 * 13 + 4);

  if (warp == 0) {  // 512 accumulator columns of tensor memory
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 32) {
    for (int s = 0; s < n_ls; ++s) {
      mbar_init(full + 8 * s, 1);
      mbar_init(empty + 8 * s, 1 + kDqWarps);  // the MMA commit and every dequantising warp
    }
    for (int b = 0; b < kBBufs; ++b) {
      mbar_init(bfull + 8 * b, kDqWarps);
      mbar_init(bempty + 8 * b, 1);
    }
    mbar_init(accfull, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (tid == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int n_k = (int)(K / kBK);
  // x may be written by the preceding kernel of the stream
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ── TMA producer ──
    if (lane == 0) {
      const uint32_t tx = (uint32_t)(kATile + w_tile);
      int s = 0, n_issued = 0;
      uint32_t ph = 0, issued_ph = 0;  // bit s: parity of stage s's last issue
      for (int kt = 0; kt < n_k; ++kt) {
        if (!mbar_wait(empty + 8 * s, ph ^ 1u, abort_flag)) break;
        mbar_expect_tx(full + 8 * s, tx);
        tma_load_2d(a_ring + s * kATile, &map_x, kt * kBK, (int)tok0, full + 8 * s);
        tma_load_2d(w_ring + s * w_tile, &map_w, kt * rb, row0, full + 8 * s);
        issued_ph = (issued_ph & ~(1u << s)) | (ph << s);
        ++n_issued;
        if (++s == n_ls) { s = 0; ph ^= 1u; }
      }
      // every issued copy lands before the CTA can end
      volatile int never = 0;
      for (int t = 0; t < n_ls && t < n_issued; ++t) mbar_wait(full + 8 * t, (issued_ph >> t) & 1u, &never);
    }
  } else if (warp == 1) {
    // ── MMA issuer ──
    if (lane == 0) {
      const uint32_t idesc = instr_desc<ACT>();
      int s = 0, sb = 0;
      uint32_t ph = 0, phb = 0;
      for (int kt = 0; kt < n_k; ++kt) {
        if (!mbar_wait(full + 8 * s, ph, abort_flag)) break;
        if (!mbar_wait(bfull + 8 * sb, phb, abort_flag)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_s = a_ring + s * kATile, b_s = b_ring + sb * kBTile;
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j) {  // K = 16 per MMA: 32 bytes along the swizzled row
          const uint64_t bd = smem_desc(b_s + 32 * j);
          const uint32_t acc = (kt > 0 || j > 0) ? 1u : 0u;
          mma_f16(tmem, smem_desc(a_s + 32 * j), bd, idesc, acc);
          if (two) mma_f16(tmem + 256, smem_desc(a_s + 128 * 128 + 32 * j), bd, idesc, acc);
        }
        mma_commit(empty + 8 * s);
        mma_commit(bempty + 8 * sb);
        if (++s == n_ls) { s = 0; ph ^= 1u; }
        if (++sb == kBBufs) { sb = 0; phb ^= 1u; }
      }
      mma_commit(accfull);  // completes when every MMA issued above has
    }
  } else {
    // ── dequantise: two threads a weight row ──
    const int d = tid - 64, r = d >> 1, h = d & 1;
    const int64_t wrow = row0 + r;
    const bool live = wrow < T.n_rows;
    // Scales and zero points come from the tier's GEMV blocks when it has
    // them: there a warp's 16 rows have theirs for a 128-column chunk in 80
    // contiguous bytes (three sectors a load, against sixteen for rows
    // strided by n_groups in the reference layout).
    const int rl = lane >> 1;  // row within the warp's 16
    const uint8_t* meta = nullptr;
    if (use_meta && BITS != 16 && live) {
      const int64_t tile16 = wrow / kTileRows;
      meta = T.blocks + (tile16 / unit_tiles(BITS)) * (K / 128) * chunk_bytes(BITS) +
             (tile16 % unit_tiles(BITS)) * tile_block_bytes(BITS) + code_bytes(BITS);
    }
    // scale and zero point of step k (raw: nothing waits on the loads here)
    auto load_sz = [&](int k, uint32_t& z, float& sc) {
      z = 0u;
      sc = 0.0f;
      if (live && BITS != 16 && k < n_k) {
        if (meta) {
          const uint8_t* m = meta + (int64_t)(k >> 1) * chunk_bytes(BITS);
          sc = reinterpret_cast<const float*>(m)[rl];
          z = m[64 + rl];
        } else {
          const int64_t gi = wrow * T.n_groups + (T.n_groups > 1 ? ((int64_t)k * kBK) / T.group_size : 0);
          sc = T.scales[gi];
          z = T.zps[gi];
        }
      }
    };
    int s = 0, sb = 0;
    uint32_t ph = 0, phb = 0;
    // one step: wait for the stage's codes and a free B buffer, dequantise, publish
    auto step = [&](uint32_t z, float sc) -> bool {
      if (!mbar_wait(full + 8 * s, ph, abort_flag)) return false;
      if (!mbar_wait(bempty + 8 * sb, phb ^ 1u, abort_flag)) return false;
      dequant_half<ACT, BITS>(gbase + (w_ring - base) + s * w_tile, r, h, 8388608.0f + (float)z, sc,
                              gbase + (b_ring - base) + sb * kBTile + r * 128, live);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(empty + 8 * s);   // this warp's raw codes are read
        mbar_arrive(bfull + 8 * sb);  // and its 16 rows of B written
      }
      if (++s == n_ls) { s = 0; ph ^= 1u; }
      if (++sb == kBBufs) { sb = 0; phb ^= 1u; }
      return true;
    };
    // two steps a trip, each with its own scale registers, refilled for two
    // steps later right after use: the loads have a step to land and no
    // register copy waits on them
    uint32_t za, zb;
    float sa, sb2;
    load_sz(0, za, sa);
    load_sz(1, zb, sb2);
    for (int kt = 0; kt < n_k; kt += 2) {
      if (!step(za, sa)) break;
      load_sz(kt + 2, za, sa);
      if (kt + 1 < n_k) {
        if (!step(zb, sb2)) break;
        load_sz(kt + 3, zb, sb2);
      }
    }

    // ── epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (the lanes its
    // rank may access) of accumulator ((w - 2) / 4) % 2, columns 128 ((w - 2) / 8) .. +127 ──
    // 32 x 32 blocks pass through shared memory (the A and raw rings, idle once
    // every MMA is done), so that a store instruction writes one token's 32
    // consecutive tier rows (ascending output columns) rather than 32 tokens'
    // rows of one column.
    volatile int never = 0;
    const bool done = mbar_wait(accfull, 0u, &never) && !*abort_flag;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int q = warp & 3, half = ((warp - 2) >> 2) & 1, c0 = ((warp - 2) >> 3) * 128;
    const int64_t tokw = tok0 + 128 * half + 32 * q;  // this warp's first token
    float* buf = reinterpret_cast<float*>(gbase) + (warp - 2) * (32 * 33);
    if (done && (half == 0 || two) && tokw < M) {
#pragma unroll 1
      for (int cb = c0; cb < c0 + 128 && row0 + cb < T.n_rows; cb += 32) {
        uint32_t v[32];
        const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(256 * half + cb);
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
              "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),
              "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),
              "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; ++j) buf[lane * 33 + j] = __uint_as_float(v[j]);  // [token][row]
        __syncwarp();
        const int row = row0 + cb + lane;  // lane = tier row
        const int orow = row < T.n_rows ? T.out_rows[row] : 0;
        const bool rlive = row < T.n_rows &&
                           CSAQ_GUARD(orow >= 0 && orow < T.ldy && (!T.residual || orow < T.ldr),
                                      CSAQ_GUARD_GEMM_OUT_ROW, orow, T.ldy);
        const float bv = (rlive && T.bias) ? to_f32<ACT>(reinterpret_cast<const ACT*>(T.bias)[orow]) : 0.0f;
        const int nt_w = M - tokw < 32 ? (int)(M - tokw) : 32;
        for (int t = 0; t < nt_w; ++t) {
          const int64_t tok = tokw + t;
          float y = buf[t * 33 + lane];
          if (rlive) {
            if (T.bias) y = __fadd_rn(y, bv);
            if (T.residual)
              y = __fadd_rn(y, to_f32<ACT>(reinterpret_cast<const ACT*>(T.residual)[tok * T.ldr + orow]));
            reinterpret_cast<ACT*>(T.y)[tok * T.ldy + orow] = from_f32<ACT>(y);
          }
        }
        __syncwarp();
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (tid == 0 && *abort_flag) atomicAdd(&g_qgemm_timeouts, 1u);
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
}

// ── host: tensor maps ───────────────────────────────────────────────────────
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    (void)cudaGetLastError();
  });
  return fn;
}

// activations: K x M elements of 2 bytes, row stride ldx; box 64 x 256, 128-byte swizzle
bool map_activations(CUtensorMap* m, const void* x, int x_dtype, int64_t K, int64_t M, int64_t ldx) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)ldx * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)kBM};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, x_dtype == CSAQ_DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// raw codes of a tier: row_bytes x n_rows bytes; box (64 * bits / 8) x 256,
// swizzled by the box width
bool map_codes(CUtensorMap* m, const csaq_tier& t) {
  auto fn = encode_fn();
  if (!fn) return false;
  const int rb = raw_row_bytes(t.bits);
  const cuuint64_t dims[2] = {(cuuint64_t)t.row_bytes, (cuuint64_t)t.n_rows};
  const cuuint64_t strides[1] = {(cuuint64_t)t.row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)rb, (cuuint32_t)kBN};
  const cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = rb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : rb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : rb == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                           : CU_TENSOR_MAP_SWIZZLE_NONE;
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(t.codes), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename ACT, int BITS>
int launch_tier(const CUtensorMap& mx, const CUtensorMap& mw, const csaq_tier& T, int64_t K, int64_t M,
                unsigned n_tiles, cudaStream_t st) {
  // the GEMV blocks hold one scale per (row, 128 columns): usable when K and
  // the group size are whole chunks (csaq_repack_tiles accepts nothing else)
  const int use_meta = T.blocks && K % 128 == 0 && (T.n_groups == 1 || T.group_size % 128 == 0) ? 1 : 0;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(qgemm_kernel<ACT, BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem_bytes(BITS));
  });
  if (attr != cudaSuccess) {
    set_last_cuda_error(attr);
    return CSAQ_ERR_CUDA;
  }
  return launch_pdl(qgemm_kernel<ACT, BITS>, dim3(n_tiles), dim3(kThreads), (size_t)smem_bytes(BITS), st, mx, mw, T,
                    K, M, use_meta);
}

template <typename ACT>
int launch_qgemm(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x, int x_dtype, int64_t M, int64_t ldx,
                 cudaStream_t st) {
  CUtensorMap mx;
  if (!map_activations(&mx, x, x_dtype, K, M, ldx)) return CSAQ_ERR_UNSUPPORTED;
  for (int i = 0; i < n_tiers; ++i) {
    const csaq_tier& T = tiers[i];
    if (T.n_rows == 0) continue;
    CUtensorMap mw;
    if (!map_codes(&mw, T)) return CSAQ_ERR_UNSUPPORTED;
    const int64_t n_tiles = ((M + kBM - 1) / kBM) * ((T.n_rows + kBN - 1) / kBN);
    if (n_tiles > INT32_MAX) return CSAQ_ERR_UNSUPPORTED;
    const unsigned nt = (unsigned)n_tiles;
    const int rc = T.bits == 2   ? launch_tier<ACT, 2>(mx, mw, T, K, M, nt, st)
                   : T.bits == 4 ? launch_tier<ACT, 4>(mx, mw, T, K, M, nt, st)
                   : T.bits == 8 ? launch_tier<ACT, 8>(mx, mw, T, K, M, nt, st)
                                 : launch_tier<ACT, 16>(mx, mw, T, K, M, nt, st);
    if (rc) return rc;
  }
  return CSAQ_OK;
}

}  // namespace
}  // namespace csaq

using namespace csaq;

extern "C" int csaq_qgemm(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x, int x_dtype, int64_t M,
                          int64_t ldx, void* stream) {
  if (!tiers || n_tiers < 1 || n_tiers > CSAQ_MAX_TIERS || !x || M < 0 || K <= 0 || ldx < K)
    return CSAQ_ERR_ARG;
  if (x_dtype != CSAQ_DT_F16 && x_dtype != CSAQ_DT_BF16) return CSAQ_ERR_ARG;
  if (K % kBK || ldx % 8 || reinterpret_cast<uintptr_t>(x) % 16 || M > INT32_MAX) return CSAQ_ERR_UNSUPPORTED;
  for (int i = 0; i < n_tiers; ++i) {
    const csaq_tier& t = tiers[i];
    if (t.bits != 2 && t.bits != 4 && t.bits != 8 && t.bits != 16) return CSAQ_ERR_BITS;
    if (t.n_rows < 0 || (t.n_rows > 0 && (!t.codes || !t.out_rows || !t.y))) return CSAQ_ERR_ARG;
    if (t.row_bytes < packed_row_bytes(K, t.bits)) return CSAQ_ERR_ARG;
    if (t.bits != 16 && t.n_rows > 0) {
      if (!t.scales || !t.zps || t.n_groups < 1) return CSAQ_ERR_ARG;
      if (t.n_groups > 1 && (t.group_size % kBK || t.n_groups < (K + t.group_size - 1) / t.group_size))
        return CSAQ_ERR_UNSUPPORTED;
    }
    // the codes arrive by TMA: 16-byte aligned base and row stride
    if (t.n_rows > 0 && (reinterpret_cast<uintptr_t>(t.codes) % 16 || t.row_bytes % 16))
      return CSAQ_ERR_UNSUPPORTED;
  }
  if (M == 0) return CSAQ_OK;
  cudaStream_t st = as_stream(stream);
  return x_dtype == CSAQ_DT_BF16 ? launch_qgemm<__nv_bfloat16>(tiers, n_tiers, K, x, x_dtype, M, ldx, st)
                                 : launch_qgemm<__half>(tiers, n_tiers, K, x, x_dtype, M, ldx, st);
}

extern "C" int csaq_qgemm_wait_timeouts(int64_t* count) {
  if (!count) return CSAQ_ERR_ARG;
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_qgemm_timeouts, sizeof(v)) != cudaSuccess) return launch_status();
  *count = v;
  return CSAQ_OK;
}
