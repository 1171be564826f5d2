/*
 * csaq_b200.h — C ABI of the B200 (sm_100a) quantised hot path of csaq-quant.
 *
 * Every compute entry point is stream-ordered (enqueues work on `stream`, a
 * cudaStream_t passed as void*), never synchronises, never allocates, and
 * returns an int status (CSAQ_OK = 0, negative on error). The exception is
 * the one-time set-up of the tensor-parallel exchange (csaq_p2p_alloc/free,
 * csaq_ipc_open/close), which allocates and maps its buffers synchronously.
 * Buffers are caller-owned device pointers. Sizes are int64_t. Layouts are
 * row-major.
 *
 * Packed-code layout (identical to csaq-quant's storage):
 *   bits 8: one byte per code;   bits 4: byte j = col 2j (low nibble) | col 2j+1 (high);
 *   bits 2: byte j holds cols 4j..4j+3 at bit offsets 0,2,4,6;
 *   bits 16: the fp16 bit pattern, 2 bytes per column.
 *   packed row length = ceil(cols * bits / 8) bytes.
 * Scales are fp32 and zero points int32, one per (row, group); per-channel
 * quantisation has one group per row.
 */
#ifndef CSAQ_B200_H
#define CSAQ_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  CSAQ_OK = 0,
  CSAQ_ERR_ARG = -1,          /* null pointer, bad size, bad dtype            */
  CSAQ_ERR_BITS = -2,         /* unsupported bit-width                          */
  CSAQ_ERR_CUDA = -3,         /* a CUDA launch failed; see csaq_last_cuda_error */
  CSAQ_ERR_TIMEOUT = -4,      /* a bounded device wait gave up                  */
  CSAQ_ERR_UNSUPPORTED = -5,  /* shape/alignment outside what the kernel serves */
  CSAQ_ERR_SCRATCH = -6,      /* the call needs more scratch than csaq_decode_attention_static holds */
};

enum { CSAQ_DT_F32 = 0, CSAQ_DT_F16 = 1, CSAQ_DT_BF16 = 2 };

/* Library identification and diagnostics (no reference counterpart). */
const char* csaq_version(void);
const char* csaq_status_string(int status);
int csaq_last_cuda_error(void);   /* cudaError_t of the last failed launch in this thread */

/* Checked builds (no reference counterpart: the reference has no device
 * code). libcsaq_b200_checked.so (build.py --checked) tests the
 * indices that kernels take from caller data before using them; a failed
 * test is counted, the first one is recorded (site, value, bound) and the
 * access is skipped. The default library has no such tests and reports
 * CSAQ_ERR_UNSUPPORTED from csaq_guard_report / csaq_guard_clear. */
enum {
  CSAQ_GUARD_GEMV_OUT_ROW = 1,  /* csaq_qgemv: out_rows[i] outside [0, ldy) (or [0, ldr) with a residual) */
  CSAQ_GUARD_GEMM_OUT_ROW = 2,  /* csaq_qgemm: the same                                               */
  CSAQ_GUARD_ROPE_POS = 3,      /* csaq_rope_kv: position pos0[b] + s outside [0, Lmax)                */
  CSAQ_GUARD_ATTN_POS = 4       /* csaq_decode_attention: pos0[b] < 0 or pos0[b] + S > Lmax           */
};
int csaq_checked_build(void);     /* 1 for the checked library, else 0 */
int csaq_guard_report(int64_t* count, int64_t* site, int64_t* value, int64_t* bound);
int csaq_guard_clear(void);

/* ── Quantisation primitives ─────────────────────────────────────────────── */

/* Packed bytes per row: replaces the cols_packed arithmetic of
 * csaq/kernels.py:336-345 and the shapes produced by _pack (csaq/kernels.py:539-569). */
int64_t csaq_packed_row_bytes(int64_t cols, int bits);

/* Per-(row, group) asymmetric scale and zero point from min/max:
 * csaq/kernels.py:495-508 (_compute_scale_zp) on the per-channel
 * (csaq/kernels.py:113-118) or zero-padded per-group (csaq/kernels.py:129-138)
 * statistics. group_size <= 0 or >= cols selects per-channel (one group, no
 * padding). scales/zero_points: rows x n_groups. row_absmax (nullable): max |W|
 * per row, used for the follower-outlier warning of csaq/kernels.py:208-218. */
int csaq_group_scales(const void* W, int w_dtype, int64_t rows, int64_t cols, int64_t ld_w,
                      int bits, int64_t group_size, float* scales, int32_t* zero_points,
                      float* row_absmax, void* stream);

/* Quantise + pack with given scales: csaq/kernels.py:511-523 (_quantize_rows) then
 * csaq/kernels.py:539-569 (_pack).
 * scale_mode 0: row r uses scales[r, :]; 1: every row uses row 0 (shared scale,
 * csaq/kernels.py:220-223, 247-252); 2: row r uses row src_row[r].
 * requant != 0 reproduces CSAQLinear.from_cliques (csaq/kernels.py:414-434):
 * dequantise (q - zp) * scale in fp32, then _float_to_int (csaq/kernels.py:526-536). */
int csaq_quant_pack_rows(const void* W, int w_dtype, int64_t rows, int64_t cols, int64_t ld_w,
                         int bits, int64_t group_size, const float* scales,
                         const int32_t* zero_points, int64_t ld_s, int scale_mode,
                         const int32_t* src_row, int requant, uint8_t* qdata, void* stream);

/* quantize_per_channel (csaq/kernels.py:77-158) for bits 2/4/8: scales +
 * codes in one pass where the group layout allows it (fused warp-per-group
 * kernel with 128-bit loads and shuffle min/max), else csaq_group_scales +
 * csaq_quant_pack_rows. */
int csaq_quant_pack(const void* W, int w_dtype, int64_t rows, int64_t cols, int64_t ld_w,
                    int bits, int64_t group_size, uint8_t* qdata, float* scales,
                    int32_t* zero_points, void* stream);

/* quantize_per_channel(bits=16): the fp16 cast (csaq/kernels.py:94-107). */
int csaq_cast_f16(const void* W, int w_dtype, int64_t rows, int64_t cols, int64_t ld_w,
                  uint16_t* out, void* stream);

/* _pack (csaq/kernels.py:539-569): int32 codes -> packed bytes (low byte kept). */
int csaq_pack(const int32_t* q, int bits, int64_t rows, int64_t cols, uint8_t* out, void* stream);

/* _unpack (csaq/kernels.py:572-600): packed bytes -> int32 codes. */
int csaq_unpack(const uint8_t* packed, int bits, int64_t rows, int64_t cols, int32_t* out,
                void* stream);

/* _float_to_int (csaq/kernels.py:526-536): row-wise requantisation to int32 codes. */
int csaq_float_to_int(const float* W, const float* scales, const int32_t* zero_points, int bits,
                      int64_t rows, int64_t cols, int32_t* out, void* stream);

/* _dequantize (csaq/kernels.py:603-619) and CSAQLinear._get_weight_fp32
 * (csaq/kernels.py:450-468): (q - zp) * scale in fp32, bit-exact; column c
 * uses group c / group_size (group_size <= 0: per-channel). bits 16 reads fp16.
 * nan_to_num != 0 applies csaq/kernels.py:467. out_dtype F16/BF16 rounds the
 * fp32 value once (the .to(x.dtype) of csaq/kernels.py:471). */
int csaq_dequant(const uint8_t* qdata, const float* scales, const int32_t* zero_points, int bits,
                 int64_t rows, int64_t cols, int64_t group_size, int nan_to_num, int out_dtype,
                 void* out, void* stream);

/* ── Mixed-precision quantised linear ────────────────────────────────────── */

/* One row tier of a mixed linear: rows stored at one bit-width. A linear is a
 * list of tiers; several linears that read the same activation (q/k/v,
 * gate/up) can share one launch. The verify pass of self-speculative decoding
 * is the same launch with each tier's protected rows left out (n_rows covers
 * only the unprotected head of the tier) plus a 16-bit tier holding the fp16
 * backups of the protected rows, scattered to their output rows.
 * Replaces CSAQLinear._get_weight_fp32 + F.linear (csaq/kernels.py:450-475)
 * and the verify weight swap (csaq/inference.py:219-237). */
typedef struct csaq_tier {
  int32_t bits;            /* 2, 4, 8, or 16 (fp16 rows)                       */
  int32_t n_rows;          /* rows computed from this tier                     */
  int32_t group_size;      /* columns per scale group (K for per-channel)      */
  int32_t n_groups;        /* scale/zp columns per row                         */
  int64_t row_bytes;       /* byte stride between packed rows                  */
  const uint8_t* codes;    /* n_rows x row_bytes                               */
  const float* scales;     /* n_rows x n_groups (ignored for bits 16)          */
  const uint8_t* zps;      /* n_rows x n_groups, zero points as uint8          */
  const int32_t* out_rows; /* output column of y for each tier row             */
  const uint8_t* blocks;   /* nullable: the tier repacked by csaq_repack_tiles;
                              the tensor-core kernel reads only this           */
  void* y;                 /* output, M x ldy, activation dtype                */
  int64_t ldy;
  const void* bias;        /* nullable; indexed by output row, activation dtype */
  const void* residual;    /* nullable; M x ldr, activation dtype: y = residual + W x */
  int64_t ldr;
} csaq_tier;

#define CSAQ_MAX_TIERS 16

/* GEMV block layout of a tier: one contiguous block per (16-row tile,
 * 128-column chunk), tile-major; inside a block the codes are ordered by the
 * MMA lane that consumes them, followed by the 16 rows' fp32 scales and uint8
 * zero points of that chunk's group (rows past n_rows are zero). Built once
 * per layer from the reference layout; K must be a multiple of 128 and the
 * group size a power-of-two multiple of 128 (or per-channel). */
int64_t csaq_tile_blocks_bytes(int bits, int64_t n_rows, int64_t K);
int csaq_repack_tiles(const csaq_tier* tier, int64_t K, uint8_t* blocks, void* stream);

/* y[m, out_rows[i]] = residual + sum_k W[i, k] * x[m, k] + bias, fp32
 * accumulation; x is M x ldx in x_dtype (F32, F16 or BF16), y and bias and
 * residual in the same dtype. F16/BF16 use the tensor-core kernel when every
 * tier with rows has `blocks` (csaq_repack_tiles) and x is 16-byte aligned with
 * ldx % 8 == 0; everything else (and F32) uses the CUDA-core kernel, which
 * reads the reference layout (`codes`, `scales`, `zps`). Results of the
 * tensor-core kernel for one token do not depend on M. */
int csaq_qgemv(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x, int x_dtype,
               int64_t M, int64_t ldx, void* stream);

/* The HF LlamaMLP gate fused into the tensor-core GEMV, for the decode
 * runtime (no reference counterpart; the reference runs act_fn(gate(x)) *
 * up(x) as separate torch ops). Bit i of silu_tiers: tier i stores
 * dtype(silu(y)), y the value csaq_qgemv would store (the gate tiers of a
 * fused gate/up launch). x_mul non-null: the input is h = dtype(x * x_mul),
 * elementwise, x_mul M x ldx like x (the down projection reading g' and u).
 * Together they give bit for bit csaq_qgemv, csaq_silu_mul, csaq_qgemv.
 * Needs the tensor-core kernel's conditions (else CSAQ_ERR_UNSUPPORTED). */
typedef struct csaq_gemv_ext {
  uint32_t silu_tiers;
  const void* x_mul;
} csaq_gemv_ext;
int csaq_qgemv_ext(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x, int x_dtype,
                   int64_t M, int64_t ldx, const csaq_gemv_ext* ext, void* stream);

/* The same product for many tokens (prefill / verify with M in the tens to
 * thousands), on the tcgen05 tensor cores: X (bf16 or fp16) times the tier
 * weights dequantised in shared memory to X's dtype, exactly as the
 * reference's forward materialises them (csaq/kernels.py:450-475: fp32
 * (q - zp) * s, then .to(x.dtype)), fp32 accumulation in tensor memory.
 * Reads the reference layout (`codes`, `scales`, `zps`; `blocks` unused).
 * Needs K % 64 == 0, 16-byte aligned x with ldx % 8 == 0, group sizes that
 * are multiples of 64, and code rows (pointer and row_bytes) aligned to 16
 * bytes (8 for 2-bit tiers) (else CSAQ_ERR_UNSUPPORTED). One launch per tier. */
int csaq_qgemm(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x, int x_dtype, int64_t M,
               int64_t ldx, void* stream);
/* CTAs of csaq_qgemm whose bounded wait for the tensor core gave up
 * (diagnostic; no reference counterpart). */
int csaq_qgemm_wait_timeouts(int64_t* count);

/* Number of warps, since the library was loaded on this device, whose bounded
 * wait for a weight copy in the tensor-core kernel gave up (the launch still
 * ends; its output is then unreliable). Synchronises the device. No
 * counterpart in the reference (its kernels have no device-side waits). */
int csaq_qgemv_wait_timeouts(int64_t* count);

/* Same contract as csaq_qgemv (the forward of csaq/kernels.py:450-475),
 * always the CUDA-core kernel (any K, any group size, any M); a second GPU
 * path used to cross-check the tensor-core kernel. */
int csaq_qgemv_simt(const csaq_tier* tiers, int n_tiers, int64_t K, const void* x, int x_dtype,
                    int64_t M, int64_t ldx, void* stream);


/* ── Calibration ─────────────────────────────────────────────────────────── */

/* Co-activation mask of one activation block (n_tok x C, row stride ld),
 * bit-packed channel-major: bits[c * ld_bits + (tok_offset + t) / 32] bit
 * (tok_offset + t) % 32. tok_offset must be a multiple of 32.
 * mode 0: act > thr (thr given in the activation dtype's value).
 * mode 1: the profiler hook of csaq/core.py:143-155: per token keep channels
 *         with |act| >= the k-th largest |act| (ties kept); tok_thr is an
 *         n_tok scratch array of uint32 written by the call. */
int csaq_act_mask(const void* act, int dtype, int64_t n_tok, int64_t C, int64_t ld, int mode,
                  float thr, int64_t k, uint32_t* tok_thr, uint32_t* bits, int64_t ld_bits,
                  int64_t tok_offset, void* stream);

/* Intersection counts inter[i][j] = popc(mask_i & mask_j) summed over words
 * (the exact integers of mask^T mask, csaq/core.py:261-262) and activation
 * counts f[i] (csaq/core.py:263; nullable). */
int csaq_coact_counts(const uint32_t* bits, int64_t C, int64_t n_words, int64_t ld_bits,
                      int32_t* inter, int64_t ld_i, int32_t* f, void* stream);

/* Jaccard threshold bits: adj[i] bit j = (I/max(f_i+f_j-I, 1) >= threshold) in
 * fp32 (csaq/core.py:263-275); threshold is the fp32-rounded value. */
int csaq_jaccard_bits(const int32_t* inter, int64_t ld_i, const int32_t* f, int64_t C,
                      float threshold, uint32_t* adj, int64_t ld_adj, void* stream);

/* Seed-order greedy clique partition (csaq/core.py:268-285):
 * labels[c] = clique index of channel c in seed order; *n_cliques = count.
 * Bits of columns >= C are ignored. labels also serves as the call's scratch
 * (per-row flags between its two launches), so it must not alias adj.
 * C up to 1.6M channels (the taken set, C/8 bytes, lives in shared memory;
 * up to 819,200 channels singleton runs are labelled a word at a time). */
int csaq_greedy_cliques(const uint32_t* adj, int64_t ld_adj, int64_t C, int32_t* labels,
                        int32_t* n_cliques, void* stream);

/* Salience accumulation acc += |G * W| in fp32 over n contiguous elements
 * (csaq/core.py:204-210), and the final acc /= n_batches (csaq/core.py:232-233). */
int csaq_salience_accum(const void* G, const void* W, int dtype, int64_t n, float* acc,
                        void* stream);
int csaq_salience_finalize(float* acc, int64_t n, int64_t n_batches, void* stream);

/* ── Decoder runtime (Llama / Qwen2 decode around the quantised linears) ─── */
/* Token (b, s) of a step with S tokens per sequence is row b*S+s of every
 * activation matrix and sits at position pos0[b] + s. KV caches are
 * (B, Hkv, Lmax, D). These replace the HF module forwards that
 * CSAQInferenceEngine drives (csaq/inference.py:443-476). */

/* HF RMSNorm: y = w * dtype(x * rsqrt(mean(x^2) + eps)). */
int csaq_rmsnorm(const void* x, int64_t ldx, const void* w, void* y, int64_t ldy, int64_t M,
                 int64_t H, float eps, int dtype, void* stream);

/* Rotary embedding (rotate_half convention, cos/sin tables (Lmax, D) fp32)
 * of q and k; writes q_out (M, Hq, D) and k/v into the caches. */
int csaq_rope_kv(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                 const int32_t* pos0, int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D,
                 const float* cos_t, const float* sin_t, void* q_out, void* k_cache, void* v_cache,
                 int64_t Lmax, int dtype, void* stream);

/* Causal GQA decode attention of the step's S tokens against the cache
 * (keys 0..pos0[b]+s for token s), split over 64-key chunks; the last CTA of
 * a KV head merges the chunks. part: csaq_attention_workspace_floats floats;
 * tickets: B*Hkv int32, zero before the first call (calls leave them zero).
 * D must be 64 or 128 (Qwen1.5-0.5B-shaped and Llama-shaped heads). */
int64_t csaq_attention_workspace_floats(int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D,
                                        int64_t Lmax);
int csaq_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                          const int32_t* pos0, int64_t B, int64_t S, int64_t Hq, int64_t Hkv,
                          int64_t D, int64_t Lmax, float scale, float* part, int32_t* tickets,
                          void* out, int dtype, void* stream);

/* Tensor-parallel combine: out[m, n] = T(out[m, n] (when add_out) + sum over
 * r of parts[r*part_stride + m*ld_parts + n]), summed in fp32 in rank order.
 * Replaces the all-reduce after the row-split o/down projections (the
 * reference has no multi-GPU path; this is the combine step of its linears). */
int csaq_rank_sum(const void* parts, int n_parts, int64_t part_stride, int64_t ld_parts, void* out,
                  int64_t ldo, int64_t M, int64_t N, int add_out, int dtype, void* stream);

/* ── Tensor-parallel combine over NVLink peer memory ─────────────────────
 * No counterpart in the reference (it has no multi-GPU path); these replace
 * the NCCL all-gather + csaq_rank_sum pair after the row-split o/down
 * projections with one kernel per rank that reads the peers' partials over
 * NVLink. Buffers come from csaq_p2p_alloc (cudaMalloc, zeroed) and are
 * mapped into the other ranks' processes with csaq_ipc_handle/csaq_ipc_open
 * (the handles travel over the caller's process group). */
#define CSAQ_MAX_RANKS 8
#define CSAQ_IPC_HANDLE_BYTES 64

typedef struct csaq_p2p_group {
  int32_t n_ranks, rank;
  const void* parts[CSAQ_MAX_RANKS]; /* rank r's partial buffer, as mapped in this process */
  uint64_t* flags[CSAQ_MAX_RANKS];   /* rank r's flag array (n_ranks u64), as mapped here  */
  uint64_t* seq;                     /* this rank's exchange count (device, starts at 0)   */
  uint32_t* ticket;                  /* this rank's CTA ticket (device, starts at 0)       */
  uint32_t* err;                     /* this rank's abandoned-wait counter (device)        */
} csaq_p2p_group;

int csaq_p2p_alloc(int64_t bytes, void** ptr);
int csaq_p2p_free(void* ptr);
int csaq_ipc_handle(const void* ptr, uint8_t* handle);
int csaq_ipc_open(const uint8_t* handle, void** ptr);
int csaq_ipc_close(void* ptr);

/* out[m, n] = T(out[m, n] + sum over r of parts[r][part_offset + m*ld_parts + n])
 * in fp32, in rank order: csaq_rank_sum over the ranks' own buffers. Every
 * rank launches it for the same exchange in the same order; it signals the
 * peers that this rank's partial is complete and waits (bounded; an
 * abandoned wait counts in *err, read with csaq_p2p_errors) for theirs. A
 * rank may rewrite a partial buffer only after the next exchange. */
int csaq_tp_exchange_sum(const csaq_p2p_group* group, int64_t part_offset, int64_t ld_parts, void* out,
                         int64_t ldo, int64_t M, int64_t N, int dtype, void* stream);
/* csaq_tp_exchange_sum followed by csaq_rmsnorm of its result in one launch
 * (one CTA per row), bit for bit the two calls: out as above, then
 * xn[m, :] = RMSNorm(out[m, :]) with weights norm_w (N values) and eps. For
 * the combine after a row-split o/down projection that the next layer norm
 * reads. */
int csaq_tp_exchange_sum_rmsnorm(const csaq_p2p_group* group, int64_t part_offset, int64_t ld_parts,
                                 void* out, int64_t ldo, int64_t M, int64_t N, const void* norm_w,
                                 void* xn, int64_t ldn, float eps, int dtype, void* stream);
int csaq_p2p_errors(const csaq_p2p_group* group, int64_t* count);
/* Polls of a peer flag before csaq_tp_exchange_sum gives up its wait (default
 * 2^22, a few seconds), for launches made after the call (a captured graph
 * keeps the value it was captured with); polls >= 1. No counterpart in the
 * reference (it has no multi-GPU path). */
int csaq_p2p_set_spin_limit(int64_t polls);

/* Greedy token of each row: the global index of the largest logit over
 * n_parts vocabulary slices of part_len values (slice r at r*part_stride,
 * rows ld apart), the smallest index on ties; torch.argmax of the sampler
 * at temperature 0 (csaq/inference.py:269-304). */
int csaq_argmax_parts(const void* logits, int n_parts, int64_t part_stride, int64_t ld, int64_t part_len,
                      int64_t M, int64_t* idx, int dtype, void* stream);

/* csaq_rope_kv followed by csaq_decode_attention in one launch, bit for bit:
 * q, k, v are the step's unrotated queries and keys and its values, rows `ld`
 * elements apart (row slices of one fused q/k/v buffer); the new keys are
 * rotated and, with the values, written to the caches at positions
 * pos0[b] .. pos0[b]+S-1; the queries are rotated in registers (no rotated
 * copy is written). Same part/tickets contract as csaq_decode_attention.
 * Needs 16-byte aligned q/k/v/caches/tables and ld % 8 == 0 (else
 * CSAQ_ERR_UNSUPPORTED). No counterpart in the reference (HF applies the
 * rotary embedding and attention as separate ops, csaq/inference.py:443-474). */
int csaq_decode_attention_rope(const void* q, const void* k, const void* v, int64_t ld, const int32_t* pos0,
                               int64_t B, int64_t S, int64_t Hq, int64_t Hkv, int64_t D, const float* cos_t,
                               const float* sin_t, void* k_cache, void* v_cache, int64_t Lmax, float scale,
                               float* part, int32_t* tickets, void* out, int dtype, void* stream);

/* csaq_decode_attention for callers that cannot allocate device memory: a
 * host-language binding that is handed raw device pointers (q, the caches,
 * pos0, out) by an application owning all device memory, or a
 * latency-critical caller for which cudaMalloc/cudaFree (which may
 * synchronise the device) are not acceptable. No counterpart in the reference
 * (its attention is the HF module's, allocating through PyTorch).
 *
 * Same arguments and results as csaq_decode_attention minus `part` and
 * `tickets`: those live in a fixed CSAQ_ATTENTION_STATIC_SCRATCH_BYTES buffer
 * inside the library, one per device. The buffer starts with
 * CSAQ_ATTENTION_STATIC_MAX_HEADS int32 tickets, which every completed call
 * leaves at zero whatever its shape; the partial softmax results follow. A
 * call with B*Hkv above CSAQ_ATTENTION_STATIC_MAX_HEADS, or whose partials
 * (csaq_attention_workspace_floats floats) do not fit after the tickets,
 * returns CSAQ_ERR_SCRATCH before anything is enqueued. The first call on
 * each device sets the buffer up (looks up its address and zero-fills it,
 * synchronously); make that first call before any stream capture (during a
 * capture it returns CSAQ_ERR_UNSUPPORTED). The set-up is done once per
 * process: after cudaDeviceReset, reload the library. Calls on one device
 * share the buffer, so calls that can overlap on the GPU (other streams,
 * other host threads) race; calls ordered on one stream do not. */
#define CSAQ_ATTENTION_STATIC_SCRATCH_BYTES (4 << 20)
#define CSAQ_ATTENTION_STATIC_MAX_HEADS 1024
int csaq_decode_attention_static(const void* q, const void* k_cache, const void* v_cache,
                                 const int32_t* pos0, int64_t B, int64_t S, int64_t Hq, int64_t Hkv,
                                 int64_t D, int64_t Lmax, float scale, void* out, int dtype, void* stream);

/* HF LlamaMLP gate: h = dtype(silu(g)) * u. */
int csaq_silu_mul(const void* g, int64_t ldg, const void* u, int64_t ldu, void* h, int64_t ldh,
                  int64_t M, int64_t N, int dtype, void* stream);

/* Greedy acceptance of one self-speculative block on the device: the fixed
 * form of csaq/inference.py:482-549 (draft token k is compared with the
 * verifier's prediction at position k, and the verifier's token after the
 * accepted prefix is appended). */
int csaq_spec_accept(const int64_t* draft, const int64_t* verify_argmax, int64_t B, int64_t K,
                     int32_t* pos0, int64_t* out_tokens, int32_t* n_out, int64_t cap,
                     int64_t* next_tok, int32_t* n_new, int64_t* stats, int32_t* remaining,
                     void* stream);

/* ── Sampling at temperature > 0 (csaq/inference.py:269-304, :482-518) ────
 * Logit rows are given as n_parts vocabulary slices of part_len values
 * (slice r at r*part_stride, rows ld apart; one part for a single GPU).
 * counter: two u64 in device memory, zero before the first call; each call
 * advances counter[0] so that graph replays draw new numbers (Philox, seed). */
int csaq_sample_rows(const void* logits, int n_parts, int64_t part_stride, int64_t ld, int64_t part_len,
                     int64_t rows, float temperature, float top_p, uint64_t seed, uint64_t* counter, int64_t* out,
                     int dtype, void* stream);
/* vt (B x (K+1)) for csaq_spec_accept from the draft tokens (B x K), the
 * draft steps' full-vocabulary logits (K x B x V, contiguous) and the verify
 * logits (rows b*(K+1)+k): rejection sampling of each draft token, a residual
 * draw at the first rejection, a bonus draw when all are accepted. */
int csaq_spec_sample_verify(const int64_t* draft, const void* draft_logits, const void* verify_logits, int n_parts,
                            int64_t part_stride, int64_t ld, int64_t part_len, int64_t B, int64_t K,
                            float temperature, float top_p, uint64_t seed, uint64_t* counter, int64_t* vt,
                            int dtype, void* stream);

/* Bookkeeping of one plain greedy decode step: append the argmax token and
 * advance the position, what the standard mode's model.generate does per
 * token (csaq/inference.py:383). */
int csaq_greedy_commit(const int64_t* tok, int64_t B, int32_t* pos0, int64_t* out_tokens,
                       int32_t* n_out, int64_t cap, int64_t* next_tok, int32_t* remaining,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CSAQ_B200_H */
