/*
 * spark_b200.h -- C ABI of the B200 (sm_100a) batch-1 decode hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t (passed
 * as void*), launches on that stream, never synchronises, never allocates, and
 * returns a status code (0 = success, see SPARK_* below).  All entry points are
 * safe to capture into a CUDA graph.  bf16 / fp16 tensors are passed as uint16_t
 * bit patterns.
 *
 * Q4_0 weights are stored as two planes (a lossless split of the gguf block
 * layout [rows][K/32][2-byte fp16 d | 16 nibble bytes]):
 *   qs  uint8  [rows][K/2]   nibble bytes, gguf order (byte j: low = element j,
 *                            high = element j+16 of the 32-element block)
 *   d   fp16   [rows][K/32]  block scale, w = d * (q - 8)
 *
 * The reference's host boundary is the torch custom op spark_v43::layer_run
 * (src/spark_vllm_ascend/integration/model.py:46-82) which hands a flat tensor
 * list to the compiled DecodeLayer megakernel (integration/model.py:118-139,
 * kernels/layer.py:48-109).  This ABI replaces that monolith with one entry
 * point per fused stage; each declaration names the reference code it replaces.
 */
#ifndef SPARK_B200_H
#define SPARK_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPARK_OK 0
#define SPARK_ERR_INVALID_ARG 1
#define SPARK_ERR_UNSUPPORTED_SHAPE 2
#define SPARK_ERR_ALIGNMENT 3
#define SPARK_ERR_LAUNCH 4
#define SPARK_ERR_TOO_LARGE 5
#define SPARK_ERR_CUDA 6 /* a CUDA runtime call (allocation, IPC) failed */

/* Library version (major * 10000 + minor * 100 + patch). */
int spark_version(void);

/* Human readable text for a status code. */
const char* spark_status_string(int status);

/* Q4_0 quantization of fp32 weights [rows][k] on the device, bit-identical to
 * gguf 0.19.0 quants.Q4_0.quantize_blocks (third-party; the reference calls it
 * through gguf.quants at integration/weights.py:30 and
 * tools/deployment/prepare_model.py:63).  k % 32 == 0. */
int spark_q4_quantize(const float* w, int64_t rows, int64_t k, uint8_t* qs, uint16_t* d, void* stream);

/* Split gguf Q4_0 block bytes [rows][k/32][18] into the qs / d planes.
 * Replaces the repack in integration/weights.py:34-54 (unpack_q4 + pack). */
int spark_q4_split_gguf(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* qs, uint16_t* d, void* stream);

/* Dequantize to bf16 [rows][k] (w = d * (q - 8), rounded to bf16).  Used by
 * prefill-side matmuls; replaces gguf dequantize -> bf16 at integration/weights.py:28-32. */
int spark_q4_dequantize_bf16(const uint8_t* qs, const uint16_t* d, int64_t rows, int64_t k, uint16_t* w,
                             void* stream);

/* Prefill GEMM on the tensor cores: y[t][n] = bf16(sum_k W[n][k] * x[t][k]) for t < T
 * tokens, W the Q4_0 planes [n][k] dequantized to bf16 in shared memory (the same
 * rounding as spark_q4_dequantize_bf16), fp32 accumulation (tcgen05.mma; activation and
 * weight tiles brought in by TMA).  Replaces the prefill's dequantize -> bf16 matmul
 * (integration/weights.py:28-31 and vLLM's torch linear layers,
 * integration/model.py:50-62) without the bf16 weight copy.  k % 256 == 0; x [T][k]
 * bf16, qs and d 16-B aligned.  Each wait inside the kernel is bounded by wait_ns
 * (< 0: the default 0.5 s; 0: give up at the second look, for testing the error path).
 * *error (caller-owned, required) becomes 1 when a wait ran out (y is then not valid);
 * the CTA still waits, with a fixed 2 s bound, for the copies and MMAs it issued before
 * it frees its shared and tensor memory.  2 means that drain ran out too and the CTA
 * kept its tensor memory: the CUDA context must then be treated as unusable. */
int spark_q4_gemm_tc(const uint16_t* x, const uint8_t* qs, const uint16_t* d, uint16_t* y, int t, int n, int k,
                     int* error, int64_t wait_ns, void* stream);

/* y[b][n] = bf16(sum_k W[n][k] * x[b][k]) for b < batch (1..8); fp32 accumulation
 * in the fixed order documented in q4_gemv.cuh.  n even, k % 32 == 0.
 * Replaces GemvStage.calculate (kernels/linear.py:17-200) as used by
 * NativeLinear.execute_o / execute_down (linear.py:339-370). */
int spark_q4_gemv(const uint16_t* x, const uint8_t* qs, const uint16_t* d, uint16_t* y, int n, int k, int batch,
                  void* stream);

/* Fused add + RMSNorm prologue + Q4_0 GEMV: s = a + b (b may be NULL),
 * res_out = bf16(s) (may be NULL), x = bf16(s / rms(s) * gamma), y = W x.
 * Replaces norm_ub (kernels/linear.py:202-224) feeding the gate_up GEMV
 * (NativeUp.execute, linear.py:585-611) and the next layer's input norm
 * (NativePool.final_norm, linear.py:298-305). */
int spark_rmsnorm_q4_gemv(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps, uint16_t* res_out,
                          const uint8_t* qs, const uint16_t* d, uint16_t* y, int n, int k, void* stream);

/* Fused add + RMSNorm + gate_up Q4_0 GEMV + SiLU*mul: rows [0, n/2) are gate,
 * [n/2, n) up; mid[i] = bf16(bf16(silu(g_i)) * u_i).
 * Replaces NativeUp.execute + FusedUpStage.activate (kernels/linear.py:228-260,
 * 540-611; the reference's activation is GELU, the synthetic model's SwiGLU). */
int spark_rmsnorm_gate_up_silu(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps,
                               uint16_t* res_out, const uint8_t* qs, const uint16_t* d, uint16_t* mid, int n, int k,
                               void* stream);

/* Fused input norm + QKV Q4_0 GEMV + neox RoPE + paged K/V store.
 * a: bf16 [k] or, when embed != NULL, the row embed[token[0]] (token int32 on device).
 * Rows of W: nq*head_dim query rows, then nkv*head_dim key rows, then value rows.
 * cos_sin: bf16 [max_pos][head_dim] (cos in the first half, sin in the second).
 * Position from pos (int64 on device).  The KV slot is slot_mapping[0] when
 * slot_mapping != NULL, else block_table[pos / block_size] * block_size + pos % block_size
 * (a negative slot skips the store).  q_out: bf16 [nq][head_dim] (rotated).
 * Replaces FusedQkvStage.execute_fused + calculate_rotated + store8
 * (kernels/qkv.py:25-236) and the slot computation of integration/slot_mapping.py:8-22. */
int spark_qkv_rope_kvstore(const uint16_t* a, const uint16_t* b, const uint16_t* embed, const int32_t* token,
                           const uint16_t* gamma, float eps, uint16_t* res_out, const uint8_t* qs, const uint16_t* d,
                           int k, int nq, int nkv, int head_dim, const uint16_t* cos_sin, const int64_t* pos,
                           const int32_t* block_table, const int64_t* slot_mapping, int block_size,
                           uint16_t* k_cache, uint16_t* v_cache, uint16_t* q_out, void* stream);

/* Split-KV paged GQA decode attention (partials).  q bf16 [nq][head_dim];
 * caches bf16 [num_blocks][nkv][block_size][head_dim]; sequence length =
 * seq_len[0] (int32) when seq_len != NULL else pos[0] + 1 (int64).
 * Split s covers tokens [s*T, min((s+1)*T, L)), T = roundup16(ceil(L / splits)),
 * and T must not exceed max_split_tokens (sizes shared memory; <= 2048).
 * part_o fp32 [splits][nq][head_dim], part_lse fp32 [splits][nq] (-inf for
 * empty splits).  error (int on device, may be NULL) is set to 1 when a split
 * exceeds max_split_tokens at run time; the split is then written as empty.
 * head_dim 128 and nq / nkv == 4 are supported.
 * Replaces AttentionStage.execute_serial / execute_pipeline (kernels/attention.py:120-286). */
int spark_attn_splitkv(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                       const int32_t* block_table, const int64_t* pos, const int32_t* seq_len, int nq, int nkv,
                       int head_dim, int block_size, int splits, int max_split_tokens, float scale, float* part_o,
                       float* part_lse, int* error, void* stream);

/* Split-KV attention with the log-sum-exp combine fused in: same inputs and
 * partial outputs as spark_attn_splitkv (part_o / part_lse are the caller's
 * workspace), plus counters (int [nkv] on device, all zero before the first call;
 * the kernel leaves them zero again) and out (bf16 [nq][head_dim]).  The CTA
 * that finishes last for a kv head merges that head's splits in the same order
 * as spark_attn_combine, so out is bit-identical to split + combine.
 * splits <= 256.  Replaces AttentionStage.execute (kernels/attention.py:120-286)
 * followed by merge_attention (kernels/vector.py:46-83). */
int spark_attn_decode(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                      const int32_t* block_table, const int64_t* pos, const int32_t* seq_len, int nq, int nkv,
                      int head_dim, int block_size, int splits, int max_split_tokens, float scale, float* part_o,
                      float* part_lse, int* counters, uint16_t* out, int* error, void* stream);

/* spark_attn_decode for callers that cannot allocate device memory (a host
 * framework that owns all GPU memory and lends none to plugins, or a loop that must
 * not call cudaMalloc after start-up, since it can synchronise the device or fail
 * under memory pressure).  No counterpart in the reference: this entry point is an
 * addition of this library.  Same inputs, output and numerics as spark_attn_decode,
 * but the partials, lse values and arrival counters live in a static device array
 * inside the library (2,113,792 bytes, held by every GPU that loads the library
 * until the process exits), so the caller passes no workspace.
 * Limits: splits <= 64, nq <= 64, nkv <= 64 (else SPARK_ERR_TOO_LARGE); otherwise
 * as spark_attn_decode (head_dim 128, nq == 4 * nkv, max_split_tokens <= 2048).
 * The first call on a device looks up the array's device address and zeroes its
 * counters, a synchronous step: make that first call before any stream capture.
 * All calls on one device share the array and it keeps the last call's contents;
 * calls that can overlap on the GPU (e.g. on different streams with no ordering
 * between them) race and corrupt each other's results, so order them on one stream.
 * Each device has its own copy.  Allocates nothing. */
int spark_attn_decode_noalloc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                              const int32_t* block_table, const int64_t* pos, const int32_t* seq_len, int nq,
                              int nkv, int head_dim, int block_size, int splits, int max_split_tokens, float scale,
                              uint16_t* out, int* error, void* stream);

/* Log-sum-exp combine of split partials -> bf16 [nq][head_dim].
 * Replaces merge_attention (kernels/vector.py:46-83) without the output gate. */
int spark_attn_combine(const float* part_o, const float* part_lse, int splits, int nq, int head_dim, uint16_t* out,
                       void* stream);

/* Final norm + LM head Q4_0 GEMV + greedy argmax.  logits bf16 [n]; argmax_key
 * (uint64 on device) must hold 0 before the call; afterwards its low 32 bits are
 * ~index of the largest logit (lowest index on ties).  Replaces the head GEMV path
 * (integration/head.py:6-16, native/head/extension.cpp:7-14) for a Q4_0 head. */
int spark_rmsnorm_q4_head_argmax(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps,
                                 const uint8_t* qs, const uint16_t* d, uint16_t* logits, int n, int k,
                                 unsigned long long* argmax_key, void* stream);

/* Decode bookkeeping after the head: token = index in argmax_key; writes
 * token_out[0] (int32, the next step's input) and, when token_log != NULL,
 * token_log[step[0]]; resets argmax_key to 0; increments pos[0] and step[0]
 * when they are non-NULL. */
int spark_decode_finalize(unsigned long long* argmax_key, int32_t* token_out, int32_t* token_log, int32_t* step,
                          int64_t* pos, void* stream);

/* Standalone fused add + RMSNorm (hidden <= 16384): res_out = bf16(a + b),
 * y = bf16((a+b) / rms * gamma).  Replaces norm_ub (kernels/linear.py:202-224). */
int spark_add_rmsnorm(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps, int hidden,
                      uint16_t* res_out, uint16_t* y, void* stream);

/* SiLU * mul over n elements: out = bf16(bf16(silu(g)) * u).  The synthetic
 * model's SwiGLU counterpart of FusedUpStage.activate (kernels/linear.py:228-260). */
int spark_silu_mul(const uint16_t* g, const uint16_t* u, int64_t n, uint16_t* out, void* stream);

/* In-place neox RoPE on bf16 heads [nh][head_dim] at position pos[0] (int64).
 * Replaces the rotation in FusedQkvStage.calculate_rotated (kernels/qkv.py:179-189). */
int spark_rope_neox(uint16_t* x, int nh, int head_dim, const uint16_t* cos_sin, const int64_t* pos, void* stream);

/* Prefill helpers over `rows` tokens at once.  The reference prefills with vLLM's torch
 * layers (integration/model.py:50-62); these replace the torch element-wise steps of the
 * batched prefill (spark_b200/prefill.py).  add + RMSNorm per row (hidden <= 12288,
 * res_out nullable): res_out = bf16(a + b), y = bf16((a+b) * rsqrt(mean((a+b)^2) + eps)
 * * gamma).  RoPE in place on `nh` heads of each row (row r at x + r * row_stride,
 * position pos0 + r; pairs (i, i + rotary_dim / 2), cos_sin rows of rotary_dim). */
int spark_add_rmsnorm_rows(const uint16_t* a, const uint16_t* b, const uint16_t* gamma, float eps, int rows,
                           int hidden, uint16_t* res_out, uint16_t* y, void* stream);
int spark_rope_neox_rows(uint16_t* x, int64_t row_stride, int rows, int nh, int head_dim, int rotary_dim,
                         const uint16_t* cos_sin, int64_t pos0, void* stream);
/* Activation * mul per row of a fused gate / up output gu bf16 [rows][2 inter]:
 * out bf16 [rows][inter] = bf16(act(gate) * up) with the decode epilogues' arithmetic:
 * bf16 SiLU (gelu_table NULL) or the GELU table of SPARK_EPI_GELU_MUL. */
int spark_act_mul_rows(const uint16_t* gu, int rows, int inter, const uint16_t* gelu_table, uint16_t* out,
                       void* stream);

/* Store this step's keys and values into the paged caches: k / v bf16
 * [tokens][nkv][head_dim] -> k_cache / v_cache bf16 [blocks][nkv][block_size][head_dim]
 * at slot_mapping[t] (int64; negative = padding, skipped).  head_dim % 8 == 0, 16-byte
 * aligned tensors.  Replaces the KV write of the reference's attention layer
 * (the slot scatter of FusedQkvStage.store8, kernels/qkv.py:192-198) for callers that
 * rotate q / k themselves (the vLLM attention backend). */
int spark_kv_store(const uint16_t* k, const uint16_t* v, const int64_t* slot_mapping, int64_t tokens, int nkv,
                   int head_dim, int block_size, uint16_t* k_cache, uint16_t* v_cache, void* stream);

/* Paged-KV slot mapping for one request (single KV group):
 * out[i] = table[pos[i] / block_size] * block_size + pos[i] % block_size for
 * i in [query_start[0], query_start[1]) and i < num_tokens, else -1, for all
 * i < max_tokens.  Replaces _slot_one (integration/slot_mapping.py:8-22). */
int spark_slot_mapping(int64_t num_tokens, int64_t max_tokens, const int32_t* query_start, const int64_t* positions,
                       const int32_t* block_table, int64_t block_size, int64_t* out, void* stream);

/* Enable / disable programmatic dependent launch on the kernels above (default on). */
int spark_set_pdl(int enabled);

/* Select the Q4_0 GEMV implementation for shapes with K % 512 == 0 and batch 1:
 * 1 (default) = persistent kernel streaming weights through a cp.async.bulk
 * shared-memory ring, 0 = register-direct kernel.  Both compute the same order
 * and give bit-identical results. */
int spark_set_gemv_ring(int enabled);

/* Copy the library's device error word to *value (synchronous; diagnostics only)
 * and clear it when reset != 0.  Non-zero means a kernel gave up a bounded wait
 * (2/3: producer side, 4: consumer side of the ring GEMV); outputs of that launch
 * are then incomplete. */
int spark_read_device_error(int* value, int reset);

/* ======================================================================
 * Persistent decode step.
 *
 * Replaces the reference's per-layer DecodeLayer launch (integration/model.py:
 * 118-139; kernels/layer.py:48-109 chains qkv, attention, o, gate_up and down in
 * one compiled program per layer) with ONE cooperative kernel per decode step
 * that runs a program of stages over all SMs.  Each SM streams the Q4_0 weights
 * of its share of every GEMV stage (and the K/V pages of its attention split)
 * through a shared-memory ring with bulk copies, running ahead of the stage
 * barriers, so HBM keeps streaming while the stages synchronise.
 *
 * Weights use the T16 layout (spark_q4_pack_t16): units of 16 rows x K/kp
 * columns, 9 * K/kp bytes each, laid out for the integer tensor-core dot
 * product of a Q4_0 block.  Unit u covers row group u / kp and K part u % kp.
 * ====================================================================== */

#define SPARK_STAGE_GEMV 0
#define SPARK_STAGE_ATTN 1  /* head_dim 128; 256 with the Spark layer features (a program using any of
                               them takes head_dim 256 attention only) */
#define SPARK_STAGE_GEMV_Q6 2  /* GEMV over Q6_K weights in the T6 layout (spark_q6k_pack_t6); rowmap
                                  SPARK_ROWS_PLAIN, (k / kp) % 256 == 0, otherwise as SPARK_STAGE_GEMV */

/* GEMV prologue: where x comes from */
#define SPARK_XCHG_TAGGED 2
#define SPARK_PRO_BF16 0  /* a: bf16 [k] (or embed row embed[*token] when embed != NULL) */
#define SPARK_PRO_PARTS 1 /* a: fp32 [a_parts][k]; x = bf16(((a_0 + a_1) + ...)) */
#define SPARK_PRO_PARTS_TAGGED 3 /* a: uint64 [a_parts][k] tagged parts written by a SPARK_XCHG_TAGGED stage:
                                   word = fp32 bits | tag << 32, tag = launch + 1 (launch =
                                   io->counters[num_stages + 2]); the prologue waits (bounded) for each
                                   word's tag, then x = bf16(((a_0 + a_1) + ...)).  `wait` orders the
                                   stage's other inputs (residual) and names no tagged stage */
#define SPARK_PRO_ATTN 2  /* o_proj fused behind the attention stage just before it (wait = -1, no norm,
                             kp = that stage's nkv, k = nq * head_dim, splits = its splits, nkv * splits
                             <= CTAs): CTA c takes K part g = c / splits (kv head g) of the row groups
                             c % splits + splits * m, its input being head g's combined attention output,
                             which the attention stage combines in every CTA of the head and leaves staged
                             in shared memory (attn_out is then not written, and no stage may wait on the
                             attention stage); a is unused */

/* GEMV epilogue */
#define SPARK_EPI_BF16 0     /* out bf16 [n] (kp == 1) */
#define SPARK_EPI_PARTS 1    /* out fp32 [kp][n], the per-part sums */
#define SPARK_EPI_ROPE_KV 2  /* qkv: neox RoPE on q/k, q -> q, k/v -> paged cache + kv_new */
#define SPARK_EPI_SILU_MUL 3 /* gate_up: out bf16 [n/2] = silu(gate) * up */
#define SPARK_EPI_ARGMAX 4   /* LM head: logits bf16 [n] (out, nullable), atomicMax into key */
#define SPARK_EPI_GELU_MUL 5 /* gate_up (Spark MLP): out bf16 [n/2] = bf16(gelu(bf16 gate) * up), gelu from
                                `table` (see SparkStage.table) */

/* logical rows of unit position p (0..15) of row group rg */
#define SPARK_ROWS_PLAIN 0     /* 16 rg + p */
#define SPARK_ROWS_PAIR_HALF 1 /* qkv heads: per head, rotary pairs (i, i + r/2) in positions (p, p + 8)
                                  (r = rotary_dim, or head_dim when 0), then the head's dims r.. in
                                  plain runs of 16; rows past the last whole head (the gate rows)
                                  plain */
#define SPARK_ROWS_GATE_UP 2   /* gate row 8 rg + p and up row n/2 + 8 rg + p in positions (p, p + 8) */

typedef struct SparkStage {
  int32_t kind, pro, epi, rowmap;
  int32_t n, k, kp, ks;         /* GEMV rows, columns, K parts, slices per part (<= 4) */
  int32_t units, rot, wait, norm; /* units = n/16*kp; rot = first CTA; wait = stage to await (-1) */
  int32_t a_parts, block_size, nq, nkv;
  int32_t head_dim, splits, max_split_tokens;
  int32_t xchg;               /* tensor-parallel exchange stage (io->tp_size > 1): SPARK_EPI_PARTS writes
                                 its part as part tp_rank * kp + kpi of `out` in EVERY rank's exchange
                                 window, SPARK_EPI_ARGMAX takes the maximum into every rank's key, and
                                 the stage's completion is counted on every rank; 0: local stage;
                                 SPARK_XCHG_TAGGED (EPI_PARTS only): the parts go to every rank as tagged
                                 64-bit words (see SPARK_PRO_PARTS_TAGGED) and the stage is not counted:
                                 its readers wait on the words themselves, no stage may wait on it */
  float eps, inv_k, scale;
  int32_t row0;               /* SPARK_EPI_ARGMAX: global index of row 0 (vocab shard start), else 0 */
  const void* w;              /* T16 weight units */
  const void* a;              /* input (see SPARK_PRO_*) */
  const void* b;              /* residual added before the norm (nullable) */
  const void* embed;          /* bf16 [vocab][k]: layer-0 input row *token (nullable) */
  const int32_t* token;
  const void* gamma;          /* RMSNorm weight (used when norm != 0) */
  void* res_out;              /* bf16(a + b) (nullable) */
  void* out;
  const void* cos_sin;        /* bf16 [max_pos][head_dim]: cos | sin */
  const int64_t* pos;         /* position of the token being decoded */
  const int32_t* block_table; /* int32 logical -> physical KV block */
  void* k_cache;              /* bf16 [blocks][nkv][block_size][head_dim] (this layer) */
  void* v_cache;
  void* q;                    /* bf16 [nq][head_dim] */
  void* kv_new;               /* bf16 [2][nkv][head_dim]: this token's k and v */
  unsigned long long* key;    /* argmax key (zero before the stage) */
  float* part_o;              /* fp32 [splits][nq][head_dim] */
  float* part_lse;            /* fp32 [splits][nq] */
  int32_t* head_counters;     /* int32 [nkv] of this stage alone, zero when io->counters was zeroed;
                                 grows by `splits` per launch */
  void* attn_out;             /* bf16 [nq][head_dim] */
  /* Spark layer features (zero / NULL: off) */
  int32_t rotary_dim;         /* SPARK_EPI_ROPE_KV: dims rotated per head (partial RoPE, pairs (i, i + r/2)),
                                 cos_sin rows of r entries; 0: head_dim */
  int32_t window;             /* SPARK_STAGE_ATTN: attend to the last `window` positions only (sliding) */
  const void* table;          /* SPARK_EPI_GELU_MUL: bf16 [4096] gelu of the bf16 inputs 0x3b00 + i (i < 2048)
                                 and 0xbb00 + i - 2048 (|x| in [2^-9, 128)); outside that range gelu is
                                 x / 2 (|x| < 2^-9), x (x >= 128), -0 (x <= -128) */
  void* gate;                 /* bf16 [nq] headwise output gate: SPARK_EPI_ROPE_KV computes it from its
                                 gate rows (rows (nq + 2 nkv) head_dim + h, h < nq, padded to 16 rows):
                                 bf16(1 / (1 + exp(-bf16(logit)))); SPARK_STAGE_ATTN multiplies head h's
                                 combined output by it: bf16(bf16(o) * gate[h]) */
  /* Small-batch decode: B sequences through one launch (the weights stream once, each
   * integer MMA of a Q4_0 block multiplies the B sequences' digit columns together). */
  int32_t batch;              /* B: 0 or 1 = one sequence; 2, 4 or 8, the same in every stage of a program.
                                 Every per-sequence buffer then holds B copies of its one-sequence layout,
                                 sequence-major: a, b, res_out, out (SPARK_EPI_PARTS: [B][kp][n]), q,
                                 kv_new, part_o, part_lse, head_counters and attn_out hold sequence s at
                                 s times their one-sequence size; token, pos and key hold B entries.
                                 Each sequence's result is bit-identical to decoding it alone with the
                                 same program.  Not combined with tensor parallelism, Q6_K stages, the
                                 Spark features or SPARK_PRO_ATTN; ks <= 2 */
  int32_t bt_stride;          /* batch > 1: block_table is int32 [B][bt_stride] (sequence s's logical ->
                                 physical blocks at s * bt_stride) */
} SparkStage;

typedef struct SparkStepIO {
  int32_t* counters;          /* int32 [num_stages + 3], zero before the first launch; the kernel keeps
                                 the first num_stages + 2 zero between launches and counts launches in
                                 the last (the attention stages' head counters follow that count) */
  int32_t* error;             /* int32 [1] status written on a timed-out wait (nullable) */
  unsigned long long* key;    /* [B] after the last stage: token = argmax of key (nullable) */
  int32_t* token_out;         /* [B] (B = the last stage's batch) */
  int32_t* token_log;         /* token_log[*step * B + s] = sequence s's token (nullable) */
  int32_t* step;              /* incremented (nullable) */
  int64_t* pos;               /* [B], each incremented (nullable) */
  unsigned long long* trace;  /* optional uint64 [ctas][num_stages][8] globaltimer stamps (ns): consumer
                                 wait start, work start, work end, producer's first copy of the stage,
                                 then stage checkpoints (GEMV: tasks start, tasks end; attention:
                                 scores, softmax, PV, partials written); for profiling, nullable */
  /* Tensor parallelism (one process per GPU, tp_size ranks; tp_size <= 1: single GPU).
   * Each rank owns an exchange window (device memory holding `counters`, the parts
   * buffers of the exchange stages and `key`), mapped into every peer's address space;
   * a peer's copy of a window address is peer_windows[p] + (address - window).
   * With tp_size > 1 the stage counters are never reset: a stage is complete once its
   * counter reaches contributors * (launch + 1), contributors = CTAs * tp_size for an
   * exchange stage, CTAs otherwise (launch = io->counters[num_stages + 2]). */
  const unsigned long long* peer_windows; /* device uint64 [tp_size]: window base as mapped here */
  const void* window;                     /* this rank's window base (host-visible value) */
  unsigned long long window_bytes;
  int32_t tp_size, tp_rank;
} SparkStepIO;

/* Bytes of a matrix in the T16 layout: n * k * 9 / 16. */
int64_t spark_t16_bytes(int n, int k, int kp);

/* Re-lay a Q4_0 matrix (qs / d planes) as T16 units.  rowmap SPARK_ROWS_*; aux =
 * head_dim for SPARK_ROWS_PAIR_HALF, unused otherwise.  Needs n % 16 == 0,
 * (k / kp) % 64 == 0.  Replaces the reference's offline packer
 * (integration/weights.py:42-55, pack into its megakernel tile layout). */
int spark_q4_pack_t16(const uint8_t* qs, const uint16_t* d, int n, int k, int kp, int rowmap, int aux, uint8_t* out,
                      void* stream);

/* Q6_K weights for the persistent step (the reference's Q6_K LM head over the tied
 * embedding, native/head/head_q6.asc + integration/head.py:6-31, repacked by
 * tools/deployment/prepare_head.py:11-28).  `blocks` are gguf Q6_K rows, uint8
 * [n][k / 256 * 210] (super-blocks of 256 weights: 128 B low nibbles, 64 B 2-bit high
 * parts, 16 int8 sub-block scales, fp16 d).  The T6 layout cuts the matrix into units
 * of 16 rows x k / kp columns, 105 (k / kp) / 8 bytes each, laid out for the integer
 * tensor-core dot product of 32 weights (see csrc/step_kernel.cuh); lossless.
 * spark_q6k_dequantize decodes gguf blocks to fp32 exactly like gguf 0.19.0. */
int64_t spark_t6_bytes(int n, int k);
int spark_q6k_pack_t6(const uint8_t* blocks, int n, int k, int kp, uint8_t* out, void* stream);
int spark_q6k_dequantize(const uint8_t* blocks, int64_t nblocks, float* out, void* stream);

/* Shared memory the step kernel keeps for the weight / KV ring (bytes), one sequence. */
int spark_step_ring_bytes(void);

/* The same for a program of batch B (1, 2, 4 or 8); 0 for another B. */
int spark_step_ring_bytes_batch(int batch);

/* Number of CTAs (one per SM) the step kernel runs with on the current device. */
int spark_step_num_ctas(void);

/* Exchange windows for tensor parallelism (one process per GPU).  A window is plain
 * device memory from cudaMalloc (zeroed), so that its IPC handle maps the whole
 * buffer; handles are CUDA IPC handles (SPARK_IPC_HANDLE_BYTES bytes) that the host
 * side passes between the ranks (torch.distributed), and spark_ipc_open maps a
 * peer's window with peer access enabled.  No counterpart in the reference, whose
 * tensor-parallel path is vLLM's own (NCCL all-reduce after row-parallel layers). */
#define SPARK_IPC_HANDLE_BYTES 64
int spark_window_alloc(unsigned long long bytes, void** ptr);
int spark_window_free(void* ptr);
int spark_ipc_handle(const void* window, void* handle);
int spark_ipc_open(const void* handle, void** ptr);
int spark_ipc_close(void* ptr);

/* Run a stage program as one cooperative launch.  host_stages is validated on the
 * host; the kernel reads dev_stages (an identical copy in device memory), or, for
 * a single stage, dev_stages may be NULL and the stage travels in the launch
 * parameters.  Stage i may only wait on a stage j < i. */
int spark_step_run(const SparkStage* host_stages, const SparkStage* dev_stages, int num_stages,
                   const SparkStepIO* io, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPARK_B200_H */
