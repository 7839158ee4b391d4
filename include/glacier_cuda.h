/*
 * glacier_cuda.h -- C ABI of the B200 (sm_100a) INT4 decode library.
 *
 * This is the drop-in boundary for Glacier Engine's native kernel seam.  The
 * reference's Zig host declares its native kernels with `extern fn` and links
 * them statically (src/backends/cpu/int4_matmul.zig:29-204,
 * src/int4_executor.zig:33-61, src/decode_lane4.zig:221-264,
 * src/sampling.zig:17) and drives its GPU backend through a persistent-weight
 * handle API (src/backends/metal/backend.zig:571-595).  Every entry point
 * below names the reference interface it replaces.
 *
 * Conventions (kept from the reference seam):
 *  - plain pointers and sizes; no framework types cross the boundary;
 *  - functions return int status: 0 = ok, negative = error; on a validation
 *    error nothing is written (validation happens before any launch, as in
 *    PreparedQ8MatvecPlan.init, int4_matmul.zig:580-635);
 *  - "device" pointers live in GPU memory of the current device; `stream` is a
 *    cudaStream_t passed as void* (NULL = legacy default stream); work is
 *    enqueued asynchronously unless the function says it synchronises;
 *  - kernels keep no global state, so concurrent calls on different streams
 *    with disjoint outputs are safe (the reference executor calls its kernels
 *    concurrently on disjoint row ranges, int4_matmul.zig:693-726).
 */
#ifndef GLACIER_CUDA_H
#define GLACIER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GLACIER_CUDA_OK 0
#define GLACIER_CUDA_EINVAL (-1)       /* arguments rejected before any write */
#define GLACIER_CUDA_ECUDA (-2)        /* CUDA runtime / driver error */
#define GLACIER_CUDA_ENOMEM (-3)       /* device allocation failed */
#define GLACIER_CUDA_EMASK (-4)        /* sampling.zig:40 InvalidEligibleMask */
#define GLACIER_CUDA_ENAN (-5)         /* sampling.zig:41 EligibleLogitNaN */
#define GLACIER_CUDA_EUNSUPPORTED (-6) /* shape outside the kernels' contract */
#define GLACIER_CUDA_EFORMAT (-7)      /* .glacier container rejected; reason in glacier_cuda_format_error() */

/* Greedy reduction result; same 24-byte layout as glacier_argmax_result
 * (src/backends/cpu/int4_neon.c:8-19). */
typedef struct glacier_argmax_result {
  float value;
  size_t index;
  int valid;
  int saw_nan;
} glacier_argmax_result;

/* Thread-local message for the last failing call on this host thread. */
const char *glacier_cuda_last_error(void);

/* Library ABI version (major << 16 | minor). */
int glacier_cuda_version(void);

/* Number of kernels this library has launched in this process (all devices). */
unsigned long long glacier_cuda_launch_count(void);

/* Device-side status word of the current device: 0 = ok, 1 = a kernel gave up
 * a bounded wait (its outputs are invalid).  Synchronises the device.  clear != 0
 * resets the word.  No reference counterpart: the reference's CPU kernels
 * cannot stall; its Metal backend reports device loss through its lifecycle
 * contract (src/core/device_loss_*.zig). */
int glacier_cuda_device_status(int clear);

/* ------------------------------------------------------------------------
 * (a) INT4 group-dequant matvec, FP32 activations, on caller device buffers.
 * packed: row-major codes, two per byte, low nibble first, zero point 7
 * (src/core/quant.zig:164-177); scales: one per group along the flat element
 * index (src/model/qio.zig:15), i.e. [out_f, in_f/group] when rows hold whole
 * groups.  bias may be NULL.  y = x * dequant(W)^T + bias.
 * ---------------------------------------------------------------------- */

/* Replaces glacier_int4_matvec_neon_f32 (src/backends/cpu/int4_matmul.zig:29-38). */
int glacier_cuda_int4_matvec_f32(const float *x, const uint8_t *packed, const float *scales,
                                 const float *bias, float *y, size_t out_features,
                                 size_t in_features, size_t group_size, void *stream);

/* Replaces glacier_int4_matvec_neon_f16scale (src/backends/cpu/int4_matmul.zig:40-49);
 * scales are IEEE binary16 bit patterns. */
int glacier_cuda_int4_matvec_f16scale(const float *x, const uint8_t *packed,
                                      const uint16_t *scales, const float *bias, float *y,
                                      size_t out_features, size_t in_features,
                                      size_t group_size, void *stream);

/* Batched form of linearInt4OnTheFly (src/backends/cpu/int4_matmul.zig:215-305):
 * x [batch, in_f] and y [batch, out_f], row-major. scale_is_f16 selects the
 * scale element type. */
int glacier_cuda_int4_linear(const float *x, size_t batch, const uint8_t *packed,
                             const void *scales, int scale_is_f16, const float *bias, float *y,
                             size_t out_features, size_t in_features, size_t group_size,
                             void *stream);

/* Q8-activation form, the reference's default decode numerics: linearInt4WeightQ8
 * (src/backends/cpu/int4_matmul.zig:422-532) as it dispatches on a non-AArch64 host, i.e.
 * linearInt4Q8OnTheFly (:335-418).  Each x row is quantized per activation block (32 codes
 * for group 8, else group): scale = max|x| / 127, q = clamp(round(x / scale), -127, 127);
 * then acc = bias and, weight group by weight group,
 * acc += (float)(sum (u - 7) * q) * w_scale * a_scale.  Bit-identical to that portable
 * path.  Outputs longer than 65536 and inputs longer than 16384 (or with more than 2048
 * activation blocks) take the FP32-activation path, as in the reference.  Same arguments
 * as glacier_cuda_int4_linear. */
int glacier_cuda_int4_linear_q8(const float *x, size_t batch, const uint8_t *packed,
                                const void *scales, int scale_is_f16, const float *bias, float *y,
                                size_t out_features, size_t in_features, size_t group_size,
                                void *stream);

/* (b) Batched form on the tensor cores (tcgen05/TMEM dequant GEMM): x [batch, in_f] fp32,
 * y [batch, out_f]; the reference's M4 weight-stationary GEMM
 * (glacier_int4_gemm_neon_q8_prequant_f16scale_rows4_k16_m4, src/decode_lane4.zig:221-264,
 * int4_neon.c:1439-1621) generalised to batch <= 128 with FP32-activation numerics.
 * scales: fp16 bit patterns [out_f, in_f/group]; group_size 8, 16 or 32 (the reference's
 * production g8/g16 layouts and g32) and in_f a multiple of 128 for the tensor-core path
 * (other shapes run the GEMV kernels).
 * workspace: glacier_cuda_int4_matmul_workspace(batch, in_f, out_f) bytes of device memory. */
size_t glacier_cuda_int4_matmul_workspace(size_t batch, size_t in_features, size_t out_features);
int glacier_cuda_int4_matmul_f16scale(const float *x, size_t batch, const uint8_t *packed,
                                      const uint16_t *scales, const float *bias, float *y,
                                      size_t out_features, size_t in_features, size_t group_size,
                                      void *workspace, size_t workspace_bytes, void *stream);

/* ------------------------------------------------------------------------
 * (c) fused norm / rotary / activation steps, on device buffers.
 * ---------------------------------------------------------------------- */

/* rmsNormF32 (src/backends/cpu/kernels.zig:141-220): out[b] = x[b] / sqrt(mean(x[b]^2) + eps) * weight. */
int glacier_cuda_rmsnorm_f32(const float *x, const float *weight, float eps, float *out, size_t batch,
                             size_t dim, void *stream);

/* addRmsNormF32 (kernels.zig:322-401): residual = a + b; out = rmsnorm(residual). residual
 * may alias a (in-place residual update). */
int glacier_cuda_add_rmsnorm_f32(const float *a, const float *b, float *residual, const float *weight,
                                 float eps, float *out, size_t batch, size_t dim, void *stream);

/* siluMulF32 (kernels.zig:465-507) over batch rows with row strides:
 * out[b, i] = silu(gate[b, i]) * up[b, i]. */
int glacier_cuda_silu_mul_f32(const float *gate, const float *up, size_t ld_in, float *out, size_t ld_out,
                              size_t batch, size_t n, void *stream);

/* loadEmbeddingRow (src/generate.zig:3653-3663) for a batch of token ids over an fp16 table. */
int glacier_cuda_embedding_f16(const uint16_t *table, size_t vocab, size_t dim, const int32_t *tokens,
                               size_t batch, float *out, void *stream);

/* RopeTable.apply (src/generate.zig:816-831) + PagedKVCache.appendRowTxn
 * (src/paged_kv_cache.zig:1074-1103), fused: qkv[b] = [q | k | v] (+ bias); q and k are
 * rotated with the cos/sin table rows at pos[b]; q goes to q_out, k and v to the page
 * block_tables[b][pos/16], row pos%16, of `layer` (payload offset
 * ((layer*2+kind)*16+row)*kv_dim, paged_kv_cache.zig:1421-1442).  bias may be NULL. */
int glacier_cuda_qkv_rope_append_f32(const float *qkv, size_t ld, const float *bias, const float *cos_table,
                                     const float *sin_table, size_t positions, const int32_t *pos,
                                     size_t batch, size_t num_heads, size_t num_kv_heads, size_t head_dim,
                                     float *q_out, size_t ldq, float *kv_pages, size_t page_floats,
                                     const int32_t *block_tables, size_t max_pages, size_t layer,
                                     void *stream);

/* ------------------------------------------------------------------------
 * (d) paged-KV decode attention.
 * ---------------------------------------------------------------------- */

/* attentionMultiHead (src/paged_attention.zig:108-216) for one query row per lane: q [lanes,
 * num_heads*head_dim]; lane b attends over positions 0..ctx_lens[b]-1 of `layer`.
 * workspace: glacier_cuda_paged_attention_workspace() floats of device memory. */
size_t glacier_cuda_paged_attention_workspace(size_t lanes, size_t num_heads, size_t num_kv_heads,
                                              size_t head_dim, size_t max_ctx);
int glacier_cuda_paged_attention_f32(const float *q, const float *kv_pages, size_t page_floats,
                                     const int32_t *block_tables, size_t max_pages, const int32_t *ctx_lens,
                                     size_t max_ctx, size_t lanes, size_t layer, size_t num_heads,
                                     size_t num_kv_heads, size_t head_dim, float *out, float *workspace,
                                     size_t workspace_floats, void *stream);

/* ------------------------------------------------------------------------
 * (e) on-device greedy selection.
 * ---------------------------------------------------------------------- */

/* argmaxEligible (src/sampling.zig:55-107) per row of logits [batch, n]; words NULL means
 * every row is eligible (sampling.zig:194-207 greedy argmax).  words: [batch][ceil(n/64)]
 * u64 bitsets on device.  Per row: tokens[b] = winner or -1, status[b] = 0,
 * GLACIER_CUDA_EMASK or GLACIER_CUDA_ENAN; results[b] (may be NULL) gets the 24-byte
 * record of int4_neon.c:8-19.  workspace: glacier_cuda_argmax_workspace() bytes. */
size_t glacier_cuda_argmax_workspace(size_t batch, size_t n);
int glacier_cuda_argmax_eligible_f32(const float *logits, size_t batch, size_t n, const uint64_t *words,
                                     size_t word_count, int32_t *tokens, int32_t *status,
                                     glacier_argmax_result *results, void *workspace, size_t workspace_bytes,
                                     void *stream);

/* Allocation-free form of glacier_cuda_argmax_eligible_f32, for callers that cannot allocate
 * device memory when they select tokens (a runtime that budgets all GPU memory at admission, a
 * plugin given buffers but no allocator).  No counterpart in the reference.  Same arguments and
 * results minus the workspace: partial winners go to a fixed 64 KiB array of device memory inside
 * the library, so batch * ceil(n/8192) * 16 + 64 must not exceed
 * GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES (e.g. up to 215 rows of a 152064-token vocabulary);
 * larger calls return GLACIER_CUDA_EINVAL before any launch.  All calls on a device share the
 * array: calls that overlap on the GPU race and must be ordered by the caller.  The first call on
 * a device looks up the array's address with that device current; make it before any stream
 * capture starts.  That address is kept for the rest of the process: it stays valid while the
 * CUDA context that first loaded the library on the device lives, so a process that resets the
 * device (cudaDeviceReset) must not call this entry point on it again. */
#define GLACIER_CUDA_ARGMAX_NOALLOC_SCRATCH_BYTES 65536
int glacier_cuda_argmax_eligible_f32_noalloc(const float *logits, size_t batch, size_t n,
                                             const uint64_t *words, size_t word_count, int32_t *tokens,
                                             int32_t *status, glacier_argmax_result *results, void *stream);

/* ------------------------------------------------------------------------
 * Persistent model, paged KV pool and the batched decode step.  Replaces the
 * compute of generate.zig forwardLayerCached (:1511-1967) + the decode loop
 * (:5366-5450) + projectLmHead (:3665), and decode_lane4.generate's per-wave
 * compute (src/decode_lane4.zig:4155) for any lane count.  Weight upload
 * mirrors glacier_metal_int4_weight_create (src/backends/metal/backend.zig:571-595):
 * host bytes in, device-resident handle out.
 * ---------------------------------------------------------------------- */

typedef struct glacier_cuda_model_config {
  uint32_t num_layers, dim, hidden, num_heads, num_kv_heads, head_dim, vocab, group_size;
  float rms_eps, rope_theta;
  uint32_t max_positions; /* RoPE table rows (generate.zig:4964) = longest context */
  uint32_t scales_f16;    /* 1: fp16 scale mirror (int4_weights.zig:348-358), 0: keep fp32 */
} glacier_cuda_model_config;

enum glacier_cuda_tensor_kind {
  GLACIER_CUDA_W_Q = 0, GLACIER_CUDA_W_K, GLACIER_CUDA_W_V, GLACIER_CUDA_W_O,
  GLACIER_CUDA_W_GATE, GLACIER_CUDA_W_UP, GLACIER_CUDA_W_DOWN, GLACIER_CUDA_W_LM_HEAD,
  GLACIER_CUDA_B_Q, GLACIER_CUDA_B_K, GLACIER_CUDA_B_V,
  GLACIER_CUDA_N_INPUT, GLACIER_CUDA_N_POST_ATTN, GLACIER_CUDA_N_FINAL
};

typedef struct glacier_cuda_model glacier_cuda_model;
typedef struct glacier_cuda_kv glacier_cuda_kv;

/* Creates an empty model on the current device; NULL on error. */
glacier_cuda_model *glacier_cuda_model_create(const glacier_cuda_model_config *cfg);
void glacier_cuda_model_destroy(glacier_cuda_model *model);

/* One INT4 matrix in Int4WeightData form (src/int4_weights.zig:79-107): packed row-major
 * codes and one f32 scale per group.  layer -1 with GLACIER_CUDA_W_LM_HEAD. */
int glacier_cuda_model_load_int4(glacier_cuda_model *model, int layer, int kind, const uint8_t *packed,
                                 size_t packed_bytes, const float *scales, size_t scale_count);

/* Same with the codes in the prepared rows4_k16 nibble order (src/int4_weights.zig:113-170):
 * uploaded as they are and put in row-major order on the device (rows % 4 == 0, in % 16 == 0). */
int glacier_cuda_model_load_int4_rows4(glacier_cuda_model *model, int layer, int kind, const uint8_t *packed,
                                       size_t packed_bytes, const float *scales, size_t scale_count);

/* A layer's gate/up PairNibble record (src/int4_weights.zig:42-54, :322-331): pair bytes in
 * rows4_k16 order (gate codes in the low nibbles, up in the high) and the fp16 scale grid
 * [tile][group][branch][lane] (2 * hidden * dim / group values).  The pairs are split on the
 * device into the gate and up rows. */
int glacier_cuda_model_load_pair_nibble(glacier_cuda_model *model, int layer, const uint8_t *pairs,
                                        size_t pair_bytes, const uint16_t *pair_scales, size_t scale_count);

/* Same from a quantized page payload (src/model/qio.zig:73-113 encodePage layout). */
int glacier_cuda_model_load_qio(glacier_cuda_model *model, int layer, int kind, const uint8_t *payload,
                                size_t payload_bytes);

/* q/k/v biases, input / post-attention norms (layer >= 0) and the final norm (layer -1). */
int glacier_cuda_model_load_f32(glacier_cuda_model *model, int layer, int kind, const float *data,
                                size_t count);

/* Token embedding table [vocab, dim] as IEEE binary16 bit patterns. */
int glacier_cuda_model_load_embedding_f16(glacier_cuda_model *model, const uint16_t *table, size_t count);

/* Same as float32 values, for tables whose rows are not fp16-exact: an INT4
 * embedding dequantized as int4_matmul.zig dequantizeRow (:3166-3196) does,
 * or bf16 / fp32 pages.  The lookup then copies rows without rounding. */
int glacier_cuda_model_load_embedding_f32(glacier_cuda_model *model, const float *table, size_t count);

/* Checks that every tensor is present and prepares the kernels' descriptors. */
int glacier_cuda_model_finalize(glacier_cuda_model *model);

/* Reserves the step workspace for up to max_lanes lanes of max_pages pages each; a decode
 * step then allocates nothing (graph-capturable). */
int glacier_cuda_model_reserve(glacier_cuda_model *model, size_t max_lanes, size_t max_pages);

/* FP32 paged KV pool: num_pages pages of [num_layers][K|V][16][kv_dim] floats
 * (src/paged_kv_cache.zig:1421-1442), so host checkpoint / restore copies pages verbatim. */
glacier_cuda_kv *glacier_cuda_kv_create(const glacier_cuda_model *model, size_t num_pages);
void glacier_cuda_kv_destroy(glacier_cuda_kv *kv);
float *glacier_cuda_kv_pages(glacier_cuda_kv *kv);
size_t glacier_cuda_kv_page_floats(const glacier_cuda_kv *kv);

/* One greedy decode step for `lanes` independent requests (device buffers): lane b feeds
 * tokens[b] at position positions[b] (its K/V row is written there; context = positions[b]+1)
 * through block_tables[b][0..max_pages).  eligible (NULL = all tokens) holds
 * ceil(vocab/64) words per lane.  tokens_out[b] = next token or -1; status_out[b] (may be
 * NULL) = 0 / GLACIER_CUDA_EMASK / GLACIER_CUDA_ENAN; logits_out [lanes, vocab] may be NULL.
 * With 4 lanes or fewer the eligible argmax runs in the LM head's epilogue (logitless greedy,
 * int4_neon.c:1075-1254): logits are written only to a given logits_out.  A position outside
 * the RoPE table or past the block table gives that lane context 0, writes no K/V and raises
 * the bad-input device status (glacier_cuda_device_status = 2). */
int glacier_cuda_decode_step(glacier_cuda_model *model, glacier_cuda_kv *kv, size_t lanes,
                             const int32_t *tokens, const int32_t *positions, const int32_t *block_tables,
                             size_t max_pages, const uint64_t *eligible, size_t eligible_words,
                             int32_t *tokens_out, int32_t *status_out, float *logits_out, void *stream);

/* Prompt prefill of one request: the batched counterpart of the reference's prompt loop
 * (runPackedBatchPrefill, src/generate.zig:3397-3548; for g32 the reference feeds prompt tokens
 * one at a time, :2377).  tokens[0..count) (device) go in at positions start..start+count-1 of
 * block_table[0..max_pages) (device), in chunks of up to the reserved lane count; each chunk is one
 * batched pass whose rows attend causally to every earlier position, and every position's K/V rows
 * are written.  The greedy token after the last prompt position goes to token_out[0] (device),
 * its status to status_out[0] (may be NULL) and its logits to logits_out[vocab] (may be NULL).
 * Requires glacier_cuda_model_reserve. */
int glacier_cuda_prefill(glacier_cuda_model *model, glacier_cuda_kv *kv, const int32_t *tokens, size_t count,
                         int32_t start, const int32_t *block_table, size_t max_pages, const uint64_t *eligible,
                         size_t eligible_words, int32_t *token_out, int32_t *status_out, float *logits_out,
                         void *stream);

/* Tensor parallelism over G GPUs, one process per GPU (no reference counterpart: the reference
 * runs on one device).  Each rank creates its model with its local geometry: num_heads/G and
 * num_kv_heads/G heads and hidden/G FFN rows.  It loads the q/k/v, gate and up rows of its slice
 * and the matching input columns of o and down; norms, embedding and LM head are replicated.
 * After glacier_cuda_model_tp_init, decode steps and prefill all-reduce the o and down
 * projections over the ranks with NCCL on the step's stream, so every rank produces the same
 * tokens.  Rank 0 makes the id with glacier_cuda_tp_unique_id and the caller hands it to every
 * rank; tp_init blocks until all ranks have joined. */
#define GLACIER_CUDA_TP_ID_BYTES 128
int glacier_cuda_tp_unique_id(void *id_out);
int glacier_cuda_model_tp_init(glacier_cuda_model *model, int rank, int world, const void *id);
/* More ranks than kv heads (7B at 8 GPUs: 4 kv heads): the ranks of one kv-head group
 * split the lanes.  This rank attends lanes b with b % groups == index only (it still writes
 * the other lanes' K/V rows to its pages, which nothing reads); its attention output for the
 * other lanes is zero, so the all-reduce of the o projection sums every lane's heads from the
 * ranks that own it.  Call after
 * glacier_cuda_model_tp_init; groups = 1 (the default) attends every lane. */
int glacier_cuda_model_tp_lanes(glacier_cuda_model *model, int groups, int index);

/* Diagnostics, no reference counterpart: per kernel class device time of decode steps.
 * glacier_cuda_model_profile(model, 1) makes later decode steps record CUDA events on their
 * stream between the step's kernel classes (no synchronisation inside the step); 0 stops.
 * glacier_cuda_model_profile_read waits for the recorded steps, writes for each class k < kinds
 * the summed milliseconds ms[k] and the number of timed launches regions[k], and forgets the
 * records.  A region runs from one class's first launch to the next class's first launch, so it
 * includes the launch gap before the next class. */
enum glacier_cuda_step_kind {
  GLACIER_CUDA_STEP_EMBED = 0,     /* context lengths + embedding gather */
  GLACIER_CUDA_STEP_NORM,          /* residual add + RMSNorm (and split-K partial sums) */
  GLACIER_CUDA_STEP_PROJ_QKV,      /* fused Q/K/V INT4 projection */
  GLACIER_CUDA_STEP_ROPE_APPEND,   /* bias, RoPE, KV page append */
  GLACIER_CUDA_STEP_ATTENTION,     /* paged attention partials over context chunks */
  GLACIER_CUDA_STEP_ATTN_COMBINE,  /* merge of the chunk partials */
  GLACIER_CUDA_STEP_PROJ_O,
  GLACIER_CUDA_STEP_PROJ_GATE_UP,  /* fused gate/up INT4 projection */
  GLACIER_CUDA_STEP_SILU,
  GLACIER_CUDA_STEP_PROJ_DOWN,
  GLACIER_CUDA_STEP_LM_HEAD,       /* with 4 lanes or fewer: the projection and its epilogue argmax */
  GLACIER_CUDA_STEP_ARGMAX,        /* the two-pass argmax over written logits (more lanes) */
  GLACIER_CUDA_STEP_ALL_REDUCE,    /* tensor parallel: split-K sum + NCCL all-reduce of o / down */
  GLACIER_CUDA_STEP_KINDS
};
int glacier_cuda_model_profile(glacier_cuda_model *model, int enable);
int glacier_cuda_model_profile_read(glacier_cuda_model *model, double *ms, uint64_t *regions, size_t kinds);

/* Step selection, no reference counterpart.  A model reserved for one lane runs each greedy
 * decode step (glacier_cuda_decode_step) as one persistent kernel over every SM, with the
 * phases of the step separated by grid barriers, when enable = 1; enable = 0 (the default)
 * runs the multi-kernel step (the same operators, one launch per kernel class), which is the
 * faster of the two on B200.  Returns 1 when the persistent step is built for the current
 * reservation, 0 when the model or reservation is outside its contract (more than one lane;
 * not group 32 with finite fp16 scales; head dim other than 64 / 128), negative on error.
 * With profiling on, its phases are filed under the kernel classes they replace. */
int glacier_cuda_model_persistent(glacier_cuda_model *model, int enable);

/* ------------------------------------------------------------------------
 * Persistent INT4 weight handles: the Metal persistent-weight API
 * (src/backends/metal/backend.zig:571-595, shim.m:4005-4111, 5502-5624) on
 * the B200 kernels.  A context binds one device and one stream.
 * ---------------------------------------------------------------------- */

typedef struct glacier_cuda_context glacier_cuda_context;
typedef struct glacier_cuda_int4_weight glacier_cuda_int4_weight;

glacier_cuda_context *glacier_cuda_context_create(int device_ordinal); /* NULL on error */
void glacier_cuda_context_destroy(glacier_cuda_context *ctx);
void *glacier_cuda_context_stream(glacier_cuda_context *ctx); /* its cudaStream_t */

/* glacier_metal_int4_weight_create: host codes and f32 scales in, device copy
 * out; NULL for a non-power-of-two group, an empty shape, more than 2^32
 * elements, or too few packed bytes / scales. */
glacier_cuda_int4_weight *glacier_cuda_int4_weight_create(glacier_cuda_context *ctx, const uint8_t *packed,
                                                         uint64_t packed_bytes, const float *scales,
                                                         uint64_t scale_count, uint32_t group_size,
                                                         uint32_t in_features, uint32_t out_features);
/* Same with a scale type: 0 f32 scales (as above), 1 IEEE fp16 bit patterns (the
 * fp16 scale cache of int4_weights.zig:348-358); fp16 weights of groups 8/16/32
 * run batches of 5..128 rows on the tcgen05 GEMM. */
glacier_cuda_int4_weight *glacier_cuda_int4_weight_create_ex(glacier_cuda_context *ctx, const uint8_t *packed,
                                                            uint64_t packed_bytes, const void *scales,
                                                            uint64_t scale_count, uint32_t scale_dtype,
                                                            uint32_t group_size, uint32_t in_features,
                                                            uint32_t out_features);
void glacier_cuda_int4_weight_destroy(glacier_cuda_int4_weight *weight);

/* glacier_metal_int4_matvec_dispatch: host input, synchronous; the output stays in
 * the handle until glacier_cuda_int4_weight_read_output copies it
 * (glacier_metal_int4_weight_read_output).  Counts must cover the matrix. */
int glacier_cuda_int4_matvec_dispatch(glacier_cuda_context *ctx, glacier_cuda_int4_weight *weight,
                                      const float *input, uint64_t input_count, float *output,
                                      uint64_t output_count);
int glacier_cuda_int4_weight_read_output(glacier_cuda_int4_weight *weight, float *output, uint64_t output_count);

/* Device-pointer forms on a caller stream. */
int glacier_cuda_int4_weight_matvec(glacier_cuda_int4_weight *weight, const float *x, float *y, const float *bias,
                                    void *stream);
int glacier_cuda_int4_weight_matmul(glacier_cuda_int4_weight *weight, const float *x, size_t ldx, float *y,
                                    size_t ldy, size_t batch, const float *bias, void *stream);

/* LM head + argmaxEligible (sampling.zig:55-107) per row: device x [batch, in],
 * optional eligibility words [batch][word_count], tokens / status / 24-byte
 * results per row as glacier_cuda_argmax_eligible_f32 writes them.  status_out,
 * results_out and logits_out may be NULL.  Up to 4 rows on the tensor-core GEMV, the argmax
 * runs in the projection's epilogue and no logits are written unless logits_out is given. */
int glacier_cuda_int4_weight_lmhead_argmax(glacier_cuda_int4_weight *weight, const float *x, size_t batch,
                                           const uint64_t *eligible_words, size_t word_count, int32_t *tokens_out,
                                           int32_t *status_out, glacier_argmax_result *results_out,
                                           float *logits_out, void *stream);

/* glacier_all_finite_f32_neon (int4_neon.c:67-80): device *result = 1 when all
 * `count` device values are finite, else 0. */
int glacier_cuda_all_finite_f32(const float *values, size_t count, int32_t *result, void *stream);

/* ------------------------------------------------------------------------
 * The portable .glacier container (docs/FORMAT_SPEC.md; src/model/format.zig,
 * src/model/qio.zig) read from a host image of the whole file (a read or an
 * mmap).  Host-only: none of these touches a GPU except
 * glacier_cuda_model_load_glacier's uploads.
 *
 * Every entry admits the image first, as FileReader.openFile does
 * (format.zig:407-478).  A rejected image returns GLACIER_CUDA_EFORMAT, and
 * glacier_cuda_format_error() then names the reference error it stands for.
 * ---------------------------------------------------------------------- */

enum glacier_cuda_format_reason {
  GLACIER_CUDA_FMT_OK = 0,
  GLACIER_CUDA_FMT_TRUNCATED_HEADER,       /* error.TruncatedHeader */
  GLACIER_CUDA_FMT_BAD_MAGIC,              /* error.BadMagic */
  GLACIER_CUDA_FMT_BAD_VERSION,            /* error.BadVersion */
  GLACIER_CUDA_FMT_BAD_HEADER_SIZE,        /* error.BadHeaderSize */
  GLACIER_CUDA_FMT_BAD_PAGE_SIZE,          /* error.BadPageSize */
  GLACIER_CUDA_FMT_BAD_RESERVED_FIELD,     /* error.BadReservedField */
  GLACIER_CUDA_FMT_BAD_LAYOUT,             /* error.BadLayout */
  GLACIER_CUDA_FMT_METADATA_TOO_LARGE,     /* error.MetadataTooLarge */
  GLACIER_CUDA_FMT_INDEX_TOO_LARGE,        /* error.IndexTooLarge */
  GLACIER_CUDA_FMT_LAYOUT_OVERFLOW,        /* error.LayoutOverflow */
  GLACIER_CUDA_FMT_TRUNCATED_META,         /* error.TruncatedMeta */
  GLACIER_CUDA_FMT_TRUNCATED_INDEX,        /* error.TruncatedIndex */
  GLACIER_CUDA_FMT_BAD_METADATA,           /* error.BadMetadata */
  GLACIER_CUDA_FMT_BAD_TENSOR_KIND,        /* error.BadTensorKind */
  GLACIER_CUDA_FMT_BAD_PRECISION,          /* error.BadPrecision */
  GLACIER_CUDA_FMT_BAD_PAGE_ID,            /* error.BadPageId */
  GLACIER_CUDA_FMT_BAD_ROW_RANGE,          /* error.BadRowRange */
  GLACIER_CUDA_FMT_EMPTY_PAGE,             /* error.EmptyPage */
  GLACIER_CUDA_FMT_BAD_QUANT_GROUP,        /* error.BadQuantGroup */
  GLACIER_CUDA_FMT_PAGE_GEOMETRY_TOO_LARGE, /* error.PageGeometryTooLarge */
  GLACIER_CUDA_FMT_UNSUPPORTED_PRECISION,  /* error.UnsupportedPrecision (INT2, ternary) */
  GLACIER_CUDA_FMT_BAD_PAGE_GEOMETRY,      /* error.BadPageGeometry */
  GLACIER_CUDA_FMT_NON_CONTIGUOUS_PAYLOAD, /* error.NonContiguousPayload */
  GLACIER_CUDA_FMT_TRUNCATED_PAGE,         /* error.TruncatedPage */
  GLACIER_CUDA_FMT_TRAILING_BYTES,         /* error.TrailingBytes */
  GLACIER_CUDA_FMT_BAD_QUANT_PAYLOAD,      /* error.BadQuantPayload */
  GLACIER_CUDA_FMT_CRC_MISMATCH,           /* error.CrcMismatch */
  GLACIER_CUDA_FMT_SIZE_MISMATCH,          /* error.SizeMismatch (decode buffer) */
  GLACIER_CUDA_FMT_NO_LAYERS,              /* LoaderError.NoLayers */
  GLACIER_CUDA_FMT_MISSING_TENSOR,         /* LoaderError.MissingTensor */
  GLACIER_CUDA_FMT_BAD_PAYLOAD,            /* LoaderError.BadPayload */
  /* Prepared runtime image (src/model/runtime_image.zig) */
  GLACIER_CUDA_FMT_BAD_RECORD_SIZE,        /* error.BadRecordSize */
  GLACIER_CUDA_FMT_BAD_ALIGNMENT,          /* error.BadAlignment */
  GLACIER_CUDA_FMT_BAD_CONFIG,             /* error.BadConfig */
  GLACIER_CUDA_FMT_HEADER_CRC_MISMATCH,    /* error.HeaderCrcMismatch */
  GLACIER_CUDA_FMT_INDEX_CRC_MISMATCH,     /* error.IndexCrcMismatch */
  GLACIER_CUDA_FMT_LEGACY_VERSION_DISABLED, /* error.LegacyVersionDisabled */
  GLACIER_CUDA_FMT_BAD_HEADER,             /* error.BadHeader */
  GLACIER_CUDA_FMT_BAD_BOUNDS,             /* error.BadBounds */
  GLACIER_CUDA_FMT_SOURCE_FINGERPRINT_MISMATCH, /* error.SourceFingerprintMismatch */
  GLACIER_CUDA_FMT_ABI_FINGERPRINT_MISMATCH,    /* error.AbiFingerprintMismatch */
  GLACIER_CUDA_FMT_BAD_ENCODING,           /* error.BadEncoding */
  GLACIER_CUDA_FMT_BAD_PACKED_LAYOUT,      /* error.BadPackedLayout */
  GLACIER_CUDA_FMT_BAD_ROLE,               /* error.BadRole */
  GLACIER_CUDA_FMT_BAD_PAIR_NIBBLE_LAYOUT, /* error.BadPairNibbleLayout */
  GLACIER_CUDA_FMT_BAD_FLAGS,              /* error.BadFlags */
  GLACIER_CUDA_FMT_BAD_VERSIONED_RECORD,   /* error.BadVersionedRecord */
  GLACIER_CUDA_FMT_MISSING_DIGEST,         /* error.MissingDigest */
  GLACIER_CUDA_FMT_BAD_TENSOR_SHAPE,       /* error.BadTensorShape */
  GLACIER_CUDA_FMT_MISSING_SCALES,         /* error.MissingScales */
  GLACIER_CUDA_FMT_OVERLAPPING_PAYLOAD,    /* error.OverlappingPayload */
  GLACIER_CUDA_FMT_DUPLICATE_RECORD,       /* error.DuplicateRecord */
  GLACIER_CUDA_FMT_DIGEST_MISMATCH         /* error.DigestMismatch */
};

/* Reason for this thread's last GLACIER_CUDA_EFORMAT (0 after a success). */
int32_t glacier_cuda_format_error(void);

/* CRC-32 as std.hash.Crc32 (IEEE reflected polynomial), the per-page checksum. */
uint32_t glacier_cuda_crc32(const uint8_t *data, size_t len);

typedef struct glacier_cuda_file_info {
  uint64_t container_bytes, meta_offset, meta_len, num_pages, page_index_offset, page_data_offset;
} glacier_cuda_file_info;

/* One 64-byte page index entry, decoded (PageEntry, format.zig:141-202). */
typedef struct glacier_cuda_page_entry {
  uint64_t page_id;
  uint32_t layer_idx, tensor_kind; /* TensorKind 0..15 or 255 */
  uint64_t row_start, row_end;     /* flat element range of the tensor */
  uint8_t precision;               /* 0 fp16, 1 bf16, 2 int8, 3 int4, 6 fp32 */
  uint8_t quant_group;             /* 0 for raw pages */
  uint16_t reserved;
  uint32_t crc32;
  uint64_t data_offset, data_len;
} glacier_cuda_page_entry;

/* Model geometry as loader.zig derives it from page metadata (:1224-1260):
 * dim from the norms, hidden and vocab from the flat sizes of the MLP and
 * vocabulary tensors, layers from the largest layer_idx. */
typedef struct glacier_cuda_file_geometry {
  uint32_t num_layers, dim, hidden, vocab, group_size;
  uint32_t has_lm_head, has_qkv_bias;
} glacier_cuda_file_geometry;

/* Header, layout, metadata JSON and page index admission
 * (FileReader.openFile, format.zig:407-478). */
int glacier_cuda_glacier_open(const uint8_t *bytes, uint64_t len, glacier_cuda_file_info *info);

/* Admission plus every page's quantized sub-header and CRC-32
 * (FileReader.validateAllPageCrcs, format.zig:497-534), pages checked in
 * parallel on the host; the first failing page in page order is reported. */
int glacier_cuda_glacier_validate_pages(const uint8_t *bytes, uint64_t len);

int glacier_cuda_glacier_page(const uint8_t *bytes, uint64_t len, uint64_t index, glacier_cuda_page_entry *out);

/* Every page entry in one admission: writes min(capacity, pages) entries and
 * sets *count to the page count (capacity 0 queries the count). */
int glacier_cuda_glacier_pages(const uint8_t *bytes, uint64_t len, glacier_cuda_page_entry *out, uint64_t capacity,
                               uint64_t *count);

/* One page's elements as f32 (FileReader.readPageDequant(f32), format.zig:638-662):
 * CRC first, then the quantized sub-header, then the decode.  count must equal
 * the page's element count. */
int glacier_cuda_glacier_page_decode_f32(const uint8_t *bytes, uint64_t len, uint64_t index, float *out,
                                         uint64_t count);

int glacier_cuda_glacier_geometry(const uint8_t *bytes, uint64_t len, glacier_cuda_file_geometry *out);

/* Loads every tensor of a .glacier image into a model created with the
 * matching config (loader.zig loadWithOptions, :1214-1540, compact INT4):
 * INT4 projection, LM head and embedding pages are concatenated in packed
 * form (concatInt4Pages, :1633-1730), norms and biases decoded to f32, and a
 * tied LM head reuses the INT4 embedding (:1521-1523).  Every page's CRC is
 * checked before the first upload.  The caller then runs
 * glacier_cuda_model_finalize.  Dense (non-INT4) projections and an attention
 * output bias return GLACIER_CUDA_EUNSUPPORTED. */
int glacier_cuda_model_load_glacier(glacier_cuda_model *model, const uint8_t *bytes, uint64_t len,
                                    int tie_word_embeddings);

/* ------------------------------------------------------------------------
 * The prepared runtime image `.glrt` (docs/RUNTIME_IMAGE.md;
 * src/model/runtime_image.zig), v1 read-only and v2, from a host image of the
 * whole file.  Admission follows MappedImage.openOwnedFileWithOptionsV1
 * (runtime_image.zig:828-850): header CRC, config, ABI fingerprint, index CRC,
 * every record's descriptor, bounds, identity and overlap, then each record's
 * payload CRC and v2 SHA-256 digest (checked on all host cores; the failure
 * reported is the one the reference's sequential walk meets first).
 * ---------------------------------------------------------------------- */

typedef struct glacier_cuda_glrt_options {
  uint32_t skip_payload_crc;    /* 0 (default): verify every record's payload CRC */
  uint32_t skip_payload_digest; /* 0 (default): verify every v2 record's SHA-256 digest */
  uint32_t reject_v1;           /* 0 (default): v1 images are read */
  uint32_t abi_policy;          /* 0: either preparation policy; 1: portable only; 2: AArch64 only */
  const uint8_t *expected_source_fingerprint; /* 32 bytes, or NULL */
} glacier_cuda_glrt_options;

typedef struct glacier_cuda_glrt_info {
  uint32_t version, abi_policy; /* abi_policy 1 portable, 2 AArch64 */
  uint64_t record_count, data_offset, file_size;
  uint8_t source_fingerprint[32], abi_fingerprint[32];
  uint32_t dim, hidden, num_layers, vocab, num_heads, head_dim, num_kv_heads, tie_embeddings;
  float rms_eps, rope_theta;
  /* Filled by glacier_cuda_glrt_model_info only: */
  uint32_t mlp_layout; /* 1 separate gate/up records, 2 one PairNibble record per layer */
  uint32_t group_size; /* the INT4 group every quantized record shares */
} glacier_cuda_glrt_info;

/* One decoded record (runtime_image.zig Record, :308-430).  Streams in the
 * order packed_weights, scales_f32, scales_f16, scales_f16_rows4, raw. */
typedef struct glacier_cuda_glrt_entry {
  uint32_t layer_idx, tensor_kind; /* layer 0xffffffff: global tensor */
  uint16_t encoding;               /* 0 raw f32, 1 INT4, 2 PairNibble */
  uint16_t packed_layout;          /* 0 row-major, 1 rows4_k16, 0xffff none */
  uint16_t role;                   /* 0 tensor, 1 MLP gate/up pair */
  uint16_t pair_nibble_layout;     /* 0 rows4_k16, 0xffff none */
  uint32_t group_size, out_f, in_f, payload_crc32;
  uint64_t num_elements;
  uint64_t stream_offset[5], stream_len[5];
  uint8_t payload_digest[32];
} glacier_cuda_glrt_entry;

/* opts may be NULL (defaults).  info may be NULL. */
int glacier_cuda_glrt_open(const uint8_t *bytes, uint64_t len, const glacier_cuda_glrt_options *opts,
                           glacier_cuda_glrt_info *info);

/* One record of a structurally admitted image (payload content not re-verified). */
int glacier_cuda_glrt_record(const uint8_t *bytes, uint64_t len, uint64_t index, glacier_cuda_glrt_entry *out);

/* Every record in one structural admission: writes min(capacity, records)
 * entries and sets *count to the record count (capacity 0 queries the count). */
int glacier_cuda_glrt_records(const uint8_t *bytes, uint64_t len, glacier_cuda_glrt_entry *out, uint64_t capacity,
                              uint64_t *count);

/* Admission plus the prepared-model schema (loader.zig validatePreparedConfig
 * :618-652, validatePreparedRecordSet :656-714): the config to create the model
 * with, its MLP form and its INT4 group. */
int glacier_cuda_glrt_model_info(const uint8_t *bytes, uint64_t len, const glacier_cuda_glrt_options *opts,
                                 glacier_cuda_glrt_info *info);

/* Loads a prepared image into a model created with its config
 * (loader.zig loadPreparedOwnedFileWithOptionsV1, :216-385).  rows4_k16 codes,
 * rows4 fp16 scale grids and PairNibble records are put back in row-major
 * order on the host, bit for bit; the embedding becomes an f32 table
 * dequantized as dequantizeRow does, and a tied head reuses its INT4 data.
 * The caller then runs glacier_cuda_model_finalize.  An attention output bias
 * or mixed INT4 group sizes return GLACIER_CUDA_EUNSUPPORTED. */
int glacier_cuda_model_load_glrt(glacier_cuda_model *model, const uint8_t *bytes, uint64_t len,
                                 const glacier_cuda_glrt_options *opts);

/* Layout transforms (int4_weights.zig): rows4_k16 nibble order -> row-major
 * (packedNibbleIndex, :153-170); the [tile][group][lane] fp16 scale grid ->
 * row-major f32 (withRows4F16Scales, :362-386); a PairNibble record -> its gate
 * and up branches, row-major, with f32 scales (pairRows4K16, :251-346). */
int glacier_cuda_rows4_k16_to_row_major(const uint8_t *src, uint8_t *dst, size_t out_f, size_t in_f);
int glacier_cuda_rows4_scales_to_row_major(const uint16_t *src, float *dst, size_t out_f, size_t groups_per_row);
int glacier_cuda_pair_nibble_split(const uint8_t *pairs, const uint16_t *pair_scales, size_t out_f, size_t in_f,
                                   size_t group, uint8_t *gate, uint8_t *up, float *gate_scales, float *up_scales);

#ifdef __cplusplus
}
#endif

#endif /* GLACIER_CUDA_H */
