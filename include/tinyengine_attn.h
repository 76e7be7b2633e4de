/*
 * TinyEngine attention engine for NVIDIA B200 (sm_100a): device-resident
 * f16 paged KV cache, fused RoPE + append, split-K GQA flash decode and
 * causal flash prefill on tcgen05 tensor cores.
 *
 * These entry points replace the attention slice of TinyEngine's internal
 * Metal boundary (c/src/metal_backend.h:206-343: te_metal_decode_layer_f32,
 * te_metal_decode_all_layers_f32, te_metal_prefill_layer_f32,
 * te_metal_prefill_all_layers_f32) and of the resident-KV manager
 * (c/src/metal/metal_backend_layers.mm.inc:1116-1173, 2029-2181).  The
 * reference passes host fp32 caches into each call and copies them in and
 * out; here the cache lives in HBM for its whole life and only queries,
 * new K/V rows and outputs cross the boundary.
 *
 * Conventions
 * - All functions return te_status (tinyengine.h); te_attn_engine_last_error
 *   gives the detailed message of the engine's last failure.
 * - Pointers named q, k, v, out are DEVICE pointers (cudaMalloc, torch
 *   tensors' data_ptr(), ...) unless TE_ATTN_HOST_BUFFERS is set, in which
 *   case they are host pointers (pinned memory recommended) and the call
 *   copies them in and out and returns only when `out` is filled.
 * - Host arrays (seq_ids, q_positions) are read during the call only.
 * - Work is queued on the engine's stream; device-pointer calls return
 *   without synchronising.
 * - An engine and its caches are used from one host thread at a time;
 *   distinct engines are independent (no global lock).
 * - Nothing falls back to the CPU: without a CUDA device, engine creation
 *   returns TE_STATUS_UNSUPPORTED.
 *
 * Layouts (fp32 unless stated)
 *   decode  q, out:   [n_layers][n_seqs][heads][head_dim]
 *           k/v_new:  [n_layers][n_seqs][kv_heads][head_dim]   (pre-RoPE)
 *           partial:  [n_layers][n_seqs][heads][head_dim + 2]
 *                     = { acc[head_dim], m, l }: m = max of q.k*log2(e)/sqrt(head_dim),
 *                     l = sum 2^(s - m), acc = sum 2^(s - m) * v.
 *   prefill q, out:   [n_layers][n_tokens][heads][head_dim]
 *           k, v:     [n_layers][n_tokens][kv_heads][head_dim] (pre-RoPE)
 *   cache rows read/written by te_kv_cache_read_f16 / te_kv_cache_write_f16:
 *                     [n_tokens][kv_heads][head_dim] IEEE binary16 bits.
 */
#ifndef TINYENGINE_ATTN_H
#define TINYENGINE_ATTN_H

#include "tinyengine.h"

#ifdef __cplusplus
extern "C" {
#endif

#define TE_ATTN_ABI_VERSION 1u

/* Flags for the compute entry points. */
#define TE_ATTN_ADVANCE       (1u << 0) /* after the call, each sequence's length += tokens appended */
#define TE_ATTN_PARTIAL       (1u << 1) /* decode writes partial records instead of normalised output */
#define TE_ATTN_NO_ROPE       (1u << 2) /* q (and k) are used as given, without rotation */
#define TE_ATTN_INPUT_F16     (1u << 3) /* q/k/v inputs are binary16 instead of fp32 */
#define TE_ATTN_HOST_BUFFERS  (1u << 4) /* q/k/v/out are host pointers; call is synchronous */
#define TE_ATTN_QKV_BIAS      (1u << 5) /* add the cache's per-layer q/k/v biases (te_kv_cache_set_qkv_bias)
                                           to the raw inputs first, in fp32, before RoPE and rounding */
#define TE_ATTN_ACCUMULATE    (1u << 6) /* te_matvec_gguf: y += W x (the residual add of a projection) */
#define TE_ATTN_RMSNORM_INPUT (1u << 7) /* te_matvec_gguf_fused: the input is RMSNorm(x) * norm_weight */
#define TE_ATTN_SWIGLU_INPUT  (1u << 8) /* te_matvec_gguf_fused: the input is SwiGLU of x = [gate | up] */
#define TE_ATTN_EXACT_Q       (1u << 9) /* te_attention_prefill with binary16 inputs: the rotated (or biased)
                                           fp32 query enters the tensor cores as f16 hi + lo parts, as fp32
                                           inputs always do (about half the speed of the single rounding) */

typedef struct te_attn_engine te_attn_engine;
typedef struct te_kv_cache te_kv_cache;

typedef struct te_attn_options {
    uint32_t abi_version;      /* TE_ATTN_ABI_VERSION */
    int32_t device;            /* CUDA device ordinal */
    void *stream;              /* cudaStream_t to launch on; NULL = engine-owned non-blocking stream */
    uint32_t decode_chunk_tokens; /* split-K chunk length (multiple of 64); 0 = chosen per call */
    uint32_t flags;            /* reserved, 0 */
} te_attn_options;

typedef struct te_kv_cache_desc {
    uint32_t abi_version;      /* TE_ATTN_ABI_VERSION */
    uint32_t layers;
    uint32_t max_seqs;         /* sequence slots 0 .. max_seqs-1 */
    uint32_t max_tokens_per_seq;
    uint32_t kv_heads;
    uint32_t head_dim;         /* 64 or 128 */
    uint32_t page_tokens;      /* tokens per page, multiple of 64; 0 = 128 */
    uint32_t total_pages;      /* pages per layer in the pool; 0 = max_seqs * pages per full sequence */
    uint32_t max_position;     /* RoPE table length (global positions); 0 = max_tokens_per_seq */
    float rope_theta;          /* RoPE base, > 0 (Qwen2: 1e6) */
} te_kv_cache_desc;

/* Engine ------------------------------------------------------------------ */

TE_API te_attn_options te_attn_default_options(void);
TE_API te_status te_attn_engine_create(const te_attn_options *options, te_attn_engine **out_engine);
/* Frees the engine's stream (when it owns it) and scratch.  Free every cache
 * created from the engine (te_kv_cache_free) before the engine itself. */
TE_API void te_attn_engine_free(te_attn_engine *engine);
TE_API te_status te_attn_engine_set_stream(te_attn_engine *engine, void *stream);
TE_API void *te_attn_engine_stream(const te_attn_engine *engine);
/* Waits for queued work; reports (and clears) a device-side error such as an
 * expired bounded wait as TE_STATUS_RUNTIME_ERROR. */
TE_API te_status te_attn_engine_synchronize(te_attn_engine *engine);
TE_API const char *te_attn_engine_last_error(const te_attn_engine *engine);
/* Number of this library's kernels launched by the engine so far. */
TE_API uint64_t te_attn_engine_launch_count(const te_attn_engine *engine);
/* Measurement: while enabled, te_attention_prefill records a pair of CUDA
 * events around its tensor-core attention kernel on the engine's stream;
 * te_attn_engine_last_kernel_ms waits for the last recorded pair and returns
 * that kernel's duration in milliseconds (TE_STATUS_INVALID_ARGUMENT when
 * nothing was recorded). */
TE_API te_status te_attn_engine_time_kernels(te_attn_engine *engine, int enable);
TE_API te_status te_attn_engine_last_kernel_ms(te_attn_engine *engine, float *ms);
/* Bound (1 ms .. 60 s; default 2 s) of the waits in which this engine's
 * kernels wait for other GPUs (te_attn_exchange_merge's wait for the peers'
 * pushes).  A wait that runs out sets the engine's error word, which the next
 * te_attn_engine_synchronize reports as TE_STATUS_RUNTIME_ERROR; the device
 * context stays usable.  The reference's counterpart is the status check of
 * each Metal command buffer (c/src/metal/metal_backend_layers.mm.inc:2318,
 * 2581): a failed GPU step becomes TE_STATUS_RUNTIME_ERROR. */
TE_API te_status te_attn_engine_set_wait_limit(te_attn_engine *engine, uint32_t milliseconds);
/* Per-kernel device-time profile: while enabled, every launch of this
 * library's kernels on the engine's stream is bracketed by a CUDA event pair
 * (launches captured into a CUDA graph are not timed).  Also enabled at
 * engine creation by the environment variable TINYENGINE_PROFILE (any value
 * but "0"), the reference's switch (c/src/qwen.c:47-73, 2216-2304); then the
 * engine prints its totals to stderr when freed.  The report is one line,
 * "tinyengine_profile: device_ms=T decode=ms/calls append=... merge=...
 * prefill_prep=... prefill_attn=... matvec=... exchange=... step=...", the reference's
 * "name=ms/calls" format.  te_attn_engine_profile_report synchronises the
 * engine's stream and writes that line to buf (TE_STATUS_INVALID_ARGUMENT if
 * it does not fit). */
TE_API te_status te_attn_engine_profile(te_attn_engine *engine, int enable);
TE_API te_status te_attn_engine_profile_report(te_attn_engine *engine, char *buf, size_t len);

/* KV cache ---------------------------------------------------------------- */

TE_API te_kv_cache_desc te_kv_cache_default_desc(void);
TE_API te_status te_kv_cache_create(te_attn_engine *engine, const te_kv_cache_desc *desc,
                                    te_kv_cache **out_cache);
TE_API void te_kv_cache_free(te_kv_cache *cache);
/* Empties sequence `seq` (its pages return to the pool) and sets the global
 * RoPE position of its first token (0 for a whole sequence; the start of the
 * shard for a KV-split shard). */
TE_API te_status te_kv_cache_seq_reset(te_kv_cache *cache, size_t seq, size_t position_offset);
/* Drops the tokens at index >= length (length <= current length); the pages
 * stay mapped and are overwritten by later appends.  No reference counterpart
 * (the reference's generation state only grows, c/src/qwen.c:376-392). */
TE_API te_status te_kv_cache_seq_truncate(te_kv_cache *cache, size_t seq, size_t length);
TE_API te_status te_kv_cache_seq_length(const te_kv_cache *cache, size_t seq, size_t *out_length);
/* Maps pages so that sequence `seq` can grow to `tokens` tokens without any
 * page-table upload later: a decode/append that stays within reserved pages
 * issues only kernel launches and can be captured into a CUDA graph.  No
 * reference counterpart (the reference allocates the whole context up front,
 * c/src/qwen.c:458-486). */
TE_API te_status te_kv_cache_reserve(te_kv_cache *cache, size_t seq, size_t tokens);
/* Raw f16 rows (already rotated) into / out of tokens [token_begin, +n_tokens)
 * of one layer; `k`/`v` may be host or device pointers.  A write grows the
 * sequence's length to token_begin + n_tokens when that is larger. */
TE_API te_status te_kv_cache_write_f16(te_kv_cache *cache, size_t layer, size_t seq,
                                       size_t token_begin, size_t n_tokens,
                                       const uint16_t *k, const uint16_t *v);
TE_API te_status te_kv_cache_read_f16(te_kv_cache *cache, size_t layer, size_t seq,
                                      size_t token_begin, size_t n_tokens,
                                      uint16_t *k, uint16_t *v);
/* Stores the fp32 projection biases of layers [layer_begin, +n_layers):
 * q_bias [n_layers][heads * head_dim], k_bias and v_bias
 * [n_layers][kv_heads * head_dim] (host or device pointers; NULL = zeros).
 * Calls with TE_ATTN_QKV_BIAS add them to the raw q/k/v inputs, element by
 * element in fp32, before RoPE and before the binary16 rounding of the
 * cache: the reference's te_add_f32 of q/k/v and their biases
 * (c/src/qwen.c:998-1011 decode, :771-783 prefill; c/src/ops.c:408-416),
 * fused into the RoPE + append pass as the Metal
 * te_qkv_bias_rope_cache_batch_h_f32 fuses it
 * (c/src/metal/metal_kernels.metal.inc:2344-2429).  `heads` is fixed by the
 * first call (later calls and the compute calls must use the same value). */
TE_API te_status te_kv_cache_set_qkv_bias(te_kv_cache *cache, size_t layer_begin, size_t n_layers,
                                          size_t heads, const float *q_bias, const float *k_bias,
                                          const float *v_bias);

/* Compute ----------------------------------------------------------------- */

/*
 * Fused RoPE(k) + binary16 round-to-nearest-even append of n_tokens new rows
 * per layer for layers [layer_begin, +n_layers) of sequence `seq`, at local
 * token indices length .. length+n_tokens-1 (global RoPE positions offset +
 * index).  Replaces the k/v half of te_qkv_bias_rope_cache_batch_h_f32
 * (c/src/metal/metal_kernels.metal.inc:2344-2429) and the CPU append
 * (c/src/qwen.c:805-807).  Flags: TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16,
 * TE_ATTN_NO_ROPE, TE_ATTN_QKV_BIAS (k and v biases).
 */
TE_API te_status te_kv_append_rope(te_kv_cache *cache, size_t layer_begin, size_t n_layers,
                                   size_t seq, const void *k, const void *v, size_t n_tokens,
                                   uint32_t flags);

/*
 * One decode step for n_seqs sequences over layers [layer_begin, +n_layers).
 * When k_new/v_new are non-NULL, each sequence first appends one token per
 * layer (RoPE + f16 append at index `length`), then every query attends over
 * all cached tokens including the new one; q is rotated at the sequence's
 * last global position, or at q_positions[i] when q_positions is non-NULL
 * (KV-split shards that do not own the newest token).  Output is normalised
 * attention, or partial records with TE_ATTN_PARTIAL.  Flags:
 * TE_ATTN_ADVANCE, TE_ATTN_PARTIAL, TE_ATTN_NO_ROPE, TE_ATTN_HOST_BUFFERS,
 * TE_ATTN_QKV_BIAS (q, k_new and v_new get the layer's biases).  Replaces
 * te_attention_decode_f32 as called from c/src/qwen.c:1038-1046 and the
 * attention kernels of te_metal_decode_all_layers_f32
 * (c/src/metal/metal_backend_layers.mm.inc:1273-1296).
 */
TE_API te_status te_attention_decode(te_kv_cache *cache, size_t layer_begin, size_t n_layers,
                                     const uint32_t *seq_ids, size_t n_seqs,
                                     const int64_t *q_positions,
                                     const float *q, const float *k_new, const float *v_new,
                                     size_t heads, float *out, uint32_t flags);

/*
 * Log-sum-exp merge of partial records from n_parts shards:
 * partials[n_parts][rows][head_dim + 2] -> out[rows][head_dim].  No reference
 * counterpart (the reference runs on one device); the rescale is that of
 * c/src/metal/metal_kernels.metal.inc:2650-2681.
 */
TE_API te_status te_attention_merge_partials(te_attn_engine *engine, const float *partials,
                                             size_t n_parts, size_t rows, size_t head_dim,
                                             float *out, uint32_t flags);

/* Quantized matrix-vector products ------------------------------------------
 *
 * y[v][r] = sum_c W[r][c] * x[v][c] for v < n_vectors (1..8), where W is a
 * row-major GGUF matrix [rows][cols] of 32-weight blocks -- Q4_0: f16 scale
 * + 16 bytes of 4-bit quants (weight j in the low nibble of byte j, weight
 * j+16 in its high nibble, both offset by 8); Q8_0: f16 scale + 32 int8 --
 * x [n_vectors][cols] and y [n_vectors][rows] fp32.  Device pointers, w and x
 * 16-byte aligned, cols a multiple of 32; asynchronous on the engine's
 * stream.  Replaces the quantized row loop of te_model_matvec_f32
 * (c/src/ops.c:216-262, dot products :584-620) and te_metal_matvec_f32; the
 * products are the reference's, the sums run in another order (results agree
 * to fp32 rounding).  quant: TE_ATTN_QUANT_GGUF_Q4_0 or _Q8_0 (the values of
 * the reference's te_quant_kind, c/include/tinyengine.h:51,55).  With
 * TE_ATTN_ACCUMULATE each finished dot product is added to y in fp32 (y is
 * read first): the output projection and its residual add in one pass, as
 * c/src/qwen.c:1072-1079 does with te_qwen_matvec_exact then te_add_f32 (and
 * the MLP down projection at :1105-1108).
 * TE_STATUS_UNSUPPORTED for rows too long to stage (more than about 205k
 * Q4_0 or 108k Q8_0 columns).  A staging wait that runs out (2 s) sets the
 * engine's error word. */
#define TE_ATTN_QUANT_GGUF_Q4_0 4u
#define TE_ATTN_QUANT_GGUF_Q8_0 8u
TE_API te_status te_matvec_gguf(te_attn_engine *engine, uint32_t quant, const void *w, size_t rows,
                                size_t cols, const float *x, size_t n_vectors, float *y, uint32_t flags);

/* The same product (n_vectors 1..8) with the elementwise step that the
 * reference runs just before it fused into the input reads, per vector:
 *   TE_ATTN_RMSNORM_INPUT: the input is te_rmsnorm_f32(x, norm_weight, eps)
 *     (c/src/ops.c:272-293: squares summed in double, scale =
 *     1 / sqrtf((float)(sum / cols) + eps), (x[c] * scale) * norm_weight[c]),
 *     which precedes the q/k/v, gate/up and lm_head projections
 *     (c/src/qwen.c:965-971, :1082-1088, :1350-1356);
 *   TE_ATTN_SWIGLU_INPUT: x holds [gate | up] per vector (x [n_vectors][2 * cols]) and the input
 *     is te_swiglu_f32(gate, up) (ops.c:397-406: gate / (1 + expf(-gate)) *
 *     up), which precedes the down projection (qwen.c:1933-1941).
 * Exactly one of the two, optionally with TE_ATTN_ACCUMULATE.  norm_weight
 * [cols] fp32 (RMSNorm only, 16-byte aligned), eps > 0; other arguments and
 * limits as te_matvec_gguf.  The norm's sum runs in another order than the
 * reference's (in double), and expf is the device's, so results agree to
 * fp32 rounding. */
TE_API te_status te_matvec_gguf_fused(te_attn_engine *engine, uint32_t quant, const void *w, size_t rows,
                                      size_t cols, const float *x, size_t n_vectors, const float *norm_weight,
                                      float eps, float *y, uint32_t flags);

/* KV-split exchange over NVLink --------------------------------------------
 *
 * For one sequence whose cached tokens are split over `world` GPUs (one
 * process per GPU, each rank on its own device with its own engine), one
 * kernel per decode step replaces the all-gather of the partial records and
 * te_attention_merge_partials: every rank pushes its records
 * [rows][head_dim + 2] (from te_attention_decode with TE_ATTN_PARTIAL) into
 * the other ranks' exchange areas over NVLink (CUDA IPC mappings), then
 * merges [rows][head_dim] from what has arrived.  No reference counterpart
 * (the reference runs on one device); the merge is
 * te_attention_merge_partials'.
 *
 * Setup: te_attn_exchange_create on every rank (same world, rows, head_dim),
 * exchange the TE_ATTN_IPC_HANDLE_BYTES-byte handles among the ranks (any
 * host channel), te_attn_exchange_connect with all of them in rank order.
 * Every rank then calls te_attn_exchange_merge once per step, in the same
 * order; the call is asynchronous on the engine's stream and can be captured
 * in a CUDA graph.  A rank waits at most 2 s for its peers (then the engine
 * reports TE_STATUS_RUNTIME_ERROR at its next synchronisation).  Free only
 * after every rank has finished its last step (a host barrier), since the
 * peers write into this rank's area.  world <= 8.
 */
typedef struct te_attn_exchange te_attn_exchange;
#define TE_ATTN_IPC_HANDLE_BYTES 64

TE_API te_status te_attn_exchange_create(te_attn_engine *engine, size_t world, size_t rank, size_t rows,
                                         size_t head_dim, te_attn_exchange **out_exchange,
                                         unsigned char *ipc_handle);
TE_API te_status te_attn_exchange_connect(te_attn_exchange *exchange, const unsigned char *ipc_handles);
TE_API te_status te_attn_exchange_merge(te_attn_exchange *exchange, const float *partial, float *out);
TE_API void te_attn_exchange_free(te_attn_exchange *exchange);

/* Fused KV-split decode: one launch per step and rank, no collective.  This
 * rank decodes its token range of sequence `seq` of `cache` (layers
 * [layer_begin, +n_layers), heads query heads; the exchange's rows must be
 * n_layers * heads and its head_dim the cache's) like te_attention_decode
 * with TE_ATTN_PARTIAL, but as each (layer, kv head) group's record is
 * finished the kernel stores it into every rank's exchange area over NVLink
 * and counts it there (one system-scope release; nothing waits).  At its end
 * the kernel merges every group for this rank's own output from its local
 * area by log-sum-exp (te_attention_merge_partials' rescale), each CTA
 * waiting (bounded: the engine's wait limit) only for the records of the
 * groups it merges.  Output: te_attn_exchange_output, [n_layers][heads]
 * [head_dim] fp32 in this rank's HBM.  On an expired wait
 * te_attn_engine_synchronize reports TE_STATUS_RUNTIME_ERROR and the
 * exchange must be recreated.  q_position < 0: the query's position is the
 * sequence's last (the rank that owns the tail appends k_new/v_new, one token
 * per layer); otherwise the global position given (ranks without the tail
 * pass NULL k_new/v_new).  Every rank calls this once per step, in the same
 * order; a step's output is valid in stream order after the call and until
 * the next step's call on this rank.  Flags: TE_ATTN_ADVANCE,
 * TE_ATTN_NO_ROPE, TE_ATTN_QKV_BIAS.  Asynchronous on the engine's stream;
 * capturable in a CUDA graph.  No reference counterpart (the reference runs
 * on one device). */
TE_API te_status te_attention_decode_kv_split(te_attn_exchange *exchange, te_kv_cache *cache,
                                              size_t layer_begin, size_t n_layers, size_t seq,
                                              int64_t q_position, const float *q, const float *k_new,
                                              const float *v_new, size_t heads, uint32_t flags);
/* Device pointer of this rank's merged output region of the fused decode. */
TE_API te_status te_attn_exchange_output(te_attn_exchange *exchange, float **out);

/*
 * Causal prefill of n_tokens new tokens of sequence `seq` over layers
 * [layer_begin, +n_layers): RoPE + f16 append of k/v, RoPE of q, then every
 * new token t attends to cached tokens 0 .. length+t (length = tokens cached
 * before the call).  Replaces the CPU prefill loop (c/src/qwen.c:774-824) and
 * te_metal_prefill_all_layers_f32's attention
 * (c/src/metal/metal_backend_layers.mm.inc:2406-2456) and, for head_dim 64,
 * the Metal MMA prefill te_attention_flash_mma_t_f32_kernel
 * (c/src/metal/metal_kernels.metal.inc:2693-2836).  head_dim 64 or 128.
 * The tensor cores multiply f16: fp32 query inputs are fed as two f16 parts
 * (hi = f16(q), lo = f16(q - hi)) into the same accumulator, keeping the
 * fp32 query's precision; binary16 inputs whose query is rotated or biased
 * round it once to f16 unless TE_ATTN_EXACT_Q is given.  Flags:
 * TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, TE_ATTN_HOST_BUFFERS, TE_ATTN_NO_ROPE,
 * TE_ATTN_QKV_BIAS, TE_ATTN_EXACT_Q.
 */
TE_API te_status te_attention_prefill(te_kv_cache *cache, size_t layer_begin, size_t n_layers,
                                      size_t seq, const void *q, const void *k, const void *v,
                                      size_t n_tokens, size_t heads, float *out, uint32_t flags);

/* Whole-token qwen2 decode step in one launch ------------------------------
 *
 * te_qwen_forward_token (c/src/qwen.c:907-1112) for every layer of one token
 * -- RMSNorm, the q/k/v projections and their biases, RoPE, the f16 KV append,
 * GQA attention, the output projection and its residual add, RMSNorm, the
 * gate/up projections, SwiGLU, the down projection and its residual add --
 * and optionally te_qwen_project_next (:1303-1377: output RMSNorm, lm_head,
 * first-maximum argmax), as ONE cooperative kernel launch with one CTA per
 * SM, where the per-op path (te_matvec_gguf_fused + te_attention_decode +
 * te_matvec_gguf) takes five launches per layer.  The replaced reference
 * boundary is the same pair of functions; the Metal path's counterpart is
 * te_metal_decode_all_layers_f32 (c/src/metal_backend.h:206-343), which
 * batches a token's layers into one command buffer.
 *
 * te_qwen_step_create packs, once, each CTA's row slice of every projection
 * (q|k|v rows stacked, output, gate|up rows stacked, down, lm_head) into one
 * contiguous device stream, a second copy of the weights (about the size of
 * the projections); the caller's weight buffers are only read during the
 * call.  All pointers in the descriptor are device pointers except the four
 * arrays of per-layer matrix pointers, which are host arrays of `layers`
 * device pointers (read during the call only).  Matrices are row-major GGUF
 * Q4_0 / Q8_0 (TE_ATTN_QUANT_GGUF_*), 2-byte aligned:
 *   w_qkv[l]  [(heads + 2 * kv_heads) * head_dim][hidden]  q rows, k rows, v rows
 *   w_o[l]    [hidden][hidden]        w_gu[l] [2 * ffn][hidden]  gate rows, up rows
 *   w_down[l] [hidden][ffn]           w_head  [vocab][hidden]
 * attn_norm / ffn_norm [layers][hidden], out_norm [hidden] and the
 * dequantised embedding table [vocab][hidden] are fp32, 16-byte aligned.
 * kv_heads and head_dim are the cache's (head_dim 64 or 128, heads * head_dim
 * == hidden, heads / kv_heads <= 16, hidden and ffn multiples of 32); the
 * cache's layers must equal `layers` (at most 127), and hidden may not exceed
 * 64 rows per SM of the device (TE_STATUS_UNSUPPORTED otherwise); the q/k/v biases are the cache's
 * (te_kv_cache_set_qkv_bias with `heads`, applied with TE_ATTN_QKV_BIAS).
 *
 * te_qwen_step_run appends one token to sequence `seq` at index length (RoPE
 * position offset + length) and runs every layer: *token (device int64) is
 * the token, `hidden` (device fp32 [hidden], 16-byte aligned) receives the
 * hidden state after the last layer (its previous contents are not read).
 * With TE_ATTN_STEP_HEAD it also writes logits [vocab] and the greedy next
 * token to *next_token (device int64).  Flags: TE_ATTN_ADVANCE,
 * TE_ATTN_QKV_BIAS, TE_ATTN_STEP_HEAD.  Asynchronous on the engine's stream;
 * within reserved pages (te_kv_cache_reserve) it issues only the kernel launch
 * and can be captured in a CUDA graph.  Results agree with the per-op path
 * to fp32 rounding (the same exact weight decoding, other summation orders).
 * A token outside the vocabulary, or a device-side wait that runs out (2 s),
 * sets the engine's error word (te_attn_engine_synchronize reports
 * TE_STATUS_RUNTIME_ERROR).  Free every step before its cache.
 */
#define TE_ATTN_STEP_HEAD     (1u << 10) /* te_qwen_step_run: output RMSNorm + lm_head + argmax too */

typedef struct te_qwen_step te_qwen_step;
typedef struct te_qwen_step_desc {
    uint32_t abi_version;      /* TE_ATTN_ABI_VERSION */
    uint32_t layers, hidden, heads, ffn, vocab;
    float eps;                 /* RMSNorm epsilon, > 0 */
    uint32_t quant_qkv, quant_o, quant_gu, quant_down, quant_head;
    const void *const *w_qkv;  /* host array [layers] of device pointers */
    const void *const *w_o;
    const void *const *w_gu;
    const void *const *w_down;
    const void *w_head;
    const float *attn_norm;
    const float *ffn_norm;
    const float *out_norm;
    const float *embedding;
} te_qwen_step_desc;

TE_API te_status te_qwen_step_create(te_kv_cache *cache, const te_qwen_step_desc *desc, te_qwen_step **out_step);
TE_API te_status te_qwen_step_run(te_qwen_step *step, size_t seq, const int64_t *token, float *hidden,
                                  float *logits, int64_t *next_token, uint32_t flags);
TE_API void te_qwen_step_free(te_qwen_step *step);

/*
 * Allocation-free decode for callers that cannot allocate device memory:
 * code that runs where cudaMalloc is not allowed or would break its memory
 * plan (a host framework or plugin host that owns every device allocation, a
 * fixed-budget serving runtime, work issued from a context that must not
 * synchronise the device).  Such callers cannot create an engine, whose
 * decode scratch grows with cudaMalloc.  No counterpart in the reference
 * (TinyEngine's CPU and Metal paths allocate freely).
 *
 * One layer, one sequence: q[heads][head_dim] fp32 (used as given, already
 * rotated) attends the first n_tokens tokens of a caller-owned paged f16
 * cache laid out like one layer of the engine's pool,
 * k_pool/v_pool[num_pages][kv_heads][page_tokens][head_dim], with
 * page_table[i] = page holding tokens [i*page_tokens, (i+1)*page_tokens).
 * All pointers are device pointers; out[heads][head_dim] fp32.  Work is
 * queued on `stream` (cudaStream_t, NULL = legacy default stream) on the
 * current device; the call does not synchronise.
 *
 * The split-K scratch is a fixed 4 MiB + 1.25 KiB file-scope device array
 * that every GPU which loads this library holds until the process exits.
 * Limits: head_dim 64 or 128; heads / kv_heads <= 16; kv_heads <= 256.
 * The partial records take kv_heads * (heads / kv_heads) * (head_dim + 4) * 4
 * bytes per CTA segment and the split shrinks its grid until they fit, so
 * every shape within these limits fits the 4 MiB (at most 2.16 MB on a one-CTA
 * grid); the TE_STATUS_UNSUPPORTED check behind it is defensive.  The call
 * allocates nothing: no cudaMalloc or cudaFree and no allocating library
 * routine.
 *
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current), so make that first call
 * before any stream capture.  Every call shares the one array: calls whose
 * kernels overlap on the GPU (different streams, or different host threads)
 * race on it and must be serialised by the caller.  Counters and the error
 * word are cleared at the start of each call; a device-side wait that expires
 * (2 s) is not reported by this asynchronous call but left in the error word,
 * which te_attention_decode_paged_noalloc_status reads.
 */
TE_API te_status te_attention_decode_paged_noalloc(
    const uint16_t *k_pool, const uint16_t *v_pool, const int32_t *page_table,
    size_t num_pages, size_t page_tokens, size_t n_tokens,
    const float *q, size_t heads, size_t kv_heads, size_t head_dim,
    float *out, void *stream);

/* Synchronises `stream` (cudaStream_t, NULL = legacy default stream) and
 * reads the current device's error word of te_attention_decode_paged_noalloc:
 * *code = 0 and TE_STATUS_OK, or the code a bounded device-side wait of the
 * last call left (then cleared) and TE_STATUS_RUNTIME_ERROR.  Allocates
 * nothing.  The next te_attention_decode_paged_noalloc call on the device
 * clears the word, so read it before that call.  No counterpart in the
 * reference. */
TE_API te_status te_attention_decode_paged_noalloc_status(void *stream, int *code);

#ifdef __cplusplus
}
#endif

#endif
