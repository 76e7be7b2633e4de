// Internal declarations shared by the C-ABI layer (te_api.cpp) and the
// kernel translation units (*.cu).  Not installed; not part of the ABI.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/tinyengine_attn.h"

namespace te {

// Decode work description for one sequence, passed to the decode kernel by
// value (kernel parameter space), so a launch needs no host->device copy.
struct SeqEntry {
  int32_t slot;         // cache sequence slot (row of the page table)
  int32_t len;          // tokens attended (after the optional append)
  int32_t q_pos;        // RoPE position of the query
  int32_t new_pos;      // RoPE position of the appended token, or -1 (no append)
  int32_t stage_begin;  // first 64-token stage of this sequence within a (layer, kv head) block
  int32_t n_stages;     // max(1, ceil(old tokens / 64)): the stages of tokens cached before the call
  int32_t page_base;    // >= 0: the sequence's pages are page_base, page_base + 1, ... (no table read); -1: read the table
};

constexpr int kMaxParamSeqs = 64;  // sequences per decode launch
constexpr int kMaxExchangeRanks = 8;  // ranks of a KV-split exchange

// Raises a kernel's dynamic shared-memory limit to `bytes` once per device.
// The attribute applies to the current device only, so every device a
// process launches on needs its own call; `done` holds one bit per device
// ordinal (< 64) and may be shared by host threads (a repeated call is
// harmless).
inline cudaError_t set_smem_limit_once(std::atomic<uint64_t>& done, const void* kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  const uint64_t bit = 1ull << dev;
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

// Stream-K split: CTA b of `grid` owns stages [stage_start(b), stage_start(b+1)).
// Quotient of non-negative a / b; on the device a 32-bit divide when both fit
// (the 64-bit one is a long software sequence).
__host__ __device__ inline long long div_nonneg(long long a, long long b) {
#ifdef __CUDA_ARCH__
  if ((((unsigned long long)a | (unsigned long long)b) >> 32) == 0) return (long long)((unsigned)a / (unsigned)b);
#endif
  return a / b;
}
__host__ __device__ inline long long stage_start(long long b, long long total, long long grid) {
  return div_nonneg(b * total, grid);
}
// Floats per split-K scratch record: acc[head_dim], m, l, two pad (16-byte aligned records).
inline size_t decode_scratch_rec(int head_dim) { return (size_t)head_dim + 4; }

constexpr int kStageTokens = 64;   // tokens per TMA stage

struct DecodeParams {
  CUtensorMap tmap_k;  // 2-D view [rows][head_dim] of the K pool, box 64x64, 128B swizzle
  CUtensorMap tmap_v;
  const int32_t* page_table;  // [max_seqs][max_pages_per_seq]
  const float* q;             // [n_layers][n_seqs][heads][hd]
  const float* k_new;         // [n_layers][n_seqs][kv_heads][hd] or null
  const float* v_new;
  float* out;                 // normalised [..][heads][hd] or partial [..][heads][hd+2]
  float* partials;            // split-K scratch
  uint32_t* counters;         // [n_layers][kv_heads][n_seqs], zero between launches
  uint16_t* k_pool;           // for the fused append (generic stores)
  uint16_t* v_pool;
  const float* rope_cos;      // [max_position][hd/2]
  const float* rope_sin;
  const float* q_bias;        // null, or [cache layers][heads * hd] added to q before RoPE
  const float* k_bias;        // null, or [cache layers][kv_heads * hd] added to k_new / v_new
  const float* v_bias;
  int* error;
  int32_t n_seqs;             // sequences in this launch (<= kMaxParamSeqs)
  int32_t seq_total;          // sequences in the caller's arrays (row stride of q/out)
  int32_t seq_base;           // index of this launch's first sequence in those arrays
  int32_t layer_begin;
  int32_t n_layers;
  int32_t kv_heads;
  int32_t group;              // heads per kv head (<= 16)
  int32_t block_stages;       // stages of one (layer, kv head) block: sum of n_stages
  int32_t grid;               // CTAs sharing the stages (stream-K split)
  int32_t cluster_k;          // > 1: clusters of cluster_k CTAs, CTA b takes part b % k of group b / k
                              // and the parts combine in distributed shared memory; else stream-K
  int32_t max_segs;           // partial-record slots per CTA
  long long total_stages;     // n_layers * kv_heads * block_stages
  int32_t num_pages;          // pages per layer
  int32_t page_tokens;
  int32_t max_pages_per_seq;
  int32_t rope;               // 1: rotate q (and appended k)
  int32_t partial_out;        // 1: write partial records {acc, m, l} (stride hd + 2); 2: the same with stride
                              // hd + 4 (16-byte aligned rows), the fused KV-split exchange's records
  float scale_log2;           // log2(e) / sqrt(hd)
  // Fused KV-split exchange (xch_world > 1; one sequence; partial_out = 2):
  // every rank stores its record rows of each finished (layer, kv head) group
  // into its slot of every rank's gather area and counts the group there; at
  // the end of the kernel each rank's CTAs merge every group for the rank's
  // own output from local memory, once all world records have arrived
  // (bounded waits, xch_wait_ns).
  int32_t xch_world, xch_rank, xch_rows;
  uint64_t xch_wait_ns;
  float* xch_rec[kMaxExchangeRanks];      // every rank's gather area [2 parities][world][rows][hd + 4] (mapped)
  float* xch_out;                         // this rank's merged output [rows][hd]
  uint32_t* xch_cnt[kMaxExchangeRanks];   // every rank's per-group arrival counts (cumulative)
  uint32_t* xch_done;                     // this rank's {unused, CTA ticket, steps}
  SeqEntry seqs[kMaxParamSeqs];
};
static_assert(sizeof(DecodeParams) <= 4096, "decode parameters exceed the kernel parameter space");

// 2-D f16 tensor map over [rows][cols] (box box_rows x 64, 128B swizzle); false on failure.
bool encode_tmap_f16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows);

// Tokens of sequence entry i cached before the call: the appended token (if
// any) is not streamed from the cache but scored from its k/v rows.
__host__ __device__ inline int old_tokens(const DecodeParams& p, int i) {
  return p.seqs[i].len - ((p.seqs[i].new_pos >= 0 && p.k_new != nullptr) ? 1 : 0);
}

// Plans the stream-K split of a decode launch: fills each sequence's stage
// range (from its old tokens), block_stages, total_stages, grid (<= max_grid CTAs,
// at least one stage each) and max_segs (groups any one CTA touches).
inline void plan_stream_k(DecodeParams& p, long long max_grid) {
  int acc = 0;
  for (int i = 0; i < p.n_seqs; ++i) {
    const int n_old = old_tokens(p, i);
    p.seqs[i].n_stages = n_old > 0 ? (n_old + kStageTokens - 1) / kStageTokens : 1;
    p.seqs[i].stage_begin = acc;
    acc += p.seqs[i].n_stages;
  }
  p.block_stages = acc;
  p.total_stages = (long long)p.n_layers * p.kv_heads * acc;
  long long grid = max_grid < p.total_stages ? max_grid : p.total_stages;
  if (grid < 1) grid = 1;
  p.grid = (int32_t)grid;
  auto gidx = [&](long long st) {
    const long long blk = st / acc;
    const int rem = (int)(st - blk * acc);
    int lo = 0, hi = p.n_seqs - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.seqs[mid].stage_begin <= rem) lo = mid; else hi = mid - 1;
    }
    return blk * p.n_seqs + lo;
  };
  long long segs = 1;
  for (long long b = 0; b < grid; ++b) {
    const long long s0 = stage_start(b, p.total_stages, grid);
    const long long s1 = stage_start(b + 1, p.total_stages, grid) - 1;
    const long long n = gidx(s1) - gidx(s0) + 1;
    if (n > segs) segs = n;
  }
  p.max_segs = (int32_t)segs;
}

// Cluster split, when every (layer, kv head, sequence) group can take k >= 2
// whole SMs (k = 2 or 4, at most one CTA per SM, each part >= 1 stage): the
// split-K combine then stays in distributed shared memory.  Otherwise keeps
// the stream-K plan.
inline void plan_cluster(DecodeParams& p, int sm_count) {
  p.cluster_k = 0;
  const long long groups = (long long)p.n_layers * p.kv_heads * p.n_seqs;
  if (groups <= 0) return;
  long long k = sm_count / groups;
  if (k < 2) return;
  k = k >= 4 ? 4 : 2;
  for (int i = 0; i < p.n_seqs; ++i) {
    if (p.seqs[i].n_stages < k) return;
  }
  p.cluster_k = (int32_t)k;
  p.grid = (int32_t)(groups * k);
  p.max_segs = 1;
}

// Launchers (kernels live in the .cu files).  All return cudaError_t of the launch.
cudaError_t launch_decode_f16(const DecodeParams& p, int head_dim, cudaStream_t s);
cudaError_t launch_decode_f32_generic(const float* q, const float* k, const float* v, float* scores, float* out,
                                      size_t n_tokens, int heads, int kv_heads, int head_dim, cudaStream_t s);
cudaError_t launch_rope_rows(float* values, const float* cos_row, const float* sin_row, int heads, int head_dim,
                             cudaStream_t s);
cudaError_t launch_merge_partials(const float* partials, int n_parts, int rows, int head_dim, float* out,
                                  int partial_out, cudaStream_t s);
// Host-visible (pinned, device-mapped) buffers copied to device memory by one
// kernel: chunks[i] 16-byte units from src[i] to dst[i], both 16-byte aligned.
struct GatherParams {
  const void* src[3];
  void* dst[3];
  size_t chunks[3];
  int32_t n;
};
cudaError_t launch_gather_host(const GatherParams& p, cudaStream_t s);

struct AppendParams {
  const void* k;            // [n_layers][n_tokens][kv_heads][hd], fp32 or f16
  const void* v;
  uint16_t* k_pool;
  uint16_t* v_pool;
  const int32_t* page_row;  // page table row of the sequence
  const float* rope_cos;
  const float* rope_sin;
  const float* k_bias;      // null, or [cache layers][kv_heads * hd] added before RoPE / rounding
  const float* v_bias;
  int32_t input_f16;
  int32_t rope;
  int32_t n_layers;
  int32_t layer_begin;
  int32_t n_tokens;
  int32_t first_index;      // local token index of the first new token
  int32_t first_pos;        // global RoPE position of the first new token
  int32_t kv_heads;
  int32_t head_dim;
  int32_t num_pages;
  int32_t page_tokens;
  int* error;               // engine error word (bounded waits of the streamed variant)
};
cudaError_t launch_append_rope(const AppendParams& p, cudaStream_t s);

// Rotates (optionally) and converts prefill queries to f16 in the same
// [n_layers][n_tokens][heads][hd] layout (the prefill kernel reads f16 queries)
struct QPrepParams {
  const void* q;            // [n_layers][n_tokens][heads][hd], fp32 or f16
  __half* qh;               // same layout, f16
  const float* rope_cos;
  const float* rope_sin;
  const float* q_bias;      // null, or [cache layers][heads * hd] added before RoPE / rounding
  int32_t input_f16;
  int32_t rope;
  int32_t n_layers;
  int32_t layer_begin;      // cache layer of local layer 0 (bias rows)
  int32_t n_tokens;
  int32_t heads;
  int32_t head_dim;
  int32_t first_pos;
  int32_t split;            // 1: write each query row as two f16 rows, hi = f16(q) and lo = f16(q - hi):
                            // qh [n_layers][n_tokens][heads][2][hd]
};
cudaError_t launch_q_prep(const QPrepParams& p, cudaStream_t s);
// One pass over a prefill call's inputs: the K/V append of `a` and, when
// with_q, the query preparation of `q` (same layers and tokens).
cudaError_t launch_prefill_prep(const AppendParams& a, const QPrepParams& q, bool with_q, int sm_count,
                                cudaStream_t s);

struct PrefillParams {
  CUtensorMap tmap_q;   // f16 queries [n_layers][n_tokens][heads][hd], box 64 x 1 x 64 x 1, 128B swizzle
                        // (rows past n_tokens read as zeros)
  CUtensorMap tmap_k;   // K pool view (as for decode)
  CUtensorMap tmap_v;
  const int32_t* page_table_row;  // page table row of the sequence
  float* out;           // [n_layers][n_tokens][heads][hd]
  int* error;
  int32_t n_layers;
  int32_t layer_begin;
  int32_t heads;
  int32_t kv_heads;
  int32_t n_tokens;
  int32_t n_tokens_padded;  // multiple of 128
  int32_t q_offset;     // tokens cached before the first new token
  int32_t num_pages;    // pages per layer in the pool
  int32_t page_tokens;
  int32_t n_pages_mapped;  // mapped pages of the sequence (covers q_offset + n_tokens)
  int32_t n_items;      // work items (prefill_items)
  int32_t head_dim;     // 64 or 128
  int32_t split;        // 1: queries as hi/lo f16 rows (tmap_q over 2 * heads rows per token), one head per item
  float scale_log2;
};
cudaError_t launch_prefill_tc(const PrefillParams& p, int sm_count, cudaStream_t s);
// Work items of the prefill kernel: (layer, kv head, query-head pair -- or one
// head when split --, 128-query tile).
int prefill_items(int n_layers, int heads, int kv_heads, int n_tokens_padded, bool split);

// KV-split exchange over NVLink (k_exchange.cu): one kernel per decode step
// pushes this rank's partial records into every rank's exchange area and
// merges the rows once the peers' pushes have arrived.
struct ExchangeParams {
  const float* partial;                 // this rank's records [rows][head_dim + 2]
  float* out;                           // merged [rows][head_dim]
  float* base[kMaxExchangeRanks];       // every rank's exchange area (this process's mapping)
  uint32_t* steps;                      // this rank's per-CTA step counts
  int* error;
  int32_t world, rank, rows, head_dim, rows_per_cta, grid;
  uint64_t wait_ns;                     // bound of the wait for the peers' pushes
};
size_t exchange_area_bytes(int world, int rows, int head_dim, int grid);
// Regions of the fused KV-split exchange (te_attention_decode_kv_split) in
// the same area, after the push exchange's: byte offsets, 256-byte aligned.
struct FusedLayout {
  size_t rec;   // gather area [2 parities][world][rows][head_dim + 4] fp32: every rank's records
  size_t out;   // merged output [rows][head_dim] fp32 (written by this rank's decode)
  size_t cnt;   // per-group arrival counters [rows] u32 (groups <= rows)
  size_t done;  // {merged groups, CTA ticket, completed steps, pad} u32
  size_t end;
};
inline FusedLayout fused_layout(size_t push_bytes, int world, int rows, int head_dim) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  FusedLayout f;
  f.rec = up(push_bytes);
  f.out = up(f.rec + 2 * (size_t)world * rows * (head_dim + 4) * sizeof(float));
  f.cnt = up(f.out + (size_t)rows * head_dim * sizeof(float));
  f.done = up(f.cnt + (size_t)rows * sizeof(uint32_t));
  f.end = up(f.done + 4 * sizeof(uint32_t));
  return f;
}
int exchange_grid(int rows);
cudaError_t launch_exchange_merge(const ExchangeParams& p, cudaStream_t s);

// GGUF Q4_0 / Q8_0 matrix-vector products (k_gemv.cu).
struct GemvParams {
  const void* w;            // [rows][cols / 32 blocks], 16-byte aligned base
  const float* x;           // [n_vectors][cols]
  float* y;                 // [n_vectors][rows]
  int32_t rows, cols;
  int32_t rows_per_group;   // set by the launcher
  int32_t stage_bytes;      // set by the launcher
  int32_t stages;           // set by the launcher (2..4)
  int32_t accumulate;       // 1: y += W x (fp32 add of each finished dot product)
  int* error;               // engine error word (a staging wait that ran out)
  int32_t prologue;         // 0: x as given; 1: RMSNorm(x) * norm_w; 2: SwiGLU of x = [gate | up] (one vector)
  const float* norm_w;      // RMSNorm weight [cols] (prologue 1)
  float eps;                // RMSNorm epsilon (prologue 1)
};
// block_bytes 18 (Q4_0) or 34 (Q8_0); 1 <= n_vectors <= 8.
cudaError_t launch_gemv_gguf(GemvParams p, int block_bytes, int n_vectors, int sm_count, cudaStream_t s);

// ---- whole-token qwen2 decode step (k_step.cu) -----------------------------
// One cooperative launch runs every layer of one token: CTA b owns a fixed
// slice of rows of every projection, and its share of all weights is packed
// into one contiguous, 16-byte aligned byte stream (stages of whole rows, in
// the order the kernel consumes them), which a producer warp copies into a
// shared-memory ring ahead of the consumer warps, across phase boundaries.
enum StepKind { kStepQKV = 0, kStepO = 1, kStepGU = 2, kStepDown = 3, kStepHead = 4, kStepKinds = 5 };
constexpr int kStepMaxStageRows = 64;  // rows per stage: one or two per lane (gate/up: 32 pairs)
constexpr int kStepMaxSlots = 32;      // stages in flight (mbarrier pairs)
constexpr int kStepChunk = 128;        // attention tokens per work item
constexpr int kStepMaxGroup = 16;      // query heads per kv head
constexpr int kStepMaxOwnRows = 64;    // rows of x one CTA owns (hidden <= 64 * grid)
constexpr int kStepMaxLayers = 127;    // layers a tag can name
// Attention work area of the step kernel (queries, scores, row maxima and
// sums, pool row ids, the chunk's V and K rows in f16).
constexpr int step_attn_bytes(int head_dim) {
  return 4 * (kStepMaxGroup * head_dim + kStepMaxGroup * kStepChunk + 2 * kStepMaxGroup + kStepChunk) +
         2 * 2 * kStepChunk * head_dim;
}

struct StepMat {
  int32_t rows, cols;
  int32_t block_bytes;  // 18 (Q4_0) or 34 (Q8_0)
  int32_t row_bytes;    // cols / 32 * block_bytes
  int32_t rpc;          // rows per CTA (CTA b: rows [b * rpc, min(rows, (b + 1) * rpc)))
  int32_t rps;          // most rows per stage
  int32_t pair;         // 1: gate/up -- row r is gate row r and up row r (rows = ffn); a stage of R
                        // rows holds the R gate rows, then the R up rows
};

// Rows of matrix m owned by CTA b (first row in r0).
__host__ __device__ inline int step_cta_rows(const StepMat& m, int b, int& r0) {
  r0 = b * m.rpc;
  const int r1 = r0 + m.rpc < m.rows ? r0 + m.rpc : m.rows;
  return r1 > r0 ? r1 - r0 : 0;
}
__host__ __device__ inline int step_n_stages(int n, int rps) { return n > 0 ? (n + rps - 1) / rps : 0; }
// Stage s of n rows split into ns stages covers rows [lo(s), lo(s + 1)):
// n / ns rows each, the first n % ns stages one more.
__host__ __device__ inline int step_stage_lo(int s, int n, int ns) {
  const int q = n / ns, rem = n - q * ns;
  return s * q + (s < rem ? s : rem);
}
// A stage of `rows` physical rows of nb blocks is stored transposed, so that
// each block's parts are aligned and consecutive rows of one block are
// consecutive in shared memory: first the f16 scales [nb][rows], padded to 16
// bytes, then the quants in 16-byte chunks -- Q4_0 [nb][rows] x 16 bytes,
// Q8_0 [nb][2][rows] x 16 bytes (first and second half of the 32 int8).
__host__ __device__ inline uint32_t step_scale_bytes(int rows, int nb) {
  return ((uint32_t)rows * (uint32_t)nb * 2u + 15u) & ~15u;
}
__host__ __device__ inline uint32_t step_stage_bytes(int rows, int nb, int block_bytes) {
  return step_scale_bytes(rows, nb) + (uint32_t)rows * (uint32_t)nb * (uint32_t)(block_bytes - 2);
}

struct StepParams {
  const unsigned char* wpack;  // packed weight streams
  const long long* cta_off;    // [grid + 1] byte offset of each CTA's stream
  StepMat mat[kStepKinds];
  int32_t layers, hidden, heads, kv_heads, head_dim, ffn, vocab, group;
  float eps;
  float scale_log2;            // log2(e) / sqrt(head_dim)
  // KV cache (one sequence)
  uint16_t* k_pool;
  uint16_t* v_pool;
  const int32_t* page_row;     // the sequence's page-table row
  int32_t page_base;           // >= 0: pages are page_base, page_base + 1, ... (no table read)
  int32_t num_pages, page_tokens;
  int32_t n_tokens;            // tokens attended, the new one included (its cache index is n_tokens - 1)
  int32_t rope_pos;            // RoPE position of the new token (= of the query)
  const float* rope_cos;       // [max_position][head_dim / 2]
  const float* rope_sin;
  const float* q_bias;         // null, or [layers][heads * head_dim]
  const float* k_bias;         // null, or [layers][kv_heads * head_dim]
  const float* v_bias;
  const float* attn_norm;      // [layers][hidden]
  const float* ffn_norm;       // [layers][hidden]
  const float* out_norm;       // [hidden]
  const float* emb;            // [vocab][hidden] fp32
  const int64_t* token_in;     // device: this step's token
  int64_t* token_out;          // device: the greedy next token (head only)
  float* x;                    // [hidden] out: the hidden state after the last layer
  // Vectors passed between CTAs as 64-bit words {value bits, tag}:
  unsigned long long* ll_qkv;  // [heads * hd + 2 * kv_heads * hd]
  unsigned long long* ll_attn; // [heads * hd]
  unsigned long long* ll_h;    // [ffn] SwiGLU(gate, up): the down projection's input
  unsigned long long* ll_x[2]; // [hidden] x after the output projection / after the down projection
  float* logits;               // [vocab] (head only)
  float* rec;                  // attention partial records [kv_heads][chunks][group][hd + 2]
  float* cand;                 // [grid][2] per-CTA argmax candidates
  uint32_t* sync;              // [1] exit count, [2] argmax ticket, [3] launch epoch, [4 + g] merge count of kv head g
  int* error;
  int32_t head;                // 1: output RMSNorm + lm_head + argmax after the layers
  int32_t ring_bytes;          // weight ring (shared memory after the work area)
  int32_t union_bytes;         // phase work area
};
// Plans matrix m's split over `grid` CTAs with stages of at most stage_max bytes.
void plan_step_mat(StepMat& m, int rows, int cols, int block_bytes, int grid, int stage_max, int pair);
// Shared memory of the step kernel for these sizes.
int step_smem_bytes(int ring_bytes, int union_bytes);
int step_fixed_smem();
cudaError_t step_configure();  // raises the kernel's shared-memory limit on the current device
int step_max_ctas_per_sm(int smem);
cudaError_t launch_step(const StepParams& p, int grid, int smem, cudaStream_t s);
// Packing: one segment per stage.  Physical row r of the stage is source row
// src0 + r * row_bytes for r < split, else src1 + (r - split) * row_bytes (the
// gate/up pairs' second half); written transposed at dst + dst_off.
struct StepPackSeg {
  const void* src0;
  const void* src1;
  long long dst_off;
  int32_t rows, split, nb, block_bytes;
};
cudaError_t launch_step_pack(const StepPackSeg* segs, int n, unsigned char* dst, cudaStream_t s);

}  // namespace te
