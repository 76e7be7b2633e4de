// Split-K GQA flash decode over the paged f16 KV cache (sm_100a).
//
// One launch covers every (layer, kv head, sequence) group of a decode call.
// A CTA serves the whole GQA group of its kv head (up to 16 query heads), so
// every cached K/V byte is read from HBM exactly once per step.  Reference
// semantics: te_attention_decode_f32 (c/src/ops.c:323-395) with f16 K/V
// widened exactly, as in te_attention_flash_h_f32_kernel
// (c/src/metal/metal_kernels.metal.inc:3374-3495); the group-shared KV read
// follows te_attention_flash_gqa_f32_kernel (:3209-3372).
//
// Work split: stream-K (equal stage ranges per persistent CTA over all groups'
// 64-token stages) or, when every group can take k = 2 or 4 SMs, one
// thread-block cluster of k CTAs per group.  Parts of a split group combine by
// log-sum-exp: through distributed shared memory inside a cluster, otherwise
// through per-part records in scratch, folded by the last part to finish
// (atomic ticket, no waiting) in part order.
//
// Pipeline: the producer warp streams 64-token stages (K and V, 128B-swizzled
// 64x64 TMA boxes) into a ring of `R` shared-memory slots; warps 0-3 each take
// 16 tokens of every stage.  Scores S = Q K^T and O += P V run on
// mma.sync.m16n8k16 (f16 in, f32 accumulate) with the query heads as the M
// rows.  The head dimension is permuted per thread so that every operand
// fragment is one 16-byte shared-memory load (conflict-free under the swizzle)
// and the query fragments stay in registers for a whole segment; the
// permutation is applied identically to q and k, so q.k is unchanged.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstring>
#include <mutex>

#include "te_internal.h"
#include "te_ptx.cuh"
#include "te_rope.cuh"

namespace te {
namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 3) * 32;  // + producer, helper and appender warps
constexpr int kBoxBytes = kStageTokens * 64 * 2;  // 64 tokens x 64 dims x f16

// Shared-memory plan for head dim HD and GP = 8 or 16 padded query rows per
// group: a ring of 64-token K/V stages, and double-buffered query, RoPE,
// fragment and merge areas so one item's prologue/epilogue overlaps the next
// item's streaming.
template <int HD, int GP>
struct DecodeCfg {
  static constexpr int kBoxes = HD / 64;                   // TMA boxes per K (or V) stage
  static constexpr int kStageBytes = 2 * kBoxes * kBoxBytes;
  static constexpr int kKSteps = HD / 16;                  // mma k-steps for q.k
  static constexpr int kChunksPerThread = HD / 32;         // 16-byte chunks of a K row per thread
  static constexpr int kNTiles = HD / 8;                   // mma n-tiles for P.V
  static constexpr int kRing = HD == 128 ? (GP == 8 ? 5 : 3) : 8;  // K/V stages in flight
  static constexpr int kRowF = HD + 4;                     // padded row stride (floats): rows 4 banks apart
  static constexpr int kMergeBytes = kConsumerWarps * GP * kRowF * 4;  // one buffer: per-warp O
  static constexpr int kQBytes = GP * kRowF * 4;           // one buffer: raw q rows of the group
  static constexpr int kCSBytes = HD * 4;                  // one buffer: cos row + sin row
  // One buffer: the f16 query fragments of a warp.  GP = 8 carries each head's
  // low part in the padding rows 8-15 of the same fragments; GP = 16 needs a
  // second set of fragments for the low parts.
  static constexpr int kFragSet = kKSteps * 4 * 4 * 32;
  static constexpr int kFragBytes = kFragSet * (GP == 16 ? 2 : 1);
  static constexpr int kMLFloats = 2 * kConsumerWarps * 16;  // one buffer: m[4][16], l[4][16]
  static constexpr int kNewBytes = 3 * HD * 4;             // one buffer: new token's raw k, v, and cos/sin row
  static constexpr int kResBytes = (16 + HD) * 4;          // one buffer: new token's scores[16], v[HD] (as cached)
  static constexpr int kOffMerge = kRing * kStageBytes;
  static constexpr int kOffQ = kOffMerge + 2 * kMergeBytes;
  static constexpr int kOffCS = kOffQ + 2 * kQBytes;
  static constexpr int kOffFrag = kOffCS + 2 * kCSBytes;
  static constexpr int kOffML = kOffFrag + 2 * kFragBytes;
  static constexpr int kOffNew = kOffML + 2 * kMLFloats * 4;
  static constexpr int kOffRes = kOffNew + 2 * kNewBytes;
  static constexpr int kOffBar = kOffRes + 2 * kResBytes;
  static constexpr int kNumBars = 2 * kRing + 15;  // full, empty, [2] each: qfull qempty fready fempty mready mfree nready; cbar
  static constexpr int kOffFlag = kOffBar + kNumBars * 8;  // a flag word of the fused KV-split exchange
  static constexpr int kSmemBytes = kOffFlag + 16 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory plan exceeds the per-CTA limit");
};

// Split-K partial records in scratch: { acc[HD], m, l, pad, pad } so every
// record starts on a 16-byte boundary.
template <int HD>
constexpr int kScratchRec = HD + 4;

// Physical head-dim offset (in 16-byte chunks within a 64-column box) that a
// thread with quad index c reads for k-step pair j, and the box it lies in.
template <int HD>
__device__ __forceinline__ int k_chunk_of(int c, int j, int* box) {
  constexpr int per_thread = HD / 32;
  constexpr int threads_per_box = 8 / per_thread;
  *box = c / threads_per_box;
  return per_thread * (c % threads_per_box) + ((j + c) % per_thread);
}

// Stream-K work: the stages of all (layer, kv head, sequence) groups are laid
// end to end and CTA b owns the contiguous range [start(b), start(b+1)); a
// segment is the part of that range inside one group.  A CTA walks its range
// from the end: a group's newest stage (the one the fused append writes) sits
// at the start of a range, so the append's small loads, which would wait
// behind the kernel's initial K/V burst, come after the CTA's other segments.
struct Seg {
  int layer_local, kvh, si, gidx;  // gidx = (layer_local * kv_heads + kvh) * n_seqs + si
  int t0, t1, n_st;                // tokens [t0, t1) of the group, in n_st stages
  long long s_begin;               // first stage of this segment (where the next one processed ends)
  long long gs0, gs1;              // the group's stage range
};

// The group holding stage s (fills si, layer_local, kvh, gidx, gs0, gs1).
__device__ __forceinline__ Seg group_at(const DecodeParams& p, long long s) {
  Seg g;
  const int blk = (int)div_nonneg(s, p.block_stages);
  const int rem = (int)(s - (long long)blk * p.block_stages);
  int lo = 0, hi = p.n_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.seqs[mid].stage_begin <= rem) lo = mid; else hi = mid - 1;
  }
  g.si = lo;
  g.layer_local = blk / p.kv_heads;
  g.kvh = blk - g.layer_local * p.kv_heads;
  g.gidx = blk * p.n_seqs + lo;
  g.gs0 = (long long)blk * p.block_stages + p.seqs[lo].stage_begin;
  g.gs1 = g.gs0 + p.seqs[lo].n_stages;
  return g;
}

// The segment of [s_lo, s_hi) that ends at s_hi.
__device__ __forceinline__ Seg seg_ending(const DecodeParams& p, long long s_hi, long long s_lo) {
  Seg g = group_at(p, s_hi - 1);
  g.s_begin = max(s_lo, g.gs0);
  g.t0 = (int)(g.s_begin - g.gs0) * kStageTokens;
  g.t1 = min(old_tokens(p, g.si), (int)(s_hi - g.gs0) * kStageTokens);
  g.n_st = (int)(s_hi - g.s_begin);
  return g;
}

// A segment that ends at its group's last stage carries the group's new token
// (when the call appends one): the helper appends it and folds its score into
// the segment's merge; K/V stages cover only the tokens cached before.
__device__ __forceinline__ bool seg_has_new(const DecodeParams& p, const Seg& w) {
  return p.seqs[w.si].new_pos >= 0 && p.k_new != nullptr && w.s_begin + w.n_st == w.gs1;
}

// Final result of one query-head row, 4 dims at d: normalised output, or the
// public partial record {acc[HD], m, l} when the caller asked for partials.
template <int HD>
__device__ __forceinline__ void store_result(const DecodeParams& p, size_t orow, int d, const float4& O, float M,
                                             float L) {
  if (!p.partial_out) {
    const float inv = 1.f / L;
    *reinterpret_cast<float4*>(p.out + orow * HD + d) = make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
  } else if (p.partial_out == 2) {
    // fused exchange: into this rank's slot of every rank's gather area, the
    // half of the step's parity (16-byte aligned rows)
    const uint32_t par = *reinterpret_cast<volatile const uint32_t*>(p.xch_done + 2) & 1u;
    const size_t off = (((size_t)par * p.xch_world + p.xch_rank) * p.xch_rows + orow) * (HD + 4);
#pragma unroll 1
    for (int w = 0; w < p.xch_world; ++w) {
      float* r = p.xch_rec[w] + off;
      *reinterpret_cast<float4*>(r + d) = O;
      if (d == 0) *reinterpret_cast<float2*>(r + HD) = make_float2(M, L);
    }
  } else {
    float* r = p.out + orow * (HD + 2);
    *reinterpret_cast<float2*>(r + d) = make_float2(O.x, O.y);
    *reinterpret_cast<float2*>(r + d + 2) = make_float2(O.z, O.w);
    if (d == 0) *reinterpret_cast<float2*>(r + HD) = make_float2(M, L);
  }
}

// Named barrier of the four consumer warps (barrier 0 is __syncthreads).
__device__ __forceinline__ void consumer_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Fused KV-split exchange, arrival: the NT threads that stored group gidx's
// records into every rank's gather area (sync = a barrier of exactly them)
// count the group there.  One system-scope release fence by thread 0
// (cumulative over the stores the barrier ordered before it), then relaxed
// counts; nothing waits.
template <typename Sync>
__device__ __forceinline__ void xch_group_finished(const DecodeParams& p, int gidx, int t, Sync sync) {
  sync();
  if (t == 0) {
    fence_acq_rel_sys();
    for (int w = 0; w < p.xch_world; ++w) red_add_relaxed_sys(p.xch_cnt[w] + gidx, 1u);
  }
}

// Fused KV-split exchange, end of the kernel on this rank (the 128 consumer
// threads of every CTA, after their last segment).  CTA b merges groups
// g = b, b + grid, ... for this rank's own output: it waits (bounded) until
// every rank's record of g has arrived in the local gather area, combines
// them by log-sum-exp (te_attention_merge_partials' rescale) from local
// memory and writes the merged rows.  The kernel's completion then orders the
// whole output before later work on the stream.  Counts are cumulative; the
// gather area has two halves (step parity): a rank can be at most one step
// ahead of another, since its step s + 1 merges need every rank's step s + 1
// records.  done = {unused, CTA ticket, steps}.
template <int HD>
__device__ __noinline__ void xch_finish(const DecodeParams& p, int t, volatile uint32_t* flag) {
  constexpr int REC = HD + 4;
  constexpr int kC = HD / 4;
  const int world = p.xch_world;
  const int G = p.group;
  const uint32_t groups = (uint32_t)(p.n_layers * p.kv_heads * p.n_seqs);
  uint32_t* done = p.xch_done;
  const uint32_t step = *reinterpret_cast<volatile uint32_t*>(done + 2);  // advanced only after every ticket
  const float* area = p.xch_rec[p.xch_rank] + (size_t)(step & 1u) * world * p.xch_rows * REC;
  const uint32_t* cnt = p.xch_cnt[p.xch_rank];
  float* out = p.xch_out;
  for (uint32_t g = blockIdx.x; g < groups; g += (uint32_t)p.grid) {
    if (t == 0) {
      const uint32_t target = (step + 1u) * (uint32_t)world;
      uint32_t ok = 1u;
      if ((int32_t)(ld_acquire_sys_u32(cnt + g) - target) < 0) {
        const uint64_t start = globaltimer_ns();
        while ((int32_t)(ld_acquire_sys_u32(cnt + g) - target) < 0) {
          if (globaltimer_ns() - start > p.xch_wait_ns) {
            set_error(p.error, 42);
            ok = 0u;
            break;
          }
        }
      }
      *flag = ok;
    }
    consumer_bar_sync();
    const uint32_t ok = *flag;
    consumer_bar_sync();
    if (!ok) continue;
    const size_t orow0 = (size_t)g * G;
    for (int i = t; i < G * kC; i += 128) {
      const size_t orow = orow0 + i / kC;
      const int c = (i % kC) * 4;
      float2 ml[kMaxExchangeRanks];
      float4 a[kMaxExchangeRanks];
#pragma unroll
      for (int w = 0; w < kMaxExchangeRanks; ++w) {
        if (w < world) {
          const float* r = area + ((size_t)w * p.xch_rows + orow) * REC;
          ml[w] = __ldcg(reinterpret_cast<const float2*>(r + HD));
          a[w] = __ldcg(reinterpret_cast<const float4*>(r + c));
        }
      }
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kMaxExchangeRanks; ++w) {
        if (w < world && ml[w].y > 0.f) M = fmaxf(M, ml[w].x);
      }
      float L = 0.f;
      float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int w = 0; w < kMaxExchangeRanks; ++w) {
        if (w >= world || !(ml[w].y > 0.f)) continue;
        const float sw = ex2(ml[w].x - M);
        L += ml[w].y * sw;
        O.x += a[w].x * sw;
        O.y += a[w].y * sw;
        O.z += a[w].z * sw;
        O.w += a[w].w * sw;
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      *reinterpret_cast<float4*>(out + orow * HD + c) = make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
    }
  }
  consumer_bar_sync();
  if (t != 0) return;
  __threadfence();
  const uint32_t ticket = atomicAdd(done + 1, 1u);
  if (ticket != (uint32_t)p.grid - 1u) return;
  done[1] = 0u;
  done[2] = step + 1u;  // every CTA has read the step (before its ticket)
}

// CTA owning stage s: the b with start(b) <= s < start(b + 1).
__device__ __forceinline__ int cta_of(const DecodeParams& p, long long s) {
  return (int)(div_nonneg((s + 1) * p.grid + p.total_stages - 1, p.total_stages) - 1);
}

// One step of the split-K combine, taken in part order: (M, L, O) absorbs
// the record (m, l, o).  Explicit roundings, so every code path that combines
// a group (helper or consumer warps, whichever CTA finishes last) computes
// bit-identical results.
__device__ __forceinline__ void fold_part(float& M, float& L, float4& O, float m, float l, const float4& o) {
  if (m == -INFINITY) return;
  const float mn = fmaxf(M, m);
  const float a = M == -INFINITY ? 0.f : ex2(__fsub_rn(M, mn));
  const float bw = ex2(__fsub_rn(m, mn));
  L = __fmaf_rn(L, a, __fmul_rn(l, bw));
  O.x = __fmaf_rn(O.x, a, __fmul_rn(o.x, bw));
  O.y = __fmaf_rn(O.y, a, __fmul_rn(o.y, bw));
  O.z = __fmaf_rn(O.z, a, __fmul_rn(o.z, bw));
  O.w = __fmaf_rn(O.w, a, __fmul_rn(o.w, bw));
  M = mn;
}


// Scratch offset (floats) of the split-K record CTA bp wrote for group gidx:
// its segment jp = gidx - (group of bp's first stage).
template <int HD>
__device__ __forceinline__ long long record_offset(const DecodeParams& p, int bp, int gidx) {
  const int jp = gidx - group_at(p, stage_start(bp, p.total_stages, p.grid)).gidx;
  return ((long long)bp * p.max_segs + jp) * p.group * kScratchRec<HD>;
}

// Persistent: one CTA per SM loops over work items (round-robin over the grid).
//   warps 0-3  consumers: each takes 16 tokens of every K/V stage (mma.sync
//              S = Q K^T, online softmax, O += P V) and parks its state
//   warp 4     producer: query/RoPE (and new k/v) row prefetch, K/V TMA ring
//   warp 5     helper: rotates each item's query into f16 fragments ahead of
//              the consumers; appends the new token (RoPE, f16) and scores
//              it; merges the four consumer states and the new token of each
//              finished item into the output (or a split-K partial record)
template <int HD, int GP>
__global__ void __launch_bounds__(kThreads, 1) decode_f16_kernel(const __grid_constant__ DecodeParams p) {
  using C = DecodeCfg<HD, GP>;
  constexpr int R = C::kRing;
  constexpr int REC = kScratchRec<HD>;
  constexpr int half = HD / 2;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kOffBar);
  uint64_t* empty = full + R;
  uint64_t* qfull = empty + R;   // [2] producer -> helper
  uint64_t* qempty = qfull + 2;  // [2] helper -> producer
  uint64_t* fready = qempty + 2; // [2] helper -> consumers
  uint64_t* fempty = fready + 2; // [2] consumers -> helper
  uint64_t* mready = fempty + 2; // [2] consumers -> helper
  uint64_t* mfree = mready + 2;  // [2] helper -> consumers, appender
  uint64_t* nready = mfree + 2;  // [2] appender -> helper
  uint64_t* cbar = nready + 2;   // cluster mode, rank 0: one arrival per CTA of the cluster (records placed)

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = p.group;
  const int H = p.group * p.kv_heads;
  // This CTA's stage range: a stream-K slice of all groups' stages or, in
  // cluster mode, part (b % k) of group (b / k).
  long long s_beg, s_end;
  if (p.cluster_k > 1) {
    const int g = blockIdx.x / p.cluster_k, part = blockIdx.x % p.cluster_k;
    const int blk = g / p.n_seqs, si = g - blk * p.n_seqs;
    const long long gs0 = (long long)blk * p.block_stages + p.seqs[si].stage_begin;
    const int n = p.seqs[si].n_stages;
    s_beg = gs0 + (long long)part * n / p.cluster_k;
    s_end = gs0 + (long long)(part + 1) * n / p.cluster_k;
  } else {
    s_beg = stage_start(blockIdx.x, p.total_stages, p.grid);
    s_end = stage_start(blockIdx.x + 1, p.total_stages, p.grid);
  }

  if (tid == 0) {
    for (int i = 0; i < R; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kConsumerWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&qfull[b], 1);
      mbar_init(&qempty[b], 2);  // helper and appender
      mbar_init(&fready[b], 1);
      mbar_init(&fempty[b], kConsumerWarps);
      mbar_init(&mready[b], kConsumerWarps);
      mbar_init(&mfree[b], 1);
      mbar_init(&nready[b], 1);
    }
    mbar_init(cbar, p.cluster_k > 1 ? p.cluster_k : 1);
    fence_mbarrier_init();
  }
  if (tid == 32 * kConsumerWarps) {
    prefetch_tmap(&p.tmap_k);
    prefetch_tmap(&p.tmap_v);
  }
  __syncthreads();
  if (p.cluster_k > 1) cluster_sync_all();  // every CTA's barriers exist before any remote arrival
  // Launched as a programmatic dependent: everything above overlaps the
  // previous kernel's tail.  Every warp waits for that kernel (griddep_wait)
  // before its first global read or write; the producer first asks L2 for
  // its first stages (prefetch hints touch no memory state the previous
  // kernel could race with: L2 stays coherent with its writes).  The next
  // kernel may be scheduled as soon as every CTA has started.
  griddep_launch_dependents();
  if (warp != kConsumerWarps) griddep_wait();

  if (warp == kConsumerWarps) {
    // ---- producer warp: q prefetch + K/V TMA ring -----------------------------
    if (lane == 0 && s_end > s_beg) {
      const Seg w0 = seg_ending(p, s_end, s_beg);
      const SeqEntry se0 = p.seqs[w0.si];
      if (se0.page_base >= 0) {  // page ids without reading the table
        const int layer0 = p.layer_begin + w0.layer_local;
        for (int s = 0; s < w0.n_st && s < R; ++s) {
          const int tok = w0.t0 + s * kStageTokens;
          const int row = ((layer0 * p.num_pages + se0.page_base + tok / p.page_tokens) * p.kv_heads + w0.kvh) *
                              p.page_tokens + (tok % p.page_tokens);
#pragma unroll
          for (int bx = 0; bx < C::kBoxes; ++bx) {
            prefetch_tile_2d_l2(&p.tmap_k, bx * 64, row);
            prefetch_tile_2d_l2(&p.tmap_v, bx * 64, row);
          }
        }
      }
    }
    griddep_wait();
    const uint64_t policy = policy_evict_first();
    uint32_t sidx = 0, k = 0;
    bool ok = true;
    for (long long sg = s_end; sg > s_beg && ok; ++k) {
      const Seg w = seg_ending(p, sg, s_beg);
      sg = w.s_begin;
      const SeqEntry se = p.seqs[w.si];
      const int layer = p.layer_begin + w.layer_local;
      const bool has_new = seg_has_new(p, w);
      if (lane == 0) {
        const int b = k & 1;
        if (k >= 2 && !mbar_wait(&qempty[b], ((k >> 1) - 1) & 1)) {
          set_error(p.error, 5);
          ok = false;
        }
        if (ok) {
          // the group's query rows and RoPE row; with a new token also its raw
          // k and v rows (and its own RoPE row when its position differs)
          const size_t qrow0 = (size_t)(w.layer_local * p.seq_total + p.seq_base + w.si) * H + w.kvh * G;
          const bool new_cs = has_new && p.rope && se.new_pos != se.q_pos;
          uint32_t bytes = (uint32_t)(G * HD * 4) + (p.rope ? (uint32_t)(2 * half * 4) : 0u);
          if (has_new) bytes += (uint32_t)(2 * HD * 4) + (new_cs ? (uint32_t)(2 * half * 4) : 0u);
          mbar_arrive_expect_tx(&qfull[b], bytes);
          float* qdst = reinterpret_cast<float*>(smem + C::kOffQ + b * C::kQBytes);
          for (int r = 0; r < G; ++r) bulk_load(qdst + r * C::kRowF, p.q + (qrow0 + r) * HD, HD * 4, &qfull[b]);
          if (p.rope) {
            float* cs = reinterpret_cast<float*>(smem + C::kOffCS + b * C::kCSBytes);
            bulk_load(cs, p.rope_cos + (size_t)se.q_pos * half, half * 4, &qfull[b]);
            bulk_load(cs + half, p.rope_sin + (size_t)se.q_pos * half, half * 4, &qfull[b]);
          }
          if (has_new) {
            float* nb = reinterpret_cast<float*>(smem + C::kOffNew + b * C::kNewBytes);
            const size_t src = ((size_t)(w.layer_local * p.seq_total + p.seq_base + w.si) * p.kv_heads + w.kvh) * HD;
            bulk_load(nb, p.k_new + src, HD * 4, &qfull[b]);
            bulk_load(nb + HD, p.v_new + src, HD * 4, &qfull[b]);
            if (new_cs) {
              bulk_load(nb + 2 * HD, p.rope_cos + (size_t)se.new_pos * half, half * 4, &qfull[b]);
              bulk_load(nb + 2 * HD + half, p.rope_sin + (size_t)se.new_pos * half, half * 4, &qfull[b]);
            }
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      // Page ids: computed for a sequence whose pages are consecutive in the
      // pool; otherwise table entries of this chunk, one per lane, read
      // together up front (the loop refreshes the batch every 32 pages).
      const int pg0 = w.t0 / p.page_tokens;
      int pg_batch = -1;
      int pg_reg = 0;
      for (int s = 0; s < w.n_st; ++s, ++sidx) {
        const int slot = sidx % R;
        const int tok = w.t0 + s * kStageTokens;
        const int rel = tok / p.page_tokens - pg0;
        if (se.page_base < 0 && (rel >> 5) != pg_batch) {
          pg_batch = rel >> 5;
          const int idx = pg0 + pg_batch * 32 + lane;
          pg_reg = idx < p.max_pages_per_seq ? p.page_table[se.slot * p.max_pages_per_seq + idx] : 0;
        }
        const int page = se.page_base >= 0 ? se.page_base + pg0 + rel : __shfl_sync(0xffffffffu, pg_reg, rel & 31);
        if (lane == 0) {
          if (sidx >= (uint32_t)R && !mbar_wait(&empty[slot], ((sidx / R) - 1) & 1)) {
            set_error(p.error, 1);
            ok = false;
          }
          if (ok) {
            const int row = ((layer * p.num_pages + page) * p.kv_heads + w.kvh) * p.page_tokens + (tok % p.page_tokens);
            unsigned char* st = smem + slot * C::kStageBytes;
            mbar_arrive_expect_tx(&full[slot], C::kStageBytes);
#pragma unroll
            for (int bx = 0; bx < C::kBoxes; ++bx) {
              tma_load_2d_hint(st + bx * kBoxBytes, &p.tmap_k, &full[slot], bx * 64, row, policy);
              tma_load_2d_hint(st + (C::kBoxes + bx) * kBoxBytes, &p.tmap_v, &full[slot], bx * 64, row, policy);
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
    }
    // Never leave the CTA with copies in flight: the last stages and q buffers have landed.
    if (lane == 0) {
      for (uint32_t j = sidx > (uint32_t)R ? sidx - R : 0; j < sidx; ++j) {
        if (!mbar_wait(&full[j % R], (j / R) & 1)) set_error(p.error, 2);
      }
      for (uint32_t j = k > 2u ? k - 2 : 0; j < k; ++j) {
        if (!mbar_wait(&qfull[j & 1], (j >> 1) & 1)) set_error(p.error, 6);
      }
    }
    return;
  }

  if (warp == kConsumerWarps + 1) {
    // ---- helper warp: query fragments ahead of the consumers; merges behind them ----
    const int g = lane >> 2, c = lane & 3;  // the fragment owner this lane prepares for
    uint32_t k = 0;
    bool ok = true;
    // query fragments for the CTA's segment number kk (all 32 lanes; warp-uniform
    // waits); layer_local / kvh locate the segment's query bias rows
    auto prepare = [&](uint32_t kk, int layer_local, int kvh) -> bool {
      const int b = kk & 1;
      const float* qbg = p.q_bias ? p.q_bias + ((size_t)(p.layer_begin + layer_local) * H + kvh * G) * HD : nullptr;
      if (!mbar_wait_warp(&qfull[b], (kk >> 1) & 1)) return false;
      if (kk >= 2 && !mbar_wait_warp(&fempty[b], ((kk >> 1) - 1) & 1)) return false;
      const float* sq = reinterpret_cast<const float*>(smem + C::kOffQ + b * C::kQBytes);
      const float* cs = reinterpret_cast<const float*>(smem + C::kOffCS + b * C::kCSBytes);
      uint4* frag = reinterpret_cast<uint4*>(smem + C::kOffFrag + b * C::kFragBytes);
#pragma unroll
      for (int j = 0; j < C::kChunksPerThread; ++j) {
        int box;
        const int ch = k_chunk_of<HD>(c, j, &box);
        const int d0 = box * 64 + ch * 8;                  // 8 consecutive dims, all on one side of half
        const int dp = d0 < half ? d0 + half : d0 - half;  // their rotation partners
        const int di = d0 < half ? d0 : d0 - half;         // cos/sin index
        float cv[8], sv[8];
        if (p.rope) {
          const float4 c0 = *reinterpret_cast<const float4*>(cs + di);
          const float4 c1 = *reinterpret_cast<const float4*>(cs + di + 4);
          const float4 s0 = *reinterpret_cast<const float4*>(cs + half + di);
          const float4 s1 = *reinterpret_cast<const float4*>(cs + half + di + 4);
          cv[0] = c0.x; cv[1] = c0.y; cv[2] = c0.z; cv[3] = c0.w; cv[4] = c1.x; cv[5] = c1.y; cv[6] = c1.z; cv[7] = c1.w;
          sv[0] = s0.x; sv[1] = s0.y; sv[2] = s0.z; sv[3] = s0.w; sv[4] = s1.x; sv[5] = s1.y; sv[6] = s1.z; sv[7] = s1.w;
        }
        float v[2][8];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int row = g + 8 * r;
          if (GP == 8 && r == 1) {
            // padding rows 8-15 carry the low parts of rows 0-7
#pragma unroll
            for (int e = 0; e < 8; ++e) v[1][e] = f16_residual(v[0][e]);
            continue;
          }
          if (row >= G || row >= GP) {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[r][e] = 0.f;
            continue;
          }
          const float* qr = sq + row * C::kRowF;
          const float4 x0 = *reinterpret_cast<const float4*>(qr + d0);
          const float4 x1 = *reinterpret_cast<const float4*>(qr + d0 + 4);
          float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
          if (qbg) add_bias8(x, qbg + row * HD + d0);
          if (p.rope) {
            const float4 y0 = *reinterpret_cast<const float4*>(qr + dp);
            const float4 y1 = *reinterpret_cast<const float4*>(qr + dp + 4);
            float y[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
            if (qbg) add_bias8(y, qbg + row * HD + dp);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              v[r][e] = d0 < half ? rope_lo(x[e], y[e], cv[e], sv[e]) : rope_hi(y[e], x[e], cv[e], sv[e]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[r][e] = x[e];
          }
        }
        // k-step 2j uses dims d0+0..3, k-step 2j+1 uses d0+4..7; stored as [k-step][lane] uint4
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint4 f;
          f.x = pack_half2(v[0][4 * h + 0], v[0][4 * h + 1]);
          f.y = pack_half2(v[1][4 * h + 0], v[1][4 * h + 1]);
          f.z = pack_half2(v[0][4 * h + 2], v[0][4 * h + 3]);
          f.w = pack_half2(v[1][4 * h + 2], v[1][4 * h + 3]);
          frag[(2 * j + h) * 32 + lane] = f;
          if (GP == 16) {
            // second fragment set: the low parts of all 16 rows
            uint4 fl;
            fl.x = pack_half2(f16_residual(v[0][4 * h + 0]), f16_residual(v[0][4 * h + 1]));
            fl.y = pack_half2(f16_residual(v[1][4 * h + 0]), f16_residual(v[1][4 * h + 1]));
            fl.z = pack_half2(f16_residual(v[0][4 * h + 2]), f16_residual(v[0][4 * h + 3]));
            fl.w = pack_half2(f16_residual(v[1][4 * h + 2]), f16_residual(v[1][4 * h + 3]));
            frag[C::kFragSet / 16 + (2 * j + h) * 32 + lane] = fl;
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&qempty[b]);  // raw rows consumed (with the appender's arrival the producer may refill)
        mbar_arrive(&fready[b]);
      }
      return true;
    };
    const int gidx_first = s_beg < s_end ? group_at(p, s_beg).gidx : 0;  // record j of this CTA: group gidx_first + j
    if (s_beg < s_end) {
      const Seg w0 = p.q_bias ? seg_ending(p, s_end, s_beg) : Seg{};
      ok = prepare(0, w0.layer_local, w0.kvh);
    }
    for (long long sg = s_end; sg > s_beg && ok; ++k) {
      const Seg w = seg_ending(p, sg, s_beg);
      sg = w.s_begin;
      if (sg > s_beg) {
        const Seg wn = p.q_bias ? seg_ending(p, sg, s_beg) : Seg{};
        if (!prepare(k + 1, wn.layer_local, wn.kvh)) {
          ok = false;
          break;
        }
      }
      if (sg == s_beg) break;  // the CTA's last segment: the consumer warps merge it
      // merge item k: the four consumer warps' (m, l, O) -> output or split-K record
      const int b = k & 1;
      // The group's parts and (lanes < kSlots) the record offsets of the first
      // combine batch, worked out (64-bit divisions) while the consumers stream.
      const size_t qrow0 = (size_t)(w.layer_local * p.seq_total + p.seq_base + w.si) * H + w.kvh * G;
      const int b_first = cta_of(p, w.gs0);
      const int parts = cta_of(p, w.gs1 - 1) - b_first + 1;
      const bool single = parts == 1;
      constexpr int kRecFloats = GP * REC;                       // one staged record
      constexpr int kSlots = C::kMergeBytes / (kRecFloats * 4);  // records staged per combine batch
      static_assert(kSlots >= 2 && kSlots <= 8, "combine staging");
      long long first_off = 0;
      if (!single && lane < min(kSlots, parts)) first_off = record_offset<HD>(p, b_first + lane, w.gidx);
      if (!mbar_wait_warp(&mready[b], (k >> 1) & 1)) {
        ok = false;
        break;
      }
      const float* sm_o = reinterpret_cast<const float*>(smem + C::kOffMerge + b * C::kMergeBytes);
      const float* sm_m = reinterpret_cast<const float*>(smem + C::kOffML) + b * C::kMLFloats;
      const float* sm_l = sm_m + kConsumerWarps * 16;
      float* part = p.partials + ((size_t)blockIdx.x * p.max_segs + (w.gidx - gidx_first)) * G * REC;
      constexpr int kLanesPerRow = HD / 4;        // float4 per lane
      constexpr int kRowStep = 32 / kLanesPerRow; // rows handled per pass
      constexpr int NR = GP / kRowStep;           // rows per lane
      const int d = 4 * (lane % kLanesPerRow);
      const int r0 = lane / kLanesPerRow;
      // Two phases keep the dependency chains short: lane r < G computes row
      // r's max, weights and sum; then every lane weights its 4-column slices
      // of all rows (weights by shuffle from the row's lane), loads first and
      // stores last.
      // A segment with the group's new token adds it as a fifth state
      // (m = its score, l = 1, O = its v row).
      const bool has_new = seg_has_new(p, w);
      if (has_new && !mbar_wait_warp(&nready[b], (k >> 1) & 1)) {
        ok = false;
        break;
      }
      const float* res = reinterpret_cast<const float*>(smem + C::kOffRes + b * C::kResBytes);
      float mw[kConsumerWarps] = {}, mn = 0.f, Mr = -INFINITY, Lr = 0.f;
      if (lane < G) {
#pragma unroll
        for (int ww = 0; ww < kConsumerWarps; ++ww) {
          mw[ww] = sm_m[ww * 16 + lane];
          Mr = fmaxf(Mr, mw[ww]);
        }
        if (has_new) {
          mn = res[lane];
          Mr = fmaxf(Mr, mn);
        }
#pragma unroll
        for (int ww = 0; ww < kConsumerWarps; ++ww) {
          mw[ww] = mw[ww] == -INFINITY ? 0.f : ex2(mw[ww] - Mr);
          Lr += sm_l[ww * 16 + lane] * mw[ww];
        }
        if (has_new) {
          mn = ex2(mn - Mr);
          Lr += mn;
        }
      }
      const float4 vn = has_new ? *reinterpret_cast<const float4*>(res + 16 + d) : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 O[NR];
#pragma unroll
      for (int u = 0; u < NR; ++u) {
        const int row = r0 + u * kRowStep;  // < GP <= 16: the shuffle source is a valid lane
        const float wn = __shfl_sync(0xffffffffu, mn, row);
        O[u] = make_float4(vn.x * wn, vn.y * wn, vn.z * wn, vn.w * wn);
#pragma unroll
        for (int ww = 0; ww < kConsumerWarps; ++ww) {
          const float wt = __shfl_sync(0xffffffffu, mw[ww], row);
          const float4 o = *reinterpret_cast<const float4*>(sm_o + ((size_t)ww * GP + row) * C::kRowF + d);
          O[u].x += o.x * wt;
          O[u].y += o.y * wt;
          O[u].z += o.z * wt;
          O[u].w += o.w * wt;
        }
      }
#pragma unroll
      for (int u = 0; u < NR; ++u) {
        const int row = r0 + u * kRowStep;
        const float M = __shfl_sync(0xffffffffu, Mr, row);
        const float L = __shfl_sync(0xffffffffu, Lr, row);
        if (row >= G) continue;
        if (single) {
          store_result<HD>(p, qrow0 + row, d, O[u], M, L);
        } else {
          float* r = part + (size_t)row * REC;
          *reinterpret_cast<float4*>(r + d) = O[u];
          if (d == 0) *reinterpret_cast<float2*>(r + HD) = make_float2(M, L);
        }
      }
      int finished = single ? 1 : 0;  // this warp stored the group's final rows
      if (!single) {
        // The last CTA of the group to finish folds all the parts' records, in
        // part order (so the result does not depend on which CTA came last).
        // Release: the warp's record stores (ordered by __syncwarp) before the
        // ticket; acquire: the ticket before the record loads.
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          fence_acq_rel_gpu();
          const uint32_t ticket = atomicAdd(&p.counters[w.gidx], 1u);
          last = ticket == (uint32_t)(parts - 1);
          if (last) {
            fence_acq_rel_gpu();
            p.counters[w.gidx] = 0u;  // every part has taken its ticket
          }
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          // Records are copied into the just-merged buffer b (still ours), all
          // copies of a batch in flight at once, then folded in part order by
          // fold_part, as the consumer warps' combine does.  CTA b_first + pp
          // holds part pp as its segment jp = gidx - (group of its first stage).
          float* stage = reinterpret_cast<float*>(smem + C::kOffMerge + b * C::kMergeBytes);
          const uint32_t stage_s = smem_u32(stage);
          float M[NR], L[NR];
          float4 O[NR];
#pragma unroll
          for (int u = 0; u < NR; ++u) {
            M[u] = -INFINITY;
            L[u] = 0.f;
            O[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
#pragma unroll 1
          for (int pp0 = 0; pp0 < parts; pp0 += kSlots) {
            const int nb = min(kSlots, parts - pp0);
            long long my_off = first_off;
            if (pp0 > 0 && lane < nb) my_off = record_offset<HD>(p, b_first + pp0 + lane, w.gidx);
            __syncwarp();  // the previous batch's reads of the staging slots are done
#pragma unroll 1
            for (int j = 0; j < nb; ++j) {
              const float* rec = p.partials + __shfl_sync(0xffffffffu, my_off, j);
              const uint32_t dst0 = stage_s + (uint32_t)(j * kRecFloats) * 4u;
#pragma unroll
              for (int u = 0; u < NR; ++u) {
                const int row = r0 + u * kRowStep;
                if (row >= G) continue;
                const uint32_t dst = dst0 + (uint32_t)(row * REC) * 4u;
                cp_async_cg16(dst + (uint32_t)d * 4u, rec + (size_t)row * REC + d);
                if (d == 0) cp_async_cg16(dst + HD * 4u, rec + (size_t)row * REC + HD);  // (m, l, pad, pad)
              }
            }
            cp_async_wait_all();
            __syncwarp();
#pragma unroll 1
            for (int j = 0; j < nb; ++j) {
#pragma unroll
              for (int u = 0; u < NR; ++u) {
                const int row = r0 + u * kRowStep;
                if (row >= G) continue;
                const float* r = stage + j * kRecFloats + row * REC;
                const float2 ml = *reinterpret_cast<const float2*>(r + HD);
                fold_part(M[u], L[u], O[u], ml.x, ml.y, *reinterpret_cast<const float4*>(r + d));
              }
            }
          }
#pragma unroll
          for (int u = 0; u < NR; ++u) {
            const int row = r0 + u * kRowStep;
            if (row < G) store_result<HD>(p, qrow0 + row, d, O[u], M[u], L[u]);
          }
          finished = 1;
        }
      }
      if (p.xch_world > 1 && finished) xch_group_finished(p, w.gidx, lane, [] { __syncwarp(); });
      __syncwarp();
      if (lane == 0) mbar_arrive(&mfree[b]);
    }
    if (!ok) set_error(p.error, 9);
    return;
  }

  if (warp == kConsumerWarps + 2) {
    // ---- appender warp: the new token of a segment that carries one --------
    // RoPE + f16 append to the cache (fire and forget: no K/V stage of this
    // launch reads it) and its scores q.k in log2 units for the helper's merge.
    // Every segment arrives on qempty and nready, so the phases stay in step
    // with the segment count; result buffer b is rewritten only after the
    // merge two segments back has released it (mfree).
    uint32_t k = 0;
    for (long long sg = s_end; sg > s_beg; ++k) {
      const Seg w = seg_ending(p, sg, s_beg);
      sg = w.s_begin;
      const int b = k & 1;
      if (!mbar_wait_warp(&qfull[b], (k >> 1) & 1) ||
          (k >= 2 && !mbar_wait_warp(&mfree[b], ((k >> 1) - 1) & 1))) {
        set_error(p.error, 11);
        break;
      }
      if (seg_has_new(p, w)) {
        const SeqEntry se = p.seqs[w.si];
        const float* sq = reinterpret_cast<const float*>(smem + C::kOffQ + b * C::kQBytes);
        const float* cs = reinterpret_cast<const float*>(smem + C::kOffCS + b * C::kCSBytes);
        float* nb = reinterpret_cast<float*>(smem + C::kOffNew + b * C::kNewBytes);  // raw k, v (, cos, sin)
        const float* csk = se.new_pos != se.q_pos ? nb + 2 * HD : cs;
        float* res = reinterpret_cast<float*>(smem + C::kOffRes + b * C::kResBytes);  // scores[16], v[HD]
        const int new_idx = se.len - 1;
        const int page = se.page_base >= 0 ? se.page_base + new_idx / p.page_tokens
                                           : p.page_table[se.slot * p.max_pages_per_seq + new_idx / p.page_tokens];
        const size_t row = ((size_t)((p.layer_begin + w.layer_local) * p.num_pages + page) * p.kv_heads + w.kvh) *
                               p.page_tokens + (new_idx % p.page_tokens);
        // projection biases of this layer (fp32 adds before RoPE and rounding)
        const size_t kvb = ((size_t)(p.layer_begin + w.layer_local) * p.kv_heads + w.kvh) * HD;
        const float* kb = p.k_bias ? p.k_bias + kvb : nullptr;
        const float* vb = p.v_bias ? p.v_bias + kvb : nullptr;
        const float* qbg = p.q_bias ? p.q_bias + ((size_t)(p.layer_begin + w.layer_local) * H + w.kvh * G) * HD : nullptr;
        for (int i = lane; i < half; i += 32) {
          float a = nb[i], bb = nb[i + half];
          if (kb) {
            a = __fadd_rn(a, kb[i]);
            bb = __fadd_rn(bb, kb[i + half]);
          }
          float lo = a, hi = bb;
          if (p.rope) {
            lo = rope_lo(a, bb, csk[i], csk[half + i]);
            hi = rope_hi(a, bb, csk[i], csk[half + i]);
          }
          const __half hl = __float2half_rn(lo), hh = __float2half_rn(hi);
          p.k_pool[row * HD + i] = __half_as_ushort(hl);
          p.k_pool[row * HD + i + half] = __half_as_ushort(hh);
          nb[i] = __half2float(hl);  // in place: k as the cache holds it (only this lane reads i, i + half)
          nb[i + half] = __half2float(hh);
        }
        for (int i = lane; i < HD; i += 32) {
          const __half hv = __float2half_rn(vb ? __fadd_rn(nb[HD + i], vb[i]) : nb[HD + i]);
          p.v_pool[row * HD + i] = __half_as_ushort(hv);
          res[16 + i] = __half2float(hv);
        }
        __syncwarp();
        for (int h = 0; h < G; ++h) {
          const float* qr = sq + h * C::kRowF;
          float dot = 0.f;
          for (int i = lane; i < half; i += 32) {
            float ql = qr[i], qh = qr[i + half];
            if (qbg) {
              ql = __fadd_rn(ql, qbg[h * HD + i]);
              qh = __fadd_rn(qh, qbg[h * HD + i + half]);
            }
            if (p.rope) {
              const float x = ql, y = qh;
              ql = rope_lo(x, y, cs[i], cs[half + i]);
              qh = rope_hi(x, y, cs[i], cs[half + i]);
            }
            dot = fmaf(ql, nb[i], fmaf(qh, nb[i + half], dot));
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
          if (lane == 0) res[h] = dot * p.scale_log2;
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&qempty[b]);
        mbar_arrive(&nready[b]);
      }
    }
    return;
  }

  // ---- consumer warps 0-3 ------------------------------------------------
  volatile uint32_t* cflag = reinterpret_cast<volatile uint32_t*>(smem + C::kOffFlag);
  const int g = lane >> 2;  // mma group id: head rows g and g+8, token rows
  const int c = lane & 3;   // thread in group
  const float sl = p.scale_log2;
  uint32_t sidx = 0, k = 0;
  bool failed = false;
  for (long long sg = s_end; sg > s_beg; ++k) {
    const Seg w = seg_ending(p, sg, s_beg);
    sg = w.s_begin;

    // 1) query fragments prepared by the helper warp
    const int fb = k & 1;
    if (!failed && !mbar_wait_warp(&fready[fb], (k >> 1) & 1)) {
      set_error(p.error, 7);
      failed = true;
    }
    uint32_t qa[C::kKSteps][4];
    {
      const uint4* frag = reinterpret_cast<const uint4*>(smem + C::kOffFrag + fb * C::kFragBytes);
#pragma unroll
      for (int ks = 0; ks < C::kKSteps; ++ks) {
        const uint4 f = frag[ks * 32 + lane];
        qa[ks][0] = f.x;
        qa[ks][1] = f.y;
        qa[ks][2] = f.z;
        qa[ks][3] = f.w;
      }
    }
    // GP = 16 reads the low-part fragments from shared memory at every stage,
    // so it releases the buffer only after the segment's last stage.
    const uint32_t frag_lo = smem_u32(smem + C::kOffFrag + fb * C::kFragBytes + C::kFragSet);
    __syncwarp();
    if (GP == 8 && lane == 0) mbar_arrive(&fempty[fb]);

    // 2) stream the chunk's stages
    float acc[C::kNTiles][4];
#pragma unroll
    for (int i = 0; i < C::kNTiles; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
    for (int s = 0; s < w.n_st; ++s, ++sidx) {
      const int slot = sidx % R;
      if (!failed && !mbar_wait_warp(&full[slot], (sidx / R) & 1)) {
        set_error(p.error, 3);
        failed = true;
      }
      const int tok_base = w.t0 + s * kStageTokens + 16 * warp;
      if (!failed && tok_base < w.t1) {
        const uint32_t st = smem_u32(smem + slot * C::kStageBytes);
        float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int j = 0; j < C::kChunksPerThread; ++j) {
          int box;
          const int ch = k_chunk_of<HD>(c, j, &box);
          uint4 l0, l1;
          if (GP == 16) {
            l0 = lds128(frag_lo + (uint32_t)((2 * j) * 32 + lane) * 16u);
            l1 = lds128(frag_lo + (uint32_t)((2 * j + 1) * 32 + lane) * 16u);
          }
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int r = 16 * warp + g + 8 * t;
            const uint4 kv = lds128(st + box * kBoxBytes + r * 128 + ((ch ^ (r & 7)) << 4));
            mma_16816(sacc[t], qa[2 * j], kv.x, kv.y);
            mma_16816(sacc[t], qa[2 * j + 1], kv.z, kv.w);
            if (GP == 16) {
              const uint32_t a0[4] = {l0.x, l0.y, l0.z, l0.w};
              const uint32_t a1[4] = {l1.x, l1.y, l1.z, l1.w};
              mma_16816(sacc[t], a0, kv.x, kv.y);
              mma_16816(sacc[t], a1, kv.z, kv.w);
            }
          }
        }
        if (GP == 8) {
          // rows g + 8 hold q_lo . k of row g: the score is the sum
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            sacc[t][0] += sacc[t][2];
            sacc[t][1] += sacc[t][3];
          }
        }
        // rows g + 8 are query heads only with GP = 16
        constexpr int kE = GP == 16 ? 4 : 2;
        float sc[2][4];
        float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
#pragma unroll
          for (int e = 0; e < kE; ++e) {
            const int tok = tok_base + 8 * t + 2 * c + (e & 1);
            const float v = tok < w.t1 ? sacc[t][e] * sl : -INFINITY;
            sc[t][e] = v;
            if (e < 2) mx_lo = fmaxf(mx_lo, v); else mx_hi = fmaxf(mx_hi, v);
          }
        }
        mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
        mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
        const float nm_lo = fmaxf(m_lo, mx_lo);
        const float base_lo = nm_lo == -INFINITY ? 0.f : nm_lo;
        const float al_lo = ex2(m_lo - base_lo);
        m_lo = nm_lo;
        float al_hi = 1.f, base_hi = 0.f;
        if (GP == 16) {
          mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
          mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
          const float nm_hi = fmaxf(m_hi, mx_hi);
          base_hi = nm_hi == -INFINITY ? 0.f : nm_hi;
          al_hi = ex2(m_hi - base_hi);
          m_hi = nm_hi;
        }
        float ps_lo = 0.f, ps_hi = 0.f;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
#pragma unroll
          for (int e = 0; e < kE; ++e) {
            const float pv = ex2(sc[t][e] - (e < 2 ? base_lo : base_hi));
            sc[t][e] = pv;
            if (e < 2) ps_lo += pv; else ps_hi += pv;
          }
        }
        l_lo = l_lo * al_lo + ps_lo;
        if (GP == 16) l_hi = l_hi * al_hi + ps_hi;
        if (__any_sync(0xffffffffu, al_lo != 1.f || al_hi != 1.f)) {
#pragma unroll
          for (int i = 0; i < C::kNTiles; ++i) {
            acc[i][0] *= al_lo;
            acc[i][1] *= al_lo;
            acc[i][2] *= al_hi;
            acc[i][3] *= al_hi;
          }
        }
        uint32_t pa[4];
        pa[0] = pack_half2(sc[0][0], sc[0][1]);
        pa[1] = GP == 16 ? pack_half2(sc[0][2], sc[0][3]) : 0u;
        pa[2] = pack_half2(sc[1][0], sc[1][1]);
        pa[3] = GP == 16 ? pack_half2(sc[1][2], sc[1][3]) : 0u;
        const int rv0 = 16 * warp + 2 * c;
#pragma unroll
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          const uint32_t vb = st + (C::kBoxes + bx) * kBoxBytes;
          const uint4 v0 = lds128(vb + (rv0 + 0) * 128 + ((g ^ ((rv0 + 0) & 7)) << 4));
          const uint4 v1 = lds128(vb + (rv0 + 1) * 128 + ((g ^ ((rv0 + 1) & 7)) << 4));
          const uint4 v8 = lds128(vb + (rv0 + 8) * 128 + ((g ^ ((rv0 + 8) & 7)) << 4));
          const uint4 v9 = lds128(vb + (rv0 + 9) * 128 + ((g ^ ((rv0 + 9) & 7)) << 4));
          const uint32_t w0[4] = {v0.x, v0.y, v0.z, v0.w};
          const uint32_t w1[4] = {v1.x, v1.y, v1.z, v1.w};
          const uint32_t w8[4] = {v8.x, v8.y, v8.z, v8.w};
          const uint32_t w9[4] = {v9.x, v9.y, v9.z, v9.w};
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const uint32_t sel = (jj & 1) ? 0x7632u : 0x5410u;
            const uint32_t b0 = prmt(w0[jj >> 1], w1[jj >> 1], sel);
            const uint32_t b1 = prmt(w8[jj >> 1], w9[jj >> 1], sel);
            mma_16816(acc[bx * 8 + jj], pa, b0, b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (GP == 16 && lane == 0) mbar_arrive(&fempty[fb]);  // the low-part fragments are no longer read
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);

    // 3) park this warp's state for the merge
    const int mb = k & 1;
    if (k >= 2 && !failed && !mbar_wait_warp(&mfree[mb], ((k >> 1) - 1) & 1)) {
      set_error(p.error, 8);
      failed = true;
    }
    float* sm_o = reinterpret_cast<float*>(smem + C::kOffMerge + mb * C::kMergeBytes);  // [4][GP][kRowF]
    float* sm_m = reinterpret_cast<float*>(smem + C::kOffML) + mb * C::kMLFloats;       // [4][16]
    float* sm_l = sm_m + kConsumerWarps * 16;                                          // [4][16]
    if (c == 0) {
      sm_m[warp * 16 + g] = m_lo;
      sm_m[warp * 16 + g + 8] = m_hi;
      sm_l[warp * 16 + g] = l_lo;
      sm_l[warp * 16 + g + 8] = l_hi;
    }
#pragma unroll
    for (int i = 0; i < C::kNTiles; ++i) {
      const int bx = i >> 3, jj = i & 7;
      const int d0 = 64 * bx + 8 * (2 * c) + jj;
      const int d1 = 64 * bx + 8 * (2 * c + 1) + jj;
      float* o_lo = sm_o + ((size_t)warp * GP + g) * C::kRowF;
      o_lo[d0] = acc[i][0];
      o_lo[d1] = acc[i][1];
      if (GP > 8) {
        float* o_hi = sm_o + ((size_t)warp * GP + g + 8) * C::kRowF;
        o_hi[d0] = acc[i][2];
        o_hi[d1] = acc[i][3];
      }
    }
    __syncwarp();
    if (sg > s_beg) {
      // more segments follow: the helper merges this one while the stages of the next stream
      if (lane == 0) mbar_arrive(&mready[mb]);
      continue;
    }
    // 4) the CTA's last segment is merged by the four consumer warps together
    // (nothing else is left to overlap with): thread t owns row t / kTPR and
    // the float4 columns 4 * (t % kTPR + f * kTPR).
    constexpr int kTPR = 128 / GP;        // threads per row
    constexpr int kF = HD / (4 * kTPR);   // float4 columns per thread
    const int t = tid;                    // 0..127
    const int row = t / kTPR;
    const int cl = t % kTPR;
    consumer_bar_sync();
    const bool has_new = seg_has_new(p, w);
    if (has_new && !failed && !mbar_wait_warp(&nready[mb], (k >> 1) & 1)) {
      set_error(p.error, 12);
      failed = true;
    }
    const float* res = reinterpret_cast<const float*>(smem + C::kOffRes + mb * C::kResBytes);
    float M = -INFINITY, L = 0.f, wt[kConsumerWarps], wn = 0.f;
#pragma unroll
    for (int ww = 0; ww < kConsumerWarps; ++ww) {
      wt[ww] = sm_m[ww * 16 + row];
      M = fmaxf(M, wt[ww]);
    }
    if (has_new) {
      wn = res[row];
      M = fmaxf(M, wn);
    }
#pragma unroll
    for (int ww = 0; ww < kConsumerWarps; ++ww) {
      wt[ww] = wt[ww] == -INFINITY ? 0.f : ex2(wt[ww] - M);
      L += sm_l[ww * 16 + row] * wt[ww];
    }
    if (has_new) {
      wn = ex2(wn - M);
      L += wn;
    }
    float4 O[kF];
#pragma unroll
    for (int f = 0; f < kF; ++f) {
      const int d = 4 * (cl + f * kTPR);
      const float4 vn = has_new ? *reinterpret_cast<const float4*>(res + 16 + d) : make_float4(0.f, 0.f, 0.f, 0.f);
      O[f] = make_float4(vn.x * wn, vn.y * wn, vn.z * wn, vn.w * wn);
#pragma unroll
      for (int ww = 0; ww < kConsumerWarps; ++ww) {
        const float4 o = *reinterpret_cast<const float4*>(sm_o + ((size_t)ww * GP + row) * C::kRowF + d);
        O[f].x += o.x * wt[ww];
        O[f].y += o.y * wt[ww];
        O[f].z += o.z * wt[ww];
        O[f].w += o.w * wt[ww];
      }
    }
    const size_t qrow0 = (size_t)(w.layer_local * p.seq_total + p.seq_base + w.si) * H + w.kvh * G;
    constexpr int REC = kScratchRec<HD>;
    if (p.cluster_k > 1) {
      // Cluster mode: every part writes its record {acc[hd], m, l} into slot
      // (its rank) of rank 0's unused second merge buffer (one segment per
      // CTA) and arrives on rank 0's cbar (release, cluster scope); rank 0
      // folds the slots in rank order.
      const uint32_t rank = cluster_ctarank();
      float* slots = reinterpret_cast<float*>(smem + C::kOffMerge + (mb ^ 1) * C::kMergeBytes);
      static_assert(C::kMergeBytes >= 4 * GP * REC * 4, "four cluster slots per merge buffer");
      const uint32_t slot0 = mapa_shared(smem_u32(slots + (size_t)rank * GP * REC), 0);
      if (row < G) {
#pragma unroll
        for (int f = 0; f < kF; ++f) st_cluster_v4(slot0 + (uint32_t)(row * REC + 4 * (cl + f * kTPR)) * 4u, O[f]);
        if (cl == 0) st_cluster_v2(slot0 + (uint32_t)(row * REC + HD) * 4u, make_float2(M, L));
      }
      consumer_bar_sync();
      if (t == 0) mbar_arrive_cluster(mapa_shared(smem_u32(cbar), 0));
      if (rank != 0) continue;
      if (!mbar_wait_cluster(cbar, 0)) {
        if (t == 0) set_error(p.error, 13);
        continue;
      }
      float M2 = -INFINITY, L2 = 0.f;
      float4 O2[kF];
#pragma unroll
      for (int f = 0; f < kF; ++f) O2[f] = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int j = 0; j < p.cluster_k; ++j) {
        const float* r = slots + (size_t)j * GP * REC + (size_t)row * REC;
        const float2 ml = *reinterpret_cast<const float2*>(r + HD);
#pragma unroll
        for (int f = 0; f < kF; ++f) {
          float Mf = M2, Lf = L2;
          fold_part(Mf, Lf, O2[f], ml.x, ml.y, *reinterpret_cast<const float4*>(r + 4 * (cl + f * kTPR)));
          if (f == kF - 1) {
            M2 = Mf;
            L2 = Lf;
          }
        }
      }
      if (row < G) {
#pragma unroll
        for (int f = 0; f < kF; ++f) store_result<HD>(p, qrow0 + row, 4 * (cl + f * kTPR), O2[f], M2, L2);
      }
      if (p.xch_world > 1) xch_group_finished(p, w.gidx, t, [] { consumer_bar_sync(); });
      continue;
    }
    const int b_first = cta_of(p, w.gs0);
    const int parts = cta_of(p, w.gs1 - 1) - b_first + 1;
    if (parts == 1) {
      if (row < G) {
#pragma unroll
        for (int f = 0; f < kF; ++f) store_result<HD>(p, qrow0 + row, 4 * (cl + f * kTPR), O[f], M, L);
      }
      if (p.xch_world > 1) xch_group_finished(p, w.gidx, t, [] { consumer_bar_sync(); });
      continue;
    }
    // Split group: publish this part's record, take a ticket; the last part
    // folds all records in part order (the result does not depend on which
    // CTA came last).  Release: the 128 threads' record stores (ordered by
    // the barrier) before the ticket; acquire: the ticket before the loads.
    const int gidx_first = group_at(p, s_beg).gidx;
    float* part = p.partials + ((size_t)blockIdx.x * p.max_segs + (w.gidx - gidx_first)) * G * REC;
    if (row < G) {
#pragma unroll
      for (int f = 0; f < kF; ++f) *reinterpret_cast<float4*>(part + (size_t)row * REC + 4 * (cl + f * kTPR)) = O[f];
      if (cl == 0) *reinterpret_cast<float2*>(part + (size_t)row * REC + HD) = make_float2(M, L);
    }
    // record offsets of all parts, one thread each, in the merge buffer (its
    // reads above are complete once every thread has passed the barrier)
    long long* off = reinterpret_cast<long long*>(sm_o);
    static_assert(C::kMergeBytes >= 1024 * (int)sizeof(long long), "offsets of up to 1024 parts");
    consumer_bar_sync();
    uint32_t* flag = reinterpret_cast<uint32_t*>(sm_m);
    if (t == 0) {
      fence_acq_rel_gpu();
      const uint32_t ticket = atomicAdd(&p.counters[w.gidx], 1u);
      const uint32_t last = ticket == (uint32_t)(parts - 1);
      if (last) {
        fence_acq_rel_gpu();
        p.counters[w.gidx] = 0u;  // every part has taken its ticket
      }
      *flag = last;
    }
    for (int pp = t; pp < parts && pp < 1024; pp += 128) off[pp] = record_offset<HD>(p, b_first + pp, w.gidx);
    consumer_bar_sync();
    if (*flag == 0u) continue;
    if (parts > 1024) {
      set_error(p.error, 10);  // the grid is at most one CTA per SM
      continue;
    }
    const int own = (int)blockIdx.x - b_first;  // this CTA's part: its state is still in registers
    float M2 = -INFINITY, L2 = 0.f;
    float4 O2[kF];
#pragma unroll
    for (int f = 0; f < kF; ++f) O2[f] = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int kB = 4;  // parts' loads in flight per round trip
    for (int pp0 = 0; pp0 < parts; pp0 += kB) {
      float2 ml[kB];
      float4 o[kB][kF];
#pragma unroll
      for (int j = 0; j < kB; ++j) {
        const int pp = pp0 + j;
        if (pp < parts && pp != own && row < G) {
          const float* rec = p.partials + off[pp] + (size_t)row * REC;
          ml[j] = __ldcg(reinterpret_cast<const float2*>(rec + HD));
#pragma unroll
          for (int f = 0; f < kF; ++f) o[j][f] = __ldcg(reinterpret_cast<const float4*>(rec + 4 * (cl + f * kTPR)));
        } else if (pp == own) {
          ml[j] = make_float2(M, L);
#pragma unroll
          for (int f = 0; f < kF; ++f) o[j][f] = O[f];
        } else {
          ml[j] = make_float2(-INFINITY, 0.f);
#pragma unroll
          for (int f = 0; f < kF; ++f) o[j][f] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int j = 0; j < kB; ++j) {
#pragma unroll
        for (int f = 0; f < kF; ++f) {
          // every column slice folds the same (m, l); only the f == kF - 1 fold keeps its (M, L)
          float Mf = M2, Lf = L2;
          fold_part(Mf, Lf, O2[f], ml[j].x, ml[j].y, o[j][f]);
          if (f == kF - 1) {
            M2 = Mf;
            L2 = Lf;
          }
        }
      }
    }
    if (row < G) {
#pragma unroll
      for (int f = 0; f < kF; ++f) store_result<HD>(p, qrow0 + row, 4 * (cl + f * kTPR), O2[f], M2, L2);
    }
    if (p.xch_world > 1) xch_group_finished(p, w.gidx, t, [] { consumer_bar_sync(); });
  }
  if (p.xch_world > 1) {
    consumer_bar_sync();
    xch_finish<HD>(p, tid, cflag);
  }
}

// ---------------------------------------------------------------------------
// Generic fp32 decode used by the drop-in te_attention_decode_f32: any
// head_dim, any group size, fp32 K/V in the reference's token-major layout.
// Mirrors the reference's three passes (scores, softmax, weighted V sum) and
// its per-dot accumulation order; only expf and the sum's order differ.
__global__ void decode_f32_generic_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                          const float* __restrict__ v, float* __restrict__ scores,
                                          float* __restrict__ out, int n, int kv_heads, int head_dim, int group,
                                          float scale) {
  const int h = blockIdx.x;
  const int kvh = h / group;
  const float* qh = q + (size_t)h * head_dim;
  float* sc = scores + (size_t)h * n;
  __shared__ float red[32];
  __shared__ float bcast;
  float mx = -FLT_MAX;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float* kt = k + ((size_t)t * kv_heads + kvh) * head_dim;
    float dot = 0.f;
    for (int d = 0; d < head_dim; ++d) dot = __fadd_rn(dot, __fmul_rn(qh[d], kt[d]));
    const float s = __fmul_rn(dot, scale);
    sc[t] = s;
    mx = fmaxf(mx, s);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -FLT_MAX;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
    bcast = m;
  }
  __syncthreads();
  mx = bcast;
  float sum = 0.f;
  for (int t = threadIdx.x; t < n; t += blockDim.x) {
    const float e = expf(sc[t] - mx);
    sc[t] = e;
    sum += e;
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
    bcast = s;
  }
  __syncthreads();
  const float total = bcast;
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float acc = 0.f;
    for (int t = 0; t < n; ++t) {
      const float pt = total > 0.f ? __fdiv_rn(sc[t], total) : sc[t];
      acc = __fadd_rn(acc, __fmul_rn(pt, v[((size_t)t * kv_heads + kvh) * head_dim + d]));
    }
    out[(size_t)h * head_dim + d] = acc;
  }
}

// Log-sum-exp merge of partial records [n_parts][rows][hd + 2].
__global__ void merge_partials_kernel(const float* __restrict__ partials, int n_parts, int rows, int head_dim,
                                      float* __restrict__ out, int partial_out) {
  const int row = blockIdx.x;
  const int rec = head_dim + 2;
  __shared__ float sM, sL;
  if (threadIdx.x == 0) {
    float M = -INFINITY;
    for (int k = 0; k < n_parts; ++k) {
      const float* r = partials + ((size_t)k * rows + row) * rec;
      if (r[head_dim + 1] > 0.f) M = fmaxf(M, r[head_dim]);
    }
    float L = 0.f;
    for (int k = 0; k < n_parts; ++k) {
      const float* r = partials + ((size_t)k * rows + row) * rec;
      if (r[head_dim + 1] > 0.f) L += r[head_dim + 1] * ex2(r[head_dim] - M);
    }
    sM = M;
    sL = L;
  }
  __syncthreads();
  const float M = sM, L = sL;
  for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
    float O = 0.f;
    for (int k = 0; k < n_parts; ++k) {
      const float* r = partials + ((size_t)k * rows + row) * rec;
      if (r[head_dim + 1] > 0.f) O += r[d] * ex2(r[head_dim] - M);
    }
    if (partial_out) {
      float* r = out + (size_t)row * rec;
      r[d] = O;
      if (d == 0) { r[head_dim] = M; r[head_dim + 1] = L; }
    } else {
      out[(size_t)row * head_dim + d] = L > 0.f ? O / L : 0.f;
    }
  }
}

template <int HD, int GP>
cudaError_t launch_decode_impl(const DecodeParams& p, cudaStream_t s) {
  using C = DecodeCfg<HD, GP>;
  static std::atomic<uint64_t> configured{0};  // one bit per device
  const cudaError_t e = set_smem_limit_once(configured, (const void*)decode_f16_kernel<HD, GP>, C::kSmemBytes);
  if (e != cudaSuccess) return e;
  // Programmatic dependent launch: the CTAs may become resident (on SMs the
  // previous kernel has left) and set up their barriers before it completes;
  // they wait for it (griddepcontrol.wait) before touching global memory.
  // In cluster mode the k CTAs of a group form one thread-block cluster.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.cluster_k > 1 ? (unsigned)p.cluster_k : 1u;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, decode_f16_kernel<HD, GP>, p);
}

}  // namespace

cudaError_t launch_decode_f16(const DecodeParams& p, int head_dim, cudaStream_t s) {
  if (head_dim == 128) return p.group <= 8 ? launch_decode_impl<128, 8>(p, s) : launch_decode_impl<128, 16>(p, s);
  if (head_dim == 64) return p.group <= 8 ? launch_decode_impl<64, 8>(p, s) : launch_decode_impl<64, 16>(p, s);
  return cudaErrorInvalidValue;
}

cudaError_t launch_decode_f32_generic(const float* q, const float* k, const float* v, float* scores, float* out,
                                      size_t n_tokens, int heads, int kv_heads, int head_dim, cudaStream_t s) {
  const float scale = 1.0f / sqrtf((float)head_dim);
  decode_f32_generic_kernel<<<heads, 256, 0, s>>>(q, k, v, scores, out, (int)n_tokens, kv_heads, head_dim,
                                                   heads / kv_heads, scale);
  return cudaGetLastError();
}

// Copies up to three buffers of host-visible (pinned, device-mapped) memory
// into device staging with plain 16-byte loads over PCIe: one launch in place
// of one copy operation per buffer.  The next kernel on the stream (a
// programmatic dependent) may be scheduled as soon as every CTA has started.
__global__ void __launch_bounds__(256) gather_host_kernel(const __grid_constant__ GatherParams p) {
  griddep_launch_dependents();
  size_t total = 0;
  for (int i = 0; i < p.n; ++i) total += p.chunks[i];
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    size_t k = e;
    int i = 0;
    while (k >= p.chunks[i]) k -= p.chunks[i++];
    reinterpret_cast<uint4*>(p.dst[i])[k] = reinterpret_cast<const uint4*>(p.src[i])[k];
  }
}

cudaError_t launch_gather_host(const GatherParams& p, cudaStream_t s) {
  size_t total = 0;
  for (int i = 0; i < p.n; ++i) total += p.chunks[i];
  const int grid = (int)std::min<size_t>((total + 255) / 256, 148);
  if (grid == 0) return cudaSuccess;
  gather_host_kernel<<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_merge_partials(const float* partials, int n_parts, int rows, int head_dim, float* out,
                                  int partial_out, cudaStream_t s) {
  merge_partials_kernel<<<rows, 128, 0, s>>>(partials, n_parts, rows, head_dim, out, partial_out);
  return cudaGetLastError();
}

}  // namespace te

// ===========================================================================
// Allocation-free decode entry point.
//
// Callers that cannot allocate device memory -- code running where
// cudaMalloc is not permitted or not wanted (inside a host callback or a
// stream-ordered region that must not synchronise, a runtime with its own
// fixed memory plan, a plugin whose host framework owns every allocation) --
// cannot create an engine, whose decode scratch grows with cudaMalloc.  This
// entry point runs the same decode kernel with its split-K scratch (partial
// records, completion counters, error word) in one fixed file-scope device
// array instead.  Every GPU that loads this library holds that array until
// the process exits.
// ===========================================================================

namespace {

constexpr size_t kNoAllocPartialBytes = size_t(4) << 20;  // split-K partial records (4 MiB)
constexpr size_t kNoAllocCounterBytes = 1024;             // 256 completion counters
constexpr size_t kNoAllocScratchBytes = kNoAllocPartialBytes + kNoAllocCounterBytes + 256;  // + error word
constexpr int kNoAllocMaxKvHeads = 256;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch per device, resolved once per device
// with that device current.  In host code the symbol itself is only a
// host-side stand-in, never a device address.
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kNoAllocMaxDevices] = {};

}  // namespace

extern "C" __attribute__((visibility("default"))) te_status te_attention_decode_paged_noalloc(
    const uint16_t* k_pool, const uint16_t* v_pool, const int32_t* page_table, size_t num_pages,
    size_t page_tokens, size_t n_tokens, const float* q, size_t heads, size_t kv_heads, size_t head_dim,
    float* out, void* stream) {
  using namespace te;
  if (!k_pool || !v_pool || !page_table || !q || !out || num_pages == 0 || n_tokens == 0 || heads == 0 ||
      kv_heads == 0 || heads % kv_heads != 0 || page_tokens == 0 || page_tokens % kStageTokens != 0) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  if (head_dim != 64 && head_dim != 128) return TE_STATUS_UNSUPPORTED;
  const size_t G = heads / kv_heads;
  if (G > 16 || kv_heads > (size_t)kNoAllocMaxKvHeads) return TE_STATUS_UNSUPPORTED;
  const size_t pages_needed = (n_tokens + page_tokens - 1) / page_tokens;
  const uint64_t rows = (uint64_t)num_pages * kv_heads * page_tokens;
  if (pages_needed > num_pages || rows >= (1ull << 31) || n_tokens > (size_t)INT32_MAX) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return TE_STATUS_RUNTIME_ERROR;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);

  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
        return TE_STATUS_RUNTIME_ERROR;
      }
      g_noalloc_addr[dev] = p;
    }
    base = g_noalloc_addr[dev];
  }
  unsigned char* scratch = static_cast<unsigned char*>(base);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Counters and the error word must start at zero; partial records need no clearing.
  if (cudaMemsetAsync(scratch + kNoAllocPartialBytes, 0, kNoAllocCounterBytes + 256, s) != cudaSuccess) {
    return TE_STATUS_RUNTIME_ERROR;
  }

  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  if (!encode_tmap_f16(&p.tmap_k, k_pool, rows, head_dim, kStageTokens) ||
      !encode_tmap_f16(&p.tmap_v, v_pool, rows, head_dim, kStageTokens)) {
    return TE_STATUS_RUNTIME_ERROR;
  }
  p.page_table = page_table;
  p.q = q;
  p.out = out;
  p.partials = reinterpret_cast<float*>(scratch);
  p.counters = reinterpret_cast<uint32_t*>(scratch + kNoAllocPartialBytes);
  p.error = reinterpret_cast<int*>(scratch + kNoAllocPartialBytes + kNoAllocCounterBytes);
  p.n_seqs = 1;
  p.seq_total = 1;
  p.layer_begin = 0;
  p.n_layers = 1;
  p.kv_heads = (int32_t)kv_heads;
  p.group = (int32_t)G;
  p.num_pages = (int32_t)num_pages;
  p.page_tokens = (int32_t)page_tokens;
  p.max_pages_per_seq = (int32_t)pages_needed;
  p.rope = 0;
  p.partial_out = 0;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)head_dim));
  p.seqs[0].slot = 0;
  p.seqs[0].len = (int32_t)n_tokens;
  p.seqs[0].q_pos = 0;
  p.seqs[0].new_pos = -1;
  p.seqs[0].page_base = -1;  // the caller's table is read
  // Stream-K split whose partial records fit the fixed scratch.
  const size_t rec_bytes = G * decode_scratch_rec((int)head_dim) * sizeof(float);
  long long max_grid = sms;
  plan_stream_k(p, max_grid);
  while ((size_t)p.grid * p.max_segs * rec_bytes > kNoAllocPartialBytes && max_grid > 1) {
    max_grid /= 2;
    plan_stream_k(p, max_grid);
  }
  // Defensive: with kv_heads <= 256 and groups <= 16 a one-CTA grid needs at
  // most 256 * 16 * 132 * 4 bytes (2.16 MB), so every accepted shape fits.
  if ((size_t)p.grid * p.max_segs * rec_bytes > kNoAllocPartialBytes) return TE_STATUS_UNSUPPORTED;
  return launch_decode_f16(p, (int)head_dim, s) == cudaSuccess ? TE_STATUS_OK : TE_STATUS_RUNTIME_ERROR;
}

extern "C" __attribute__((visibility("default"))) te_status te_attention_decode_paged_noalloc_status(void* stream,
                                                                                                      int* code) {
  if (!code) return TE_STATUS_INVALID_ARGUMENT;
  *code = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return TE_STATUS_RUNTIME_ERROR;
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    base = g_noalloc_addr[dev];
  }
  if (!base) return TE_STATUS_OK;  // no call on this device yet
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return TE_STATUS_RUNTIME_ERROR;
  int* word = reinterpret_cast<int*>(static_cast<unsigned char*>(base) + kNoAllocPartialBytes + kNoAllocCounterBytes);
  if (cudaMemcpy(code, word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return TE_STATUS_RUNTIME_ERROR;
  if (*code == 0) return TE_STATUS_OK;
  cudaMemset(word, 0, sizeof(int));
  return TE_STATUS_RUNTIME_ERROR;
}
