// Whole-token qwen2 decode step in one cooperative launch.
//
// Reference semantics: te_qwen_forward_token (c/src/qwen.c:907-1112) runs,
// per layer, RMSNorm -> q/k/v projections + biases -> RoPE -> KV append ->
// GQA attention -> output projection + residual -> RMSNorm -> gate/up ->
// SwiGLU -> down projection + residual; te_qwen_project_next (:1303-1377)
// then applies the output RMSNorm, the lm_head and the argmax.  The per-op
// path of this library runs that as five launches per layer; here one
// persistent grid (one CTA per SM) runs all of it, with a grid-wide
// arrival count between dependent phases instead of kernel boundaries.
//
// Weights do not depend on activations, so they are streamed without regard
// to phases: CTA b owns a fixed row slice of every projection, its share of
// all weights is packed host-side into one contiguous byte stream in the
// order it consumes them (stages of whole rows, 16-byte aligned), and a
// producer warp copies that stream through a ring of shared-memory slots
// (cp.async.bulk, completion on the slot's mbarrier) as fast as the slots
// free up.  While the eight consumer warps wait at a phase boundary, the
// producer keeps fetching the next phases' (and layers') rows, so a phase
// starts with its weights already on chip.
//
// Phases per layer (every CTA; a CTA with no rows or items only arrives):
//   A  q|k|v = W_qkv RMSNorm(x)       rows of the stacked q, k, v matrices
//   B  attention                       work items (kv head, 256-token chunk):
//                                      bias + RoPE of the group's queries, the
//                                      new k/v (bias, RoPE on k, f16 RNE) into
//                                      the paged cache, scores, softmax, P.V;
//                                      chunks of one kv head merge by
//                                      log-sum-exp in the last arriving CTA
//   C  x = x + W_o attn
//   D  g|u = W_gu RMSNorm(x)
//   E  x = x + W_down SwiGLU(g, u)
// then, optionally, logits = W_head RMSNorm(x) and the first-maximum argmax
// (per-CTA candidates, reduced by the last arriving CTA).
//
// Dot products use the same exact weight decoding as the matrix-vector
// kernel (codes under the exponent of 2^23) and fp32 sums in another order
// than the reference's, so results agree to fp32 rounding.  Every wait is
// bounded (2 s of %globaltimer); an expired wait sets the error word and the
// whole grid leaves (every consumer barrier reduces a failure flag).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <climits>

#include "te_internal.h"
#include "te_ptx.cuh"
#include "te_rope.cuh"

namespace te {
namespace {

constexpr int kCWarps = 8;                    // consumer warps
constexpr int kCThreads = kCWarps * 32;
constexpr int kStepThreads = kCThreads + 32;  // + one producer warp
constexpr int kChunk = 256;                   // attention tokens per work item
constexpr int kMaxGroup = 16;                 // query heads per kv head

// Shared memory: mbarriers, scalars, per-stage partial sums (two parities),
// the phase work area (input vector, or the attention item's buffers), ring.
constexpr int kOffFull = 0;
constexpr int kOffEmpty = kOffFull + 8 * kStepMaxSlots;
constexpr int kOffMisc = kOffEmpty + 8 * kStepMaxSlots;
constexpr int kMiscBytes = 512;
constexpr int kOffRed = kOffMisc + kMiscBytes;
constexpr int kRedFloats = kStepMaxStageRows * kCWarps;
constexpr int kOffUnion = kOffRed + 2 * kRedFloats * 4;
// misc words
constexpr int kMiscAbort = 0;    // int: the consumers gave up (the producer stops)
constexpr int kMiscLast = 4;     // int: this CTA merges (attention) / reduces (argmax)
constexpr int kMiscDred = 64;    // double[8]: RMSNorm partial sums per warp
constexpr int kMiscBest = 128;   // {float, int}[8]: argmax per warp

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// Consumer barrier that also ORs a per-thread flag: every consumer thread
// gets the same answer, so a failure seen by any thread stops all of them at
// the same point.
__device__ __forceinline__ bool cbar_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_relaxed_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_add_relaxed_gpu(uint32_t* p, uint32_t v) {
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Activations written by other CTAs in this launch are read through L2
// (ld.global.cg), never through the non-coherent or L1 paths.
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

struct Ctx {
  const StepParams* p;
  unsigned char* smem;
  uint64_t* full;
  uint64_t* empty;
  float* red;
  float* U;            // phase work area
  unsigned char* ring;
  int b, G, tid, warp, lane;
  uint32_t stage;      // stages consumed
  uint32_t phase;      // phases this CTA has arrived at
};

__device__ __forceinline__ bool stop_all(Ctx& c, bool fail) {
  const bool any = cbar_or(fail);
  if (any && c.tid == 0) *reinterpret_cast<volatile int*>(c.smem + kOffMisc + kMiscAbort) = 1;
  return any;
}

// Start of a phase: every CTA has arrived at the previous one (count >=
// phase * grid).  Thread 0 polls; the barrier hands the outcome to all.
__device__ bool grid_wait(Ctx& c) {
  bool fail = false;
  if (c.tid == 0 && c.phase > 0) {
    const uint32_t target = c.phase * (uint32_t)c.G;
    uint32_t* cnt = &c.p->sync[0];
    if (ld_relaxed_gpu(cnt) < target) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t n = 0;
      while (ld_relaxed_gpu(cnt) < target) {
        if ((++n & 63u) == 0 && (ld_relaxed_gpu_s32(c.p->error) != 0 || globaltimer_ns() - t0 > kWaitLimitNs)) {
          fail = true;
          break;
        }
      }
    }
    fence_acq_rel_gpu();
    if (fail) set_error(c.p->error, 60);
  }
  return !stop_all(c, fail);
}

// End of a phase: all consumer threads' writes of it are published by one
// release from thread 0.
__device__ __forceinline__ void grid_arrive(Ctx& c) {
  cbar();
  if (c.tid == 0) {
    fence_acq_rel_gpu();
    red_add_relaxed_gpu(&c.p->sync[0], 1u);
  }
  ++c.phase;
}

// ---- phase prologues: the input vector of a projection into U -------------

// te_rmsnorm_f32 (c/src/ops.c:272-293): squares summed in double, scale =
// 1 / sqrtf((float)(sum / n) + eps), out = (x * scale) * w.
__device__ void prologue_rmsnorm(Ctx& c, const float* src, const float* w) {
  const int H = c.p->hidden;
  double ss = 0.0;
  for (int i = c.tid * 4; i < H; i += kCThreads * 4) {
    const float4 v = ldcg4(src + i);
    *reinterpret_cast<float4*>(c.U + i) = v;
    ss += (double)v.x * (double)v.x + (double)v.y * (double)v.y + (double)v.z * (double)v.z +
          (double)v.w * (double)v.w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  double* dred = reinterpret_cast<double*>(c.smem + kOffMisc + kMiscDred);
  if (c.lane == 0) dred[c.warp] = ss;
  cbar();
  double tot = 0.0;
#pragma unroll
  for (int k = 0; k < kCWarps; ++k) tot += dred[k];
  const float scale = 1.0f / sqrtf((float)(tot / (double)H) + c.p->eps);
  for (int i = c.tid * 4; i < H; i += kCThreads * 4) {
    float4 v = *reinterpret_cast<const float4*>(c.U + i);
    const float4 ww = __ldg(reinterpret_cast<const float4*>(w + i));
    v = make_float4((v.x * scale) * ww.x, (v.y * scale) * ww.y, (v.z * scale) * ww.z, (v.w * scale) * ww.w);
    *reinterpret_cast<float4*>(c.U + i) = v;
  }
  cbar();
}

__device__ void prologue_copy(Ctx& c, const float* src, int n) {
  for (int i = c.tid * 4; i < n; i += kCThreads * 4) *reinterpret_cast<float4*>(c.U + i) = ldcg4(src + i);
  cbar();
}

// te_swiglu_f32 (c/src/ops.c:397-406): gate / (1 + expf(-gate)) * up.
__device__ void prologue_swiglu(Ctx& c) {
  const int F = c.p->ffn;
  for (int i = c.tid; i < F; i += kCThreads) c.U[i] = silu(ldcg(c.p->gu + i)) * ldcg(c.p->gu + F + i);
  cbar();
}

// ---- projections ----------------------------------------------------------

// Lane's 8 weights of one block (Q4_0: quant bytes 4j..4j+3 = weights 4j..
// 4j+3 (low nibbles) and 16+4j.. (high); Q8_0: weights 8j..8j+7) dotted with
// its 8 inputs: sum (q - offset) * x with exact weights, then * the block's
// f16 scale (the reference's te_q4_0_dot_row / te_q8_0_dot_row products,
// c/src/ops.c:584-620).
template <int BB>
__device__ __forceinline__ float block_dot(const unsigned char* blk, int j, const uint64_t (&xs)[4]) {
  constexpr float kOff = BB == 18 ? 8388616.0f : 8388736.0f;  // 2^23 + the quant offset (8 or 128)
  const uint64_t off2 = f2_pack(kOff, kOff);
  const float sc = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk)));
  const uint16_t* qp = reinterpret_cast<const uint16_t*>(blk + (BB == 18 ? 2 + 4 * j : 2 + 8 * j));
  uint32_t lo, hi;
  if (BB == 18) {
    const uint32_t q = prmt(qp[0], qp[1], 0x5410u);
    lo = q & 0x0f0f0f0fu;
    hi = (q >> 4) & 0x0f0f0f0fu;
  } else {
    lo = prmt(qp[0], qp[1], 0x5410u) ^ 0x80808080u;
    hi = prmt(qp[2], qp[3], 0x5410u) ^ 0x80808080u;
  }
  uint64_t wq[4];
  wq[0] = f2_pack(__uint_as_float(prmt(lo, 0x4B000000u, 0x7440u)), __uint_as_float(prmt(lo, 0x4B000000u, 0x7441u)));
  wq[1] = f2_pack(__uint_as_float(prmt(lo, 0x4B000000u, 0x7442u)), __uint_as_float(prmt(lo, 0x4B000000u, 0x7443u)));
  wq[2] = f2_pack(__uint_as_float(prmt(hi, 0x4B000000u, 0x7440u)), __uint_as_float(prmt(hi, 0x4B000000u, 0x7441u)));
  wq[3] = f2_pack(__uint_as_float(prmt(hi, 0x4B000000u, 0x7442u)), __uint_as_float(prmt(hi, 0x4B000000u, 0x7443u)));
#pragma unroll
  for (int k = 0; k < 4; ++k) wq[k] = f2_sub(wq[k], off2);
  uint64_t d = f2_mul(wq[0], xs[0]);
#pragma unroll
  for (int k = 1; k < 4; ++k) d = f2_fma(wq[k], xs[k], d);
  float d0, d1;
  f2_unpack(d, d0, d1);
  return sc * (d0 + d1);
}

// Warps per row for a stage of R rows and S column steps (a step is 8
// blocks, one per four lanes): the split with the least work per warp.
__device__ __forceinline__ int stage_wpr(int R, int S) {
  int best = 1, cost = ((R + kCWarps - 1) / kCWarps) * S;
#pragma unroll
  for (int w = 2; w <= kCWarps; w *= 2) {
    const int rg = kCWarps / w;
    const int cw = ((R + rg - 1) / rg) * ((S + w - 1) / w);
    if (cw < cost) {
      cost = cw;
      best = w;
    }
  }
  return best;
}

// Partial dot products of a stage's R rows into red[row][part]: warp w takes
// rows w / wpr, + 8 / wpr, ... and column steps w % wpr, + wpr, ...; the
// input values a lane loads serve up to four rows.
template <int BB>
__device__ void stage_rows(const unsigned char* base, int row_bytes, int R, int nb, int S, int wpr, const float* xin,
                           float* red, int warp, int lane) {
  const int rg = kCWarps / wpr, rgi = warp / wpr, cp = warp % wpr;
  const int j = lane & 3;
  const int xo0 = BB == 18 ? 4 * j : 8 * j;
  const int xo1 = BB == 18 ? 16 + 4 * j : 8 * j + 4;
  for (int rb = rgi; rb < R; rb += 4 * rg) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int st = cp; st < S; st += wpr) {
      const int blk = st * 8 + (lane >> 2);
      if (blk < nb) {
        const float4 a = *reinterpret_cast<const float4*>(xin + blk * 32 + xo0);
        const float4 e = *reinterpret_cast<const float4*>(xin + blk * 32 + xo1);
        const uint64_t xs[4] = {f2_pack(a.x, a.y), f2_pack(a.z, a.w), f2_pack(e.x, e.y), f2_pack(e.z, e.w)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = rb + i * rg;
          if (r < R) acc[i] += block_dot<BB>(base + (size_t)r * row_bytes + blk * BB, j, xs);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = rb + i * rg;
      if (r < R) {  // the same for the whole warp
        float s = acc[i];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) red[r * kCWarps + cp] = s;
      }
    }
  }
}

// One projection phase over this CTA's rows: y[row] = dot, or resid[row] +
// dot (fp32 add: the residual add after the output and down projections);
// with `best` also the running first-maximum (value, row) of the outputs.
__device__ bool gemv_phase(Ctx& c, int kind, float* y, const float* resid, float* best_v, int* best_i) {
  const StepParams& p = *c.p;
  const StepMat& m = p.mat[kind];
  int r0;
  const int n = step_cta_rows(m, c.b, r0);
  const int ns = step_n_stages(n, m.rps);
  const int nb = m.cols / 32;
  const int S = (nb + 7) / 8;
  for (int s = 0; s < ns; ++s) {
    const int lo = step_stage_lo(s, n, ns);
    const int R = step_stage_lo(s + 1, n, ns) - lo;
    const int wpr = stage_wpr(R, S);
    const uint32_t slot = c.stage % (uint32_t)p.n_slots;
    const bool ok = mbar_wait_warp(&c.full[slot], (c.stage / (uint32_t)p.n_slots) & 1u);
    float* red = c.red + (c.stage & 1u) * kRedFloats;
    if (ok) {
      const unsigned char* base = c.ring + (size_t)slot * p.slot_bytes;
      if (m.block_bytes == 18) {
        stage_rows<18>(base, m.row_bytes, R, nb, S, wpr, c.U, red, c.warp, c.lane);
      } else {
        stage_rows<34>(base, m.row_bytes, R, nb, S, wpr, c.U, red, c.warp, c.lane);
      }
    }
    __syncwarp();
    if (c.lane == 0) mbar_arrive(&c.empty[slot]);  // this warp is done with the slot
    ++c.stage;
    if (!ok) set_error(p.error, 61);
    if (stop_all(c, !ok)) return false;  // also: the stage's partial sums are complete
    if (c.tid < R) {
      float sum = red[c.tid * kCWarps];
      for (int k = 1; k < wpr; ++k) sum += red[c.tid * kCWarps + k];
      const int row = r0 + lo + c.tid;
      if (resid) sum = __fadd_rn(ldcg(resid + row), sum);
      y[row] = sum;
      if (best_v && sum > *best_v) {  // rows ascend per thread: the first maximum
        *best_v = sum;
        *best_i = row;
      }
    }
  }
  return true;
}

// ---- attention ------------------------------------------------------------

__device__ __forceinline__ size_t cache_row(const StepParams& p, int layer, int g, int tok) {
  const int page = p.page_base >= 0 ? p.page_base + tok / p.page_tokens : __ldg(p.page_row + tok / p.page_tokens);
  return ((size_t)((size_t)layer * p.num_pages + page) * p.kv_heads + g) * p.page_tokens + (tok % p.page_tokens);
}

// One work item: kv head g, tokens [ch * kChunk, +kChunk) of n_tokens.  The
// query of head h (of this kv head's group) is the reference's
// q + bias, rotated at the new token's position (c/src/qwen.c:998-1036);
// scores are q.k * log2(e) / sqrt(hd) and exp2 replaces expf (the same
// softmax); the new token's k (bias, RoPE) and v (bias) go into the cache
// rounded to f16 (RNE) first, as the per-op decode's appender does.
template <int HD>
__device__ void attention_item(Ctx& c, int layer, int g, int ch, int nch) {
  const StepParams& p = *c.p;
  constexpr int half = HD / 2;
  constexpr int DPL = HD / 32;  // dims per lane in P.V
  const int Gq = p.group;
  float* qs = c.U;                                   // [kMaxGroup][HD]
  float* sc = qs + kMaxGroup * HD;                   // [kMaxGroup][kChunk]
  float* ml = sc + kMaxGroup * kChunk;               // [kMaxGroup][2]
  int* rowid = reinterpret_cast<int*>(ml + 2 * kMaxGroup);  // [kChunk]
  const float* cosr = p.rope_cos + (size_t)p.rope_pos * half;
  const float* sinr = p.rope_sin + (size_t)p.rope_pos * half;
  const int QH = p.heads * HD;
  const int KV = p.kv_heads * HD;

  for (int e = c.tid; e < Gq * half; e += kCThreads) {
    const int h = e / half, d = e - h * half;
    const int qh = g * Gq + h;
    float a = ldcg(p.qkv + qh * HD + d), bb = ldcg(p.qkv + qh * HD + d + half);
    if (p.q_bias) {
      const float* qb = p.q_bias + ((size_t)layer * p.heads + qh) * HD;
      a = __fadd_rn(a, __ldg(qb + d));
      bb = __fadd_rn(bb, __ldg(qb + d + half));
    }
    const float cs = __ldg(cosr + d), sn = __ldg(sinr + d);
    qs[h * HD + d] = rope_lo(a, bb, cs, sn);
    qs[h * HD + d + half] = rope_hi(a, bb, cs, sn);
  }
  const int t0 = ch * kChunk;
  const int t1 = min(p.n_tokens, t0 + kChunk);
  const int nt = t1 - t0;
  for (int t = c.tid; t < nt; t += kCThreads) rowid[t] = (int)cache_row(p, layer, g, t0 + t);
  if (t1 == p.n_tokens) {
    const size_t row = cache_row(p, layer, g, p.n_tokens - 1);
    const size_t kvb = ((size_t)layer * p.kv_heads + g) * HD;
    for (int d = c.tid; d < half; d += kCThreads) {
      float a = ldcg(p.qkv + QH + g * HD + d), bb = ldcg(p.qkv + QH + g * HD + d + half);
      if (p.k_bias) {
        a = __fadd_rn(a, __ldg(p.k_bias + kvb + d));
        bb = __fadd_rn(bb, __ldg(p.k_bias + kvb + d + half));
      }
      const float cs = __ldg(cosr + d), sn = __ldg(sinr + d);
      p.k_pool[row * HD + d] = __half_as_ushort(__float2half_rn(rope_lo(a, bb, cs, sn)));
      p.k_pool[row * HD + d + half] = __half_as_ushort(__float2half_rn(rope_hi(a, bb, cs, sn)));
    }
    for (int d = c.tid; d < HD; d += kCThreads) {
      float v = ldcg(p.qkv + QH + KV + g * HD + d);
      if (p.v_bias) v = __fadd_rn(v, __ldg(p.v_bias + kvb + d));
      p.v_pool[row * HD + d] = __half_as_ushort(__float2half_rn(v));
    }
  }
  cbar();  // queries, row ids and the new cache row are in place

  if (c.tid < nt) {  // scores: one token per thread, every head of the group
    const uint4* kr = reinterpret_cast<const uint4*>(p.k_pool + (size_t)rowid[c.tid] * HD);
    float dot[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) dot[h] = 0.f;
#pragma unroll 2
    for (int d8 = 0; d8 < HD / 8; ++d8) {
      float kv[8];
      unpack8(__ldcg(kr + d8), kv);
#pragma unroll
      for (int h = 0; h < kMaxGroup; ++h) {
        if (h < Gq) {
          const float4 q0 = *reinterpret_cast<const float4*>(qs + h * HD + d8 * 8);
          const float4 q1 = *reinterpret_cast<const float4*>(qs + h * HD + d8 * 8 + 4);
          float s = dot[h];
          s = fmaf(q0.x, kv[0], s); s = fmaf(q0.y, kv[1], s); s = fmaf(q0.z, kv[2], s); s = fmaf(q0.w, kv[3], s);
          s = fmaf(q1.x, kv[4], s); s = fmaf(q1.y, kv[5], s); s = fmaf(q1.z, kv[6], s); s = fmaf(q1.w, kv[7], s);
          dot[h] = s;
        }
      }
    }
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) {
      if (h < Gq) sc[h * kChunk + c.tid] = dot[h] * p.scale_log2;
    }
  }
  cbar();

  for (int h = c.warp; h < Gq; h += kCWarps) {  // softmax of head h: one warp
    float mx = -INFINITY;
    for (int t = c.lane; t < nt; t += 32) mx = fmaxf(mx, sc[h * kChunk + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float l = 0.f;
    for (int t = c.lane; t < nt; t += 32) {
      const float e = ex2(sc[h * kChunk + t] - mx);
      sc[h * kChunk + t] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    __syncwarp();
    float acc[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
#pragma unroll 4
    for (int t = 0; t < nt; ++t) {  // P.V: lane -> DPL dims, coalesced rows
      const float pw = sc[h * kChunk + t];
      const uint16_t* vr = p.v_pool + (size_t)rowid[t] * HD + c.lane * DPL;
      if constexpr (DPL == 2) {
        const unsigned int u = __ldcg(reinterpret_cast<const unsigned int*>(vr));
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
        acc[0] = fmaf(pw, f.x, acc[0]);
        acc[1] = fmaf(pw, f.y, acc[1]);
      } else {
        const uint2 u = __ldcg(reinterpret_cast<const uint2*>(vr));
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
        acc[0] = fmaf(pw, f0.x, acc[0]);
        acc[1] = fmaf(pw, f0.y, acc[1]);
        acc[2] = fmaf(pw, f1.x, acc[2]);
        acc[3] = fmaf(pw, f1.y, acc[3]);
      }
    }
    if (nch == 1) {
      const float inv = 1.0f / l;
      float* o = p.attn + (size_t)(g * Gq + h) * HD + c.lane * DPL;
#pragma unroll
      for (int i = 0; i < DPL; ++i) o[i] = acc[i] * inv;
    } else {
      float* r = p.rec + ((size_t)(g * nch + ch) * Gq + h) * (HD + 2);
#pragma unroll
      for (int i = 0; i < DPL; ++i) r[c.lane * DPL + i] = acc[i];
      if (c.lane == 0) {
        r[HD] = mx;
        r[HD + 1] = l;
      }
    }
  }
  if (nch == 1) {
    cbar();  // the work area is reused by the next item
    return;
  }
  // several chunks: the last CTA to finish one of this kv head's chunks merges them
  int* s_last = reinterpret_cast<int*>(c.smem + kOffMisc + kMiscLast);
  cbar();
  if (c.tid == 0) {
    __threadfence();
    const uint32_t old = atomicAdd(&p.sync[4 + g], 1u);
    *s_last = old == (uint32_t)(nch - 1);
  }
  cbar();
  if (*s_last) {
    __threadfence();
    for (int h = c.warp; h < Gq; h += kCWarps) {
      float M = -INFINITY;
      for (int k = 0; k < nch; ++k) M = fmaxf(M, ldcg(p.rec + ((size_t)(g * nch + k) * Gq + h) * (HD + 2) + HD));
      float L = 0.f, acc[DPL];
#pragma unroll
      for (int i = 0; i < DPL; ++i) acc[i] = 0.f;
      for (int k = 0; k < nch; ++k) {
        const float* r = p.rec + ((size_t)(g * nch + k) * Gq + h) * (HD + 2);
        const float w = ex2(ldcg(r + HD) - M);
        L = fmaf(ldcg(r + HD + 1), w, L);
#pragma unroll
        for (int i = 0; i < DPL; ++i) acc[i] = fmaf(ldcg(r + c.lane * DPL + i), w, acc[i]);
      }
      const float inv = 1.0f / L;
      float* o = p.attn + (size_t)(g * Gq + h) * HD + c.lane * DPL;
#pragma unroll
      for (int i = 0; i < DPL; ++i) o[i] = acc[i] * inv;
    }
    if (c.tid == 0) atomicExch(&p.sync[4 + g], 0u);
  }
  cbar();
}

template <int HD>
__device__ void attention_phase(Ctx& c, int layer) {
  const StepParams& p = *c.p;
  const int nch = (p.n_tokens + kChunk - 1) / kChunk;
  const int items = p.kv_heads * nch;
  for (int it = c.b; it < items; it += c.G) attention_item<HD>(c, layer, it / nch, it % nch, nch);
}

// ---- argmax ---------------------------------------------------------------

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

__device__ void argmax_finish(Ctx& c, float bv, int bi) {
  const StepParams& p = *c.p;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  float* wb = reinterpret_cast<float*>(c.smem + kOffMisc + kMiscBest);
  if (c.lane == 0) {
    wb[2 * c.warp] = bv;
    wb[2 * c.warp + 1] = __int_as_float(bi);
  }
  cbar();
  if (c.tid != 0) return;
  for (int w = 1; w < kCWarps; ++w) {
    const float v = wb[2 * w];
    const int i = __float_as_int(wb[2 * w + 1]);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  // wb[0..1] already hold warp 0's, which the loop started from
  p.cand[2 * c.b] = bv;
  p.cand[2 * c.b + 1] = __int_as_float(bi);
  __threadfence();
  const uint32_t old = atomicAdd(&p.sync[2], 1u);
  if (old != (uint32_t)(c.G - 1)) return;
  __threadfence();
  float fv = -INFINITY;
  int fi = INT_MAX;
  for (int k = 0; k < c.G; ++k) {
    const float v = ldcg(p.cand + 2 * k);
    const int i = __float_as_int(ldcg(p.cand + 2 * k + 1));
    if (better(v, i, fv, fi)) {
      fv = v;
      fi = i;
    }
  }
  *p.token_out = fi == INT_MAX ? 0 : fi;
  atomicExch(&p.sync[2], 0u);
}

// ---- the two roles --------------------------------------------------------

__device__ void consumer(Ctx& c) {
  const StepParams& p = *c.p;
  const long long tok = __ldcg(reinterpret_cast<const long long*>(p.token_in));
  int token = (int)tok;
  if (tok < 0 || tok >= p.vocab) {
    if (c.tid == 0) set_error(p.error, 63);
    token = 0;
  }
  const float* emb_row = p.emb + (size_t)token * p.hidden;
  const size_t H = (size_t)p.hidden;
  for (int l = 0; l < p.layers; ++l) {
    if (!grid_wait(c)) return;  // A
    prologue_rmsnorm(c, l == 0 ? emb_row : p.x, p.attn_norm + l * H);
    if (!gemv_phase(c, kStepQKV, p.qkv, nullptr, nullptr, nullptr)) return;
    grid_arrive(c);
    if (!grid_wait(c)) return;  // B
    if (p.head_dim == 64) {
      attention_phase<64>(c, l);
    } else {
      attention_phase<128>(c, l);
    }
    grid_arrive(c);
    if (!grid_wait(c)) return;  // C
    prologue_copy(c, p.attn, p.hidden);
    if (!gemv_phase(c, kStepO, p.x, l == 0 ? emb_row : p.x, nullptr, nullptr)) return;
    grid_arrive(c);
    if (!grid_wait(c)) return;  // D
    prologue_rmsnorm(c, p.x, p.ffn_norm + l * H);
    if (!gemv_phase(c, kStepGU, p.gu, nullptr, nullptr, nullptr)) return;
    grid_arrive(c);
    if (!grid_wait(c)) return;  // E
    prologue_swiglu(c);
    if (!gemv_phase(c, kStepDown, p.x, p.x, nullptr, nullptr)) return;
    grid_arrive(c);
  }
  if (!p.head) return;
  if (!grid_wait(c)) return;
  prologue_rmsnorm(c, p.x, p.out_norm);
  float bv = -INFINITY;
  int bi = INT_MAX;
  if (!gemv_phase(c, kStepHead, p.logits, nullptr, &bv, &bi)) return;
  argmax_finish(c, bv, bi);
}

// One lane: streams this CTA's packed weights through the ring in
// consumption order, each slot refilled once all consumer warps released it.
__device__ void producer(const StepParams& p, unsigned char* ring, uint64_t* full, uint64_t* empty,
                         volatile int* s_abort) {
  const int b = blockIdx.x;
  const unsigned char* src = p.wpack + p.cta_off[b];
  const uint32_t NS = (uint32_t)p.n_slots;
  uint32_t i = 0;
  bool ok = true;
  auto put = [&](uint32_t bytes) {
    const uint32_t slot = i % NS;
    if (i >= NS) {
      const uint32_t par = ((i / NS) - 1u) & 1u;
      if (!mbar_try_wait(&empty[slot], par)) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t n = 0;
        while (!mbar_try_wait(&empty[slot], par)) {
          if ((++n & 15u) == 0 && (*s_abort != 0 || globaltimer_ns() - t0 > kWaitLimitNs)) {
            ok = false;
            break;
          }
        }
        if (!ok) {
          set_error(p.error, 62);  // keeps an earlier code (first error wins)
          return;
        }
      }
    }
    mbar_arrive_expect_tx(&full[slot], bytes);
    bulk_load(ring + (size_t)slot * p.slot_bytes, src, bytes, &full[slot]);
    src += bytes;
    ++i;
  };
  auto stream = [&](int kind) {
    const StepMat& m = p.mat[kind];
    int r0;
    const int n = step_cta_rows(m, b, r0);
    const int ns = step_n_stages(n, m.rps);
    for (int s = 0; s < ns && ok; ++s) {
      put(step_stage_bytes(step_stage_lo(s + 1, n, ns) - step_stage_lo(s, n, ns), m.row_bytes));
    }
  };
  for (int l = 0; l < p.layers && ok; ++l) {
    for (int k = kStepQKV; k <= kStepDown && ok; ++k) stream(k);
  }
  if (p.head && ok) stream(kStepHead);
  // No copy may still be landing when the CTA exits (the consumers may have
  // given up before using the last stages): wait for the newest use of every
  // slot (already complete in a normal run).
  for (uint32_t j = i > NS ? i - NS : 0; j < i; ++j) mbar_wait(&full[j % NS], (j / NS) & 1u);
}

__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kOffEmpty);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kOffMisc + kMiscAbort);
  unsigned char* ring = smem + kOffUnion + p.union_bytes;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < p.n_slots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kCWarps);
    }
    fence_mbarrier_init();
    *s_abort = 0;
  }
  __syncthreads();
  if (warp == kCWarps) {
    if (lane == 0) producer(p, ring, full, empty, s_abort);
  } else {
    Ctx c;
    c.p = &p;
    c.smem = smem;
    c.full = full;
    c.empty = empty;
    c.red = reinterpret_cast<float*>(smem + kOffRed);
    c.U = reinterpret_cast<float*>(smem + kOffUnion);
    c.ring = ring;
    c.b = blockIdx.x;
    c.G = gridDim.x;
    c.tid = tid;
    c.warp = warp;
    c.lane = lane;
    c.stage = 0;
    c.phase = 0;
    consumer(c);
    if (tid == 0) *s_abort = 1;  // done (or gave up): a producer still waiting for a slot stops
  }
  __syncthreads();
  if (tid == 0) {
    // the last CTA out clears the launch's counters for the next step
    __threadfence();
    const uint32_t old = atomicAdd(&p.sync[1], 1u);
    if (old == gridDim.x - 1) {
      atomicExch(&p.sync[0], 0u);
      atomicExch(&p.sync[2], 0u);
      for (int g = 0; g < p.kv_heads; ++g) atomicExch(&p.sync[4 + g], 0u);
      atomicExch(&p.sync[1], 0u);
    }
  }
}

__global__ void step_pack_kernel(const StepPackSeg* segs, int n, unsigned char* dst) {
  for (int s = blockIdx.x; s < n; s += gridDim.x) {
    const StepPackSeg sg = segs[s];
    const uint16_t* src = reinterpret_cast<const uint16_t*>(sg.src);
    uint16_t* d = reinterpret_cast<uint16_t*>(dst + sg.dst_off);
    for (long long i = threadIdx.x; i < sg.bytes / 2; i += blockDim.x) d[i] = src[i];
  }
}

}  // namespace

void plan_step_mat(StepMat& m, int rows, int cols, int block_bytes, int grid, int slot_bytes) {
  m.rows = rows;
  m.cols = cols;
  m.block_bytes = block_bytes;
  m.row_bytes = cols / 32 * block_bytes;
  m.rpc = (rows + grid - 1) / grid;
  int rps = slot_bytes / m.row_bytes;
  if (rps > kStepMaxStageRows) rps = kStepMaxStageRows;
  m.rps = rps < 1 ? 1 : rps;
}

int step_fixed_smem() { return kOffUnion; }

int step_smem_bytes(int slot_bytes, int n_slots, int union_bytes) {
  return kOffUnion + union_bytes + slot_bytes * n_slots;
}

cudaError_t step_configure() {
  static std::atomic<uint64_t> configured{0};  // one bit per device
  return set_smem_limit_once(configured, (const void*)step_kernel, 227 * 1024);
}

int step_max_ctas_per_sm(int smem) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, step_kernel, kStepThreads, (size_t)smem) != cudaSuccess) {
    return 0;
  }
  return n;
}

cudaError_t launch_step(const StepParams& p, int grid, int smem, cudaStream_t s) {
  // cooperative: every CTA is resident at once (the phases wait on each other)
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, step_kernel, p);
}

cudaError_t launch_step_pack(const StepPackSeg* segs, int n, unsigned char* dst, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  const int grid = n < 4096 ? n : 4096;
  step_pack_kernel<<<grid, 256, 0, s>>>(segs, n, dst);
  return cudaGetLastError();
}

}  // namespace te
