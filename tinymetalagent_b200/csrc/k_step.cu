// Whole-token qwen2 decode step in one cooperative launch.
//
// Reference semantics: te_qwen_forward_token (c/src/qwen.c:907-1112) runs,
// per layer, RMSNorm -> q/k/v projections + biases -> RoPE -> KV append ->
// GQA attention -> output projection + residual -> RMSNorm -> gate/up ->
// SwiGLU -> down projection + residual; te_qwen_project_next (:1303-1377)
// then applies the output RMSNorm, the lm_head and the argmax.  The per-op
// path of this library runs that as five launches per layer; here one
// persistent grid (one CTA per SM) runs all of it.  Between dependent phases
// there is no grid-wide barrier: every vector a phase produces for other CTAs
// (q|k|v, attention output, x, SwiGLU output) is written as 64-bit words
// {value, tag}, the tag naming the launch, layer and phase, and a reader
// takes each word as soon as its tag is the one it expects -- the data and
// its readiness arrive in one load (the low-latency protocol of NCCL's LL
// transport).  A CTA with no rows in a phase skips it and waits only where
// it has work.
//
// Weights do not depend on activations, so they are streamed without regard
// to phases: CTA b owns a fixed row slice of every projection, its share of
// all weights is packed host-side into one contiguous byte stream in the
// order it consumes them (stages of up to 64 whole rows, stored transposed
// and 16-byte aligned), and a producer warp copies that stream through a byte
// ring in shared memory (cp.async.bulk, completion on the stage's mbarrier)
// as fast as the consumers release space.  While the twelve consumer warps
// wait for a phase's input, the producer keeps fetching the next phases' (and
// layers') rows, so a phase starts with its weights already on chip.
//
// Phases per layer (a CTA with no rows or items in a phase skips it):
//   A  q|k|v = W_qkv RMSNorm(x)       rows of the stacked q, k, v matrices
//   B  attention                       work items (kv head, 128-token chunk):
//                                      bias + RoPE of the group's queries, the
//                                      new k/v (bias, RoPE on k, f16 RNE) into
//                                      the paged cache, scores, softmax, P.V;
//                                      chunks of one kv head merge by
//                                      log-sum-exp in the last arriving CTA
//   C  x = x + W_o attn
//   D  h = SwiGLU(W_gate RMSNorm(x), W_up RMSNorm(x))   (gate and up rows of
//                                      a stage side by side, SwiGLU in the epilogue)
//   E  x = x + W_down h
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

constexpr int kCWarps = 12;                   // consumer warps (three per SM sub-partition)
constexpr int kCThreads = kCWarps * 32;
constexpr int kStepThreads = kCThreads + 32;  // + one producer warp
constexpr int kChunk = kStepChunk;            // attention tokens per work item
constexpr int kMaxGroup = kStepMaxGroup;      // query heads per kv head

// Shared memory: mbarriers, scalars, per-stage partial sums (two parities),
// the phase work area (input vector, or the attention item's buffers), ring.
constexpr int kOffFull = 0;
constexpr int kOffEmpty = kOffFull + 8 * kStepMaxSlots;
constexpr int kOffMisc = kOffEmpty + 8 * kStepMaxSlots;
constexpr int kMiscBytes = 768;
constexpr int kOffRed = kOffMisc + kMiscBytes;
constexpr int kRedFloats = kStepMaxStageRows * kCWarps;
constexpr int kOffUnion = kOffRed + 2 * kRedFloats * 4;
// misc words
constexpr int kMiscAbort = 0;    // int: the consumers gave up (the producer stops)
constexpr int kMiscLast = 4;     // int: this CTA merges (attention) / reduces (argmax)
constexpr int kMiscDred = 64;    // double[kCWarps]: RMSNorm partial sums per warp
constexpr int kMiscBest = 160;   // {float, int}[kCWarps]: argmax per warp
constexpr int kMiscRing = 256;   // u32[2][kStepMaxSlots]: the producer's in-flight stage ranges
constexpr int kMiscXown = 512;   // float[kStepMaxOwnRows]: this CTA's rows of the residual stream x
constexpr uint32_t kNQ = kStepMaxSlots;  // stage descriptors (full/empty mbarrier pairs), a power of two
static_assert((kNQ & (kNQ - 1)) == 0 && kMiscRing + 8 * kStepMaxSlots <= kMiscBytes, "ring descriptors");
static_assert(kMiscDred + 8 * kCWarps <= kMiscBest && kMiscBest + 8 * kCWarps <= kMiscRing, "misc layout");
static_assert(kMiscXown + 4 * kStepMaxOwnRows <= kMiscBytes, "misc layout");

// The weight ring is a byte ring: stage i takes [off, off + bytes) at the
// running head, or at 0 when it would pass the end.  Producer and consumers
// apply the same rule to the same sequence of stage sizes, so only the
// mbarriers of stage descriptor i % kNQ pass between them.
__device__ __forceinline__ uint32_t ring_place(uint32_t& head, uint32_t bytes, uint32_t cap) {
  const uint32_t off = head + bytes <= cap ? head : 0u;
  head = off + bytes;
  return off;
}

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory"); }

// Consumer barrier that also ORs a per-thread flag: every consumer thread
// gets the same answer, so a failure seen by any thread stops all of them at
// the same point.
__device__ __forceinline__ bool cbar_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "n"(kCThreads)
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

// Activations written by other CTAs in this launch are read through L2
// (ld.global.cg), never through the non-coherent or L1 paths.
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

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
  uint32_t head;       // ring head after the stages consumed
  uint32_t epoch;      // this launch's tag field (advanced by the last CTA of each launch)
};

__device__ __forceinline__ bool stop_all(Ctx& c, bool fail) {
  const bool any = cbar_or(fail);
  if (any && c.tid == 0) *reinterpret_cast<volatile int*>(c.smem + kOffMisc + kMiscAbort) = 1;
  return any;
}

// ---- tagged words -----------------------------------------------------------
// Tag of the vector phase `ph` (0 q|k|v, 1 attention, 2 x after the output
// projection, 3 SwiGLU, 4 x after the down projection) of layer l.
__device__ __forceinline__ uint32_t tag_of(const Ctx& c, int l, int ph) {
  return ((c.epoch + 1u) << 10) | ((uint32_t)l << 3) | (uint32_t)ph;
}
// One 64-bit store: a reader that sees the tag sees the value (single-copy
// atomic 8-byte accesses).
__device__ __forceinline__ void st_ll(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_ll(const unsigned long long* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Bounded polling with a short backoff: words that are not there yet are
// re-read after 32, 64, ... 256 ns, so that the CTAs waiting for a vector do
// not crowd the L2 lines its writers are storing to.  Gives up after 2 s or
// when another CTA reported an error.
struct Poll {
  uint64_t t0 = 0;
  uint32_t tries = 0;
  __device__ __forceinline__ bool again(const StepParams& p) {
    if (tries == 0) t0 = globaltimer_ns();
    __nanosleep(32u << (tries < 3 ? tries : 3));
    ++tries;
    if ((tries & 15u) == 0 && (ld_relaxed_gpu_s32(p.error) != 0 || globaltimer_ns() - t0 > kWaitLimitNs)) {
      set_error(p.error, 60);
      return false;
    }
    return true;
  }
};
// Two words loaded together, then completed.
__device__ __forceinline__ bool ll_get2(const StepParams& p, const unsigned long long* a, const unsigned long long* b,
                                        uint32_t tag, float& va, float& vb) {
  unsigned long long wa = ld_ll(a), wb = ld_ll(b);
  Poll poll;
  while ((uint32_t)(wa >> 32) != tag || (uint32_t)(wb >> 32) != tag) {
    if (!poll.again(p)) return false;
    if ((uint32_t)(wa >> 32) != tag) wa = ld_ll(a);
    if ((uint32_t)(wb >> 32) != tag) wb = ld_ll(b);
  }
  va = __uint_as_float((uint32_t)wa);
  vb = __uint_as_float((uint32_t)wb);
  return true;
}
// n tagged words into U, up to kLL loads in flight per thread (the stale
// ones re-read together); ends with a consumer barrier (false: some word
// never arrived, the CTA stops).  With norm_w, U becomes te_rmsnorm_f32 of
// the vector (c/src/ops.c:272-293: squares summed in double, scale =
// 1 / sqrtf((float)(sum / n) + eps), out = (x * scale) * w), the squares
// summed as the words arrive.
__device__ bool ll_stage(Ctx& c, const unsigned long long* src, int n, uint32_t tag, const float* norm_w = nullptr) {
  double ss = 0.0;
  constexpr int kLL = 8;
  // the norm weights go to shared memory past the vector (cp.async), in flight while the words are awaited
  float* wn = c.U + ((n + 3) & ~3);
  if (norm_w) {
    for (int i = c.tid * 4; i < n; i += kCThreads * 4) cp_async_cg16(smem_u32(wn + i), norm_w + i);
  }
  bool ok = true;
  for (int base = c.tid; base < n && ok; base += kCThreads * kLL) {
    unsigned long long w[kLL];
    uint32_t stale = 0;
#pragma unroll
    for (int k = 0; k < kLL; ++k) {
      const int i = base + k * kCThreads;
      if (i < n) w[k] = ld_ll(src + i);
    }
#pragma unroll
    for (int k = 0; k < kLL; ++k) {
      if (base + k * kCThreads < n && (uint32_t)(w[k] >> 32) != tag) stale |= 1u << k;
    }
    Poll poll;
    while (stale) {
      if (!poll.again(*c.p)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int k = 0; k < kLL; ++k) {
        if (stale & (1u << k)) w[k] = ld_ll(src + base + k * kCThreads);
      }
#pragma unroll
      for (int k = 0; k < kLL; ++k) {
        if ((stale & (1u << k)) && (uint32_t)(w[k] >> 32) == tag) stale &= ~(1u << k);
      }
    }
#pragma unroll
    for (int k = 0; k < kLL; ++k) {
      const int i = base + k * kCThreads;
      if (i < n) {
        const float v = __uint_as_float((uint32_t)w[k]);
        c.U[i] = v;
        ss += (double)v * (double)v;
      }
    }
  }
  if (norm_w == nullptr) return !stop_all(c, !ok);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  double* dred = reinterpret_cast<double*>(c.smem + kOffMisc + kMiscDred);
  if (c.lane == 0) dred[c.warp] = ss;
  cp_async_wait_all();
  if (stop_all(c, !ok)) return false;
  double tot = 0.0;
#pragma unroll
  for (int k = 0; k < kCWarps; ++k) tot += dred[k];
  const float scale = 1.0f / sqrtf((float)(tot / (double)n) + c.p->eps);
  for (int i = c.tid; i < n; i += kCThreads) c.U[i] = (c.U[i] * scale) * wn[i];  // this thread's words
  cbar();
  return true;
}

// ---- phase prologues: the input vector of a projection into U -------------

// The embedding row (written before the launch) into U by cp.async, every
// thread's 16-byte copies in flight together.
__device__ __forceinline__ void stage_async(Ctx& c, const float* src, int n) {
  for (int i = c.tid * 4; i < n; i += kCThreads * 4) cp_async_cg16(smem_u32(c.U + i), src + i);
  cp_async_wait_all();
  cbar();
}

// te_rmsnorm_f32 (c/src/ops.c:272-293) of the vector in U, in place: squares
// summed in double, scale = 1 / sqrtf((float)(sum / n) + eps), out = (x *
// scale) * w.
__device__ void rmsnorm_u(Ctx& c, const float* w) {
  const int H = c.p->hidden;
  double ss = 0.0;
  for (int i = c.tid * 4; i < H; i += kCThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(c.U + i);
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

// ---- projections ----------------------------------------------------------

// Block b of physical row r of a stage (transposed layout, see
// step_stage_bytes): sum (q - offset) * x over its 32 weights with exact
// weights (the code under the exponent of 2^23, minus 2^23 + offset), fp32
// products and sums in two chains, times the block's f16 scale (the
// reference's te_q4_0_dot_row / te_q8_0_dot_row products,
// c/src/ops.c:584-620).  Q4_0: quant byte j holds weight j (low nibble) and
// weight j + 16 (high nibble); Q8_0: 32 int8.  x: the block's 32 inputs
// (shared memory, 16-byte aligned).
template <int BB>
__device__ __forceinline__ float block_dot(const unsigned char* stage, uint32_t scale_bytes, int RS, int r, int b,
                                           const float* x) {
  constexpr float kOff = BB == 18 ? 8388616.0f : 8388736.0f;  // 2^23 + the quant offset (8 or 128)
  const uint64_t off2 = f2_pack(kOff, kOff);
  const float sc = __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(stage)[b * RS + r]));
  const uint4* quants = reinterpret_cast<const uint4*>(stage + scale_bytes);
  uint64_t da = 0, db = 0;  // two chains of two fp32 partial sums, all +0.0f
  auto quad = [&](uint64_t& d, uint32_t codes, const float* xq) {  // 4 codes, one per byte, with x[0..3]
    const float4 xv = *reinterpret_cast<const float4*>(xq);
    const uint64_t w01 = f2_sub(f2_pack(__uint_as_float(prmt(codes, 0x4B000000u, 0x7440u)),
                                        __uint_as_float(prmt(codes, 0x4B000000u, 0x7441u))), off2);
    const uint64_t w23 = f2_sub(f2_pack(__uint_as_float(prmt(codes, 0x4B000000u, 0x7442u)),
                                        __uint_as_float(prmt(codes, 0x4B000000u, 0x7443u))), off2);
    d = f2_fma(w01, f2_pack(xv.x, xv.y), d);
    d = f2_fma(w23, f2_pack(xv.z, xv.w), d);
  };
  if (BB == 18) {
    const uint4 q = quants[b * RS + r];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {  // quant bytes 4k .. 4k + 3
      quad(da, w[k] & 0x0f0f0f0fu, x + 4 * k);
      quad(db, (w[k] >> 4) & 0x0f0f0f0fu, x + 16 + 4 * k);
    }
  } else {
    const uint4 q0 = quants[(2 * b) * RS + r], q1 = quants[(2 * b + 1) * RS + r];
    const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) quad(k & 1 ? db : da, w[k] ^ 0x80808080u, x + 4 * k);
  }
  float d0, d1;
  f2_unpack(f2_add(da, db), d0, d1);
  return sc * (d0 + d1);
}

// Blocks b of physical rows r0 and r1 of a stage together (as block_dot,
// each input quad loaded once for both rows).
template <int BB>
__device__ __forceinline__ void block_dot2(const unsigned char* stage, uint32_t scale_bytes, int RS, int r0, int r1,
                                           int b, const float* x, float& out0, float& out1) {
  constexpr float kOff = BB == 18 ? 8388616.0f : 8388736.0f;  // 2^23 + the quant offset (8 or 128)
  const uint64_t off2 = f2_pack(kOff, kOff);
  const uint16_t* scales = reinterpret_cast<const uint16_t*>(stage);
  const float sc0 = __half2float(__ushort_as_half(scales[b * RS + r0]));
  const float sc1 = __half2float(__ushort_as_half(scales[b * RS + r1]));
  const uint4* quants = reinterpret_cast<const uint4*>(stage + scale_bytes);
  uint64_t a0 = 0, b0 = 0, a1 = 0, b1 = 0;  // two chains per row, all +0.0f
  auto quad2 = [&](uint64_t& d0, uint64_t& d1, uint32_t c0, uint32_t c1, const float* xq) {
    const float4 xv = *reinterpret_cast<const float4*>(xq);
    const uint64_t x01 = f2_pack(xv.x, xv.y), x23 = f2_pack(xv.z, xv.w);
    d0 = f2_fma(f2_sub(f2_pack(__uint_as_float(prmt(c0, 0x4B000000u, 0x7440u)),
                               __uint_as_float(prmt(c0, 0x4B000000u, 0x7441u))), off2), x01, d0);
    d0 = f2_fma(f2_sub(f2_pack(__uint_as_float(prmt(c0, 0x4B000000u, 0x7442u)),
                               __uint_as_float(prmt(c0, 0x4B000000u, 0x7443u))), off2), x23, d0);
    d1 = f2_fma(f2_sub(f2_pack(__uint_as_float(prmt(c1, 0x4B000000u, 0x7440u)),
                               __uint_as_float(prmt(c1, 0x4B000000u, 0x7441u))), off2), x01, d1);
    d1 = f2_fma(f2_sub(f2_pack(__uint_as_float(prmt(c1, 0x4B000000u, 0x7442u)),
                               __uint_as_float(prmt(c1, 0x4B000000u, 0x7443u))), off2), x23, d1);
  };
  if (BB == 18) {
    const uint4 q0 = quants[b * RS + r0], q1 = quants[b * RS + r1];
    const uint32_t w0[4] = {q0.x, q0.y, q0.z, q0.w}, w1[4] = {q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      quad2(a0, a1, w0[k] & 0x0f0f0f0fu, w1[k] & 0x0f0f0f0fu, x + 4 * k);
      quad2(b0, b1, (w0[k] >> 4) & 0x0f0f0f0fu, (w1[k] >> 4) & 0x0f0f0f0fu, x + 16 + 4 * k);
    }
  } else {
    const uint4 q00 = quants[(2 * b) * RS + r0], q01 = quants[(2 * b + 1) * RS + r0];
    const uint4 q10 = quants[(2 * b) * RS + r1], q11 = quants[(2 * b + 1) * RS + r1];
    const uint32_t w0[8] = {q00.x, q00.y, q00.z, q00.w, q01.x, q01.y, q01.z, q01.w};
    const uint32_t w1[8] = {q10.x, q10.y, q10.z, q10.w, q11.x, q11.y, q11.z, q11.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k & 1) {
        quad2(b0, b1, w0[k] ^ 0x80808080u, w1[k] ^ 0x80808080u, x + 4 * k);
      } else {
        quad2(a0, a1, w0[k] ^ 0x80808080u, w1[k] ^ 0x80808080u, x + 4 * k);
      }
    }
  }
  float d0, d1, e0, e1;
  f2_unpack(f2_add(a0, b0), d0, d1);
  f2_unpack(f2_add(a1, b1), e0, e1);
  out0 = sc0 * (d0 + d1);
  out1 = sc1 * (e0 + e1);
}

// Partial dot products of a stage's R (<= 64) rows into red[row][warp]:
// rows go across lanes (RT = R rounded up to a power of two lanes per group
// of K = 32 / RT lanes), and a row's blocks are dealt to its kCWarps * K
// (warp, lane group) units, so each lane sums whole blocks of one row,
// independent of each other, and a row's K lanes meet by shuffles.  With the
// transposed stage layout the lanes of a warp read consecutive 16-byte
// chunks (no bank conflicts) and share each input load (a broadcast).
template <int BB>
__device__ void stage_rows(const unsigned char* stage, int R, int nb, const float* xin, float* red, int warp,
                           int lane) {
  const uint32_t scale_bytes = step_scale_bytes(R, nb);
  if (R > 32) {  // two rows per lane, r and r + half, sharing each input load
    const int half = (R + 1) >> 1;
    const int r1 = lane + half;
    const bool v1 = r1 < R;
    float acc0 = 0.f, acc1 = 0.f;
    if (lane < half) {
#pragma unroll 1
      for (int b = warp; b < nb; b += kCWarps) {
        float o0, o1;
        block_dot2<BB>(stage, scale_bytes, R, lane, v1 ? r1 : lane, b, xin + b * 32, o0, o1);
        acc0 += o0;
        acc1 += o1;
      }
      red[lane * kCWarps + warp] = acc0;
      if (v1) red[r1 * kCWarps + warp] = acc1;
    }
    return;
  }
  int RT = 1;
  while (RT < R) RT <<= 1;
  const int K = 32 / RT;
  const int r = lane & (RT - 1), k = lane / RT;
  const int units = kCWarps * K;
  float acc = 0.f;
  if (r < R) {
#pragma unroll 2
    for (int b = warp * K + k; b < nb; b += units) acc += block_dot<BB>(stage, scale_bytes, R, r, b, xin + b * 32);
  }
  for (int o = RT; o < 32; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (k == 0 && r < R) red[r * kCWarps + warp] = acc;
}

// One projection phase over this CTA's rows: dot, or own[row] + dot (fp32
// add: the residual add after the output and down projections);
// with `best` also the running first-maximum (value, row) of the outputs.
// For the gate/up matrix (m.pair) a stage holds R gate rows then the same R
// up rows, and y[row] = SwiGLU(gate, up) = gate / (1 + expf(-gate)) * up
// (te_swiglu_f32, c/src/ops.c:397-406): the down projection's input.
// Where a projection's rows go: tagged words for other CTAs (ll, tag), plain
// floats (plain), and/or this CTA's residual rows (own: x[row] = own + dot,
// kept in shared memory by the CTA that owns the row in both residual
// projections).
struct Out {
  unsigned long long* ll;
  uint32_t tag;
  float* plain;
  float* own;
};

__device__ bool gemv_phase(Ctx& c, int kind, const Out& o, float* best_v, int* best_i) {
  const StepParams& p = *c.p;
  const StepMat m = p.mat[kind];  // read once per phase
  int r0;
  const int n = step_cta_rows(m, c.b, r0);
  const int ns = step_n_stages(n, m.rps);
  const int nb = m.cols / 32;
  const int q = ns > 0 ? n / ns : 0, rem = n - q * ns;  // step_stage_lo, incrementally
  const uint32_t cap = (uint32_t)p.ring_bytes;
  int lo = 0;
  for (int s = 0; s < ns; lo += q + (s < rem ? 1 : 0), ++s) {
    const int R = q + (s < rem ? 1 : 0);
    const int RS = m.pair ? 2 * R : R;  // rows in the stage
    const uint32_t slot = c.stage & (kNQ - 1u);
    const uint32_t off = ring_place(c.head, step_stage_bytes(RS, nb, m.block_bytes), cap);
    const bool ok = mbar_wait_warp(&c.full[slot], (c.stage / kNQ) & 1u);
    float* red = c.red + (c.stage & 1u) * kRedFloats;
    if (ok) {
      const unsigned char* base = c.ring + off;
      if (m.block_bytes == 18) {
        stage_rows<18>(base, RS, nb, c.U, red, c.warp, c.lane);
      } else {
        stage_rows<34>(base, RS, nb, c.U, red, c.warp, c.lane);
      }
    }
    __syncwarp();
    if (c.lane == 0) mbar_arrive(&c.empty[slot]);  // this warp is done with the slot
    ++c.stage;
    if (!ok) set_error(p.error, 61);
    if (stop_all(c, !ok)) return false;  // also: the stage's partial sums are complete
    // the epilogue runs on the last warp, which has the fewest blocks (blocks go to the low warps first)
    for (int et = c.tid - (kCThreads - 32); et >= 0 && et < R; et += 32) {
      float sum = red[et * kCWarps];
#pragma unroll
      for (int k = 1; k < kCWarps; ++k) sum += red[et * kCWarps + k];
      const int row = r0 + lo + et;
      if (m.pair) {
        float up = red[(R + et) * kCWarps];
#pragma unroll
        for (int k = 1; k < kCWarps; ++k) up += red[(R + et) * kCWarps + k];
        sum = silu(sum) * up;
      }
      if (o.own) {
        sum = __fadd_rn(o.own[lo + et], sum);
        o.own[lo + et] = sum;
      }
      if (o.ll) st_ll(o.ll + row, sum, o.tag);
      if (o.plain) o.plain[row] = sum;
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
__device__ bool attention_item(Ctx& c, int layer, int g, int ch, int nch) {
  const StepParams& p = *c.p;
  constexpr int half = HD / 2;
  constexpr int DPL = HD / 32;  // dims per lane in P.V
  const int Gq = p.group;
  float* qs = c.U;                                   // [kMaxGroup][HD]
  float* sc = qs + kMaxGroup * HD;                   // [kMaxGroup][kChunk]
  float* ml = sc + kMaxGroup * kChunk;               // [kMaxGroup][2]
  int* rowid = reinterpret_cast<int*>(ml + 2 * kMaxGroup);  // [kChunk]
  uint16_t* vs = reinterpret_cast<uint16_t*>(rowid + kChunk);  // [kChunk][HD] f16: the chunk's V rows
  // [kChunk][HD] f16: the chunk's K rows, 16-byte chunk j of token t at j ^ (t & 7)
  uint16_t* ks = vs + kChunk * HD;
  const float* cosr = p.rope_cos + (size_t)p.rope_pos * half;
  const float* sinr = p.rope_sin + (size_t)p.rope_pos * half;
  const int QH = p.heads * HD;
  const int KV = p.kv_heads * HD;

  const int t0 = ch * kChunk;
  const int t1 = min(p.n_tokens, t0 + kChunk);
  const int nt = t1 - t0;
  const bool with_new = t1 == p.n_tokens;  // this chunk holds the new token
  const size_t new_row = cache_row(p, layer, g, p.n_tokens - 1);
  const size_t kvb = ((size_t)layer * p.kv_heads + g) * HD;
  // the chunk's cached K and V rows into shared memory by cp.async (16 bytes a
  // copy), in flight while this CTA waits for the step's q, k and v
  const int n_old = with_new ? nt - 1 : nt;
  for (int e = c.tid; e < n_old * (HD / 8); e += kCThreads) {
    const int t = e / (HD / 8), d8 = e - t * (HD / 8);
    const size_t row = cache_row(p, layer, g, t0 + t);
    cp_async_cg16(smem_u32(vs + t * HD + d8 * 8), p.v_pool + row * HD + d8 * 8);
    cp_async_cg16(smem_u32(ks + t * HD + ((d8 ^ (t & 7)) * 8)), p.k_pool + row * HD + d8 * 8);
  }
  const int t_new = nt - 1;  // the new token's index in the chunk (with_new)
  auto ks_at = [&](int t, int d) { return ks + t * HD + (((d >> 3) ^ (t & 7)) << 3) + (d & 7); };
  // one pass over the item's inputs, all loads of an element issued together:
  // e < Gq * half: query pair (h, d); then, with the new token, its k pairs and v values
  const uint32_t tq = tag_of(c, layer, 0);
  const int n_in = Gq * half + (with_new ? half + HD : 0);
  bool ok = true;
  for (int e = c.tid; e < n_in; e += kCThreads) {
    if (e < Gq * half + half) {
      const bool isq = e < Gq * half;
      const int h = isq ? e / half : 0;
      const int d = isq ? e - h * half : e - Gq * half;
      const unsigned long long* src = isq ? p.ll_qkv + (g * Gq + h) * HD : p.ll_qkv + QH + g * HD;
      const float* bias = isq ? (p.q_bias ? p.q_bias + ((size_t)layer * p.heads + g * Gq + h) * HD : nullptr)
                              : (p.k_bias ? p.k_bias + kvb : nullptr);
      float a, bb;
      ok = ll_get2(p, src + d, src + d + half, tq, a, bb) && ok;
      if (bias) {
        a = __fadd_rn(a, __ldg(bias + d));
        bb = __fadd_rn(bb, __ldg(bias + d + half));
      }
      const float cs = __ldg(cosr + d), sn = __ldg(sinr + d);
      const float lo = rope_lo(a, bb, cs, sn), hi = rope_hi(a, bb, cs, sn);
      if (isq) {
        qs[h * HD + d] = lo;
        qs[h * HD + d + half] = hi;
      } else {  // the new k, rotated and rounded to f16 (RNE), into the cache and the staged rows
        const uint16_t klo = __half_as_ushort(__float2half_rn(lo)), khi = __half_as_ushort(__float2half_rn(hi));
        p.k_pool[new_row * HD + d] = klo;
        p.k_pool[new_row * HD + d + half] = khi;
        *ks_at(t_new, d) = klo;
        *ks_at(t_new, d + half) = khi;
      }
    } else {
      const int d = e - Gq * half - half;
      float v, unused;
      ok = ll_get2(p, p.ll_qkv + QH + KV + g * HD + d, p.ll_qkv + QH + KV + g * HD + d, tq, v, unused) && ok;
      if (p.v_bias) v = __fadd_rn(v, __ldg(p.v_bias + kvb + d));
      const uint16_t vh = __half_as_ushort(__float2half_rn(v));
      p.v_pool[new_row * HD + d] = vh;
      vs[t_new * HD + d] = vh;
    }
  }
  cp_async_wait_all();
  if (stop_all(c, !ok)) return false;  // queries and the chunk's K and V rows are in place

  // scores: one (head, token) pair per thread, consecutive threads on consecutive tokens
  for (int e = c.tid; e < Gq * nt; e += kCThreads) {
    const int h = e / nt, t = e - h * nt;
    const uint16_t* kr = ks + t * HD;
    const float* qh = qs + h * HD;
    float dot = 0.f;
#pragma unroll 4
    for (int d8 = 0; d8 < HD / 8; ++d8) {
      float kv[8];
      unpack8(*reinterpret_cast<const uint4*>(kr + ((d8 ^ (t & 7)) << 3)), kv);
      const float4 q0 = *reinterpret_cast<const float4*>(qh + d8 * 8);
      const float4 q1 = *reinterpret_cast<const float4*>(qh + d8 * 8 + 4);
      dot = fmaf(q0.x, kv[0], dot); dot = fmaf(q0.y, kv[1], dot); dot = fmaf(q0.z, kv[2], dot);
      dot = fmaf(q0.w, kv[3], dot); dot = fmaf(q1.x, kv[4], dot); dot = fmaf(q1.y, kv[5], dot);
      dot = fmaf(q1.z, kv[6], dot); dot = fmaf(q1.w, kv[7], dot);
    }
    sc[h * kChunk + t] = dot * p.scale_log2;
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
    for (int t = 0; t < nt; ++t) {  // P.V from shared memory: lane -> DPL dims of the row
      const float pw = sc[h * kChunk + t];
      const uint16_t* vr = vs + t * HD + c.lane * DPL;
      if constexpr (DPL == 2) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(vr));
        acc[0] = fmaf(pw, f.x, acc[0]);
        acc[1] = fmaf(pw, f.y, acc[1]);
      } else {
        const uint2 u = *reinterpret_cast<const uint2*>(vr);
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
      unsigned long long* o = p.ll_attn + (size_t)(g * Gq + h) * HD + c.lane * DPL;
#pragma unroll
      for (int i = 0; i < DPL; ++i) st_ll(o + i, acc[i] * inv, tag_of(c, layer, 1));
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
    return true;
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
      unsigned long long* o = p.ll_attn + (size_t)(g * Gq + h) * HD + c.lane * DPL;
#pragma unroll
      for (int i = 0; i < DPL; ++i) st_ll(o + i, acc[i] * inv, tag_of(c, layer, 1));
    }
    if (c.tid == 0) atomicExch(&p.sync[4 + g], 0u);
  }
  cbar();
  return true;
}

template <int HD>
__device__ bool attention_phase(Ctx& c, int layer) {
  const StepParams& p = *c.p;
  const int nch = (p.n_tokens + kChunk - 1) / kChunk;
  const int items = p.kv_heads * nch;
  for (int it = c.b; it < items; it += c.G) {
    if (!attention_item<HD>(c, layer, it / nch, it % nch, nch)) return false;
  }
  return true;
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
  const int H = p.hidden;
  int r0;
  // this CTA's rows of x (the same rows in the output and down projections):
  // the residual stream's rows it updates, starting from the embedding
  float* xown = reinterpret_cast<float*>(c.smem + kOffMisc + kMiscXown);
  const int nx = step_cta_rows(p.mat[kStepO], c.b, r0);
  for (int i = c.tid; i < nx; i += kCThreads) xown[i] = ldcg(emb_row + r0 + i);
  cbar();
  const bool a_rows = step_cta_rows(p.mat[kStepQKV], c.b, r0) > 0;
  const bool gu_rows = step_cta_rows(p.mat[kStepGU], c.b, r0) > 0;
  for (int l = 0; l < p.layers; ++l) {
    if (a_rows) {  // A: q|k|v = W_qkv RMSNorm(x)
      if (l == 0) {
        stage_async(c, emb_row, H);
        rmsnorm_u(c, p.attn_norm);
      } else if (!ll_stage(c, p.ll_x[1], H, tag_of(c, l - 1, 4), p.attn_norm + (size_t)l * H)) {
        return;
      }
      if (!gemv_phase(c, kStepQKV, Out{p.ll_qkv, tag_of(c, l, 0), nullptr, nullptr}, nullptr, nullptr)) return;
    }
    if (p.head_dim == 64 ? !attention_phase<64>(c, l) : !attention_phase<128>(c, l)) return;  // B
    if (nx > 0) {  // C: x += W_o attn
      if (!ll_stage(c, p.ll_attn, H, tag_of(c, l, 1))) return;
      if (!gemv_phase(c, kStepO, Out{p.ll_x[0], tag_of(c, l, 2), nullptr, xown}, nullptr, nullptr)) return;
    }
    if (gu_rows) {  // D: h = SwiGLU(W_gate RMSNorm(x), W_up RMSNorm(x))
      if (!ll_stage(c, p.ll_x[0], H, tag_of(c, l, 2), p.ffn_norm + (size_t)l * H)) return;
      if (!gemv_phase(c, kStepGU, Out{p.ll_h, tag_of(c, l, 3), nullptr, nullptr}, nullptr, nullptr)) return;
    }
    if (nx > 0) {  // E: x += W_down h (the last layer's x also as plain floats: the hidden state)
      if (!ll_stage(c, p.ll_h, p.ffn, tag_of(c, l, 3))) return;
      if (!gemv_phase(c, kStepDown, Out{p.ll_x[1], tag_of(c, l, 4), l == p.layers - 1 ? p.x : nullptr, xown},
                      nullptr, nullptr)) {
        return;
      }
    }
  }
  if (!p.head) return;
  float bv = -INFINITY;
  int bi = INT_MAX;
  if (step_cta_rows(p.mat[kStepHead], c.b, r0) > 0) {
    if (!ll_stage(c, p.ll_x[1], H, tag_of(c, p.layers - 1, 4), p.out_norm)) return;
    if (!gemv_phase(c, kStepHead, Out{nullptr, 0u, p.logits, nullptr}, &bv, &bi)) return;
  }
  argmax_finish(c, bv, bi);  // every CTA hands in a candidate
}

// One lane: streams this CTA's packed weights through the byte ring in
// consumption order.  A stage is issued once its descriptor's previous stage
// and every in-flight stage its bytes overlap have been released by all
// consumer warps (they release in order).
__device__ void producer(const StepParams& p, unsigned char* ring, uint64_t* full, uint64_t* empty,
                         uint32_t* offs, uint32_t* ends, volatile int* s_abort) {
  const int b = blockIdx.x;
  const unsigned char* src = p.wpack + p.cta_off[b];
  const uint32_t cap = (uint32_t)p.ring_bytes;
  uint32_t i = 0, tail = 0, head = 0;
  bool ok = true;
  auto clash = [&](uint32_t off, uint32_t bytes) {
    for (uint32_t j = tail; j < i; ++j) {
      const uint32_t q = j & (kNQ - 1u);
      if (offs[q] < off + bytes && off < ends[q]) return true;
    }
    return false;
  };
  auto put = [&](uint32_t bytes) {
    const uint32_t off = ring_place(head, bytes, cap);
    while (tail < i && (i - tail >= kNQ || clash(off, bytes))) {
      const uint32_t q = tail & (kNQ - 1u), par = (tail / kNQ) & 1u;
      if (!mbar_try_wait(&empty[q], par)) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t n = 0;
        while (!mbar_try_wait(&empty[q], par)) {
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
      ++tail;
    }
    const uint32_t q = i & (kNQ - 1u);
    offs[q] = off;
    ends[q] = off + bytes;
    mbar_arrive_expect_tx(&full[q], bytes);
    bulk_load(ring + off, src, bytes, &full[q]);
    src += bytes;
    ++i;
  };
  auto stream = [&](int kind) {
    const StepMat& m = p.mat[kind];
    int r0;
    const int n = step_cta_rows(m, b, r0);
    const int ns = step_n_stages(n, m.rps);
    for (int s = 0; s < ns && ok; ++s) {
      const int rows = step_stage_lo(s + 1, n, ns) - step_stage_lo(s, n, ns);
      put(step_stage_bytes(m.pair ? 2 * rows : rows, m.cols / 32, m.block_bytes));
    }
  };
  for (int l = 0; l < p.layers && ok; ++l) {
    for (int k = kStepQKV; k <= kStepDown && ok; ++k) stream(k);
  }
  if (p.head && ok) stream(kStepHead);
  // No copy may still be landing when the CTA exits (the consumers may have
  // given up before using the last stages): wait for the newest use of every
  // descriptor (already complete in a normal run).
  for (uint32_t j = i > kNQ ? i - kNQ : 0; j < i; ++j) mbar_wait(&full[j & (kNQ - 1u)], (j / kNQ) & 1u);
}

__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffFull);
  uint64_t* empty = reinterpret_cast<uint64_t*>(smem + kOffEmpty);
  volatile int* s_abort = reinterpret_cast<volatile int*>(smem + kOffMisc + kMiscAbort);
  unsigned char* ring = smem + kOffUnion + p.union_bytes;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (uint32_t q = 0; q < kNQ; ++q) {
      mbar_init(&full[q], 1);
      mbar_init(&empty[q], kCWarps);
    }
    fence_mbarrier_init();
    *s_abort = 0;
  }
  __syncthreads();
  if (warp == kCWarps) {
    uint32_t* rr = reinterpret_cast<uint32_t*>(smem + kOffMisc + kMiscRing);
    if (lane == 0) producer(p, ring, full, empty, rr, rr + kNQ, s_abort);
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
    c.head = 0;
    c.epoch = ld_relaxed_gpu(&p.sync[3]);
    consumer(c);
    if (tid == 0) *s_abort = 1;  // done (or gave up): a producer still waiting for a slot stops
  }
  __syncthreads();
  if (tid == 0) {
    // the last CTA out clears the launch's counters and advances the epoch
    __threadfence();
    const uint32_t old = atomicAdd(&p.sync[1], 1u);
    if (old == gridDim.x - 1) {
      // every CTA read this launch's epoch before doing anything else
      atomicAdd(&p.sync[3], 1u);
      atomicExch(&p.sync[2], 0u);
      for (int g = 0; g < p.kv_heads; ++g) atomicExch(&p.sync[4 + g], 0u);
      atomicExch(&p.sync[1], 0u);
    }
  }
}

// One CTA per stage: every (block, row) of the stage's physical rows into the
// transposed layout (scale plane, then the 16-byte quant chunks).
__global__ void step_pack_kernel(const StepPackSeg* segs, int n, unsigned char* dst) {
  for (int s = blockIdx.x; s < n; s += gridDim.x) {
    const StepPackSeg sg = segs[s];
    const int R = sg.rows, nb = sg.nb, BB = sg.block_bytes;
    const int row_bytes = nb * BB;
    unsigned char* out = dst + sg.dst_off;
    const uint32_t scale_bytes = step_scale_bytes(R, nb);
    for (int e = threadIdx.x; e < R * nb; e += blockDim.x) {
      const int b = e / R, r = e - b * R;
      const unsigned char* src = r < sg.split ? static_cast<const unsigned char*>(sg.src0) + (size_t)r * row_bytes
                                              : static_cast<const unsigned char*>(sg.src1) +
                                                    (size_t)(r - sg.split) * row_bytes;
      const uint16_t* blk = reinterpret_cast<const uint16_t*>(src + (size_t)b * BB);
      reinterpret_cast<uint16_t*>(out)[b * R + r] = blk[0];
      if (BB == 18) {
        uint16_t* q = reinterpret_cast<uint16_t*>(out + scale_bytes + (size_t)(b * R + r) * 16);
        for (int i = 0; i < 8; ++i) q[i] = blk[1 + i];
      } else {
        uint16_t* q0 = reinterpret_cast<uint16_t*>(out + scale_bytes + (size_t)((2 * b) * R + r) * 16);
        uint16_t* q1 = reinterpret_cast<uint16_t*>(out + scale_bytes + (size_t)((2 * b + 1) * R + r) * 16);
        for (int i = 0; i < 8; ++i) {
          q0[i] = blk[1 + i];
          q1[i] = blk[9 + i];
        }
      }
    }
  }
}

}  // namespace

void plan_step_mat(StepMat& m, int rows, int cols, int block_bytes, int grid, int stage_max, int pair) {
  m.rows = rows;
  m.cols = cols;
  m.block_bytes = block_bytes;
  m.row_bytes = cols / 32 * block_bytes;
  m.pair = pair;
  m.rpc = (rows + grid - 1) / grid;
  const int per = pair ? 2 : 1;  // physical rows per row
  int rps = stage_max / (per * m.row_bytes);
  if (rps > kStepMaxStageRows / per) rps = kStepMaxStageRows / per;
  m.rps = rps < 1 ? 1 : rps;
}

int step_fixed_smem() { return kOffUnion; }

int step_smem_bytes(int ring_bytes, int union_bytes) { return kOffUnion + union_bytes + ring_bytes; }

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
