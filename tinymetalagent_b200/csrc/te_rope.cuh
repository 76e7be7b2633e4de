// Device helpers for RoPE, bias and f16 conversion, shared by the append,
// query-preparation, decode and prefill kernels.
//
// All rotations use the reference's exact fp32 expression shapes
//   lo = a*cos - b*sin,  hi = b*cos + a*sin     (c/src/ops.c:313-318,
//                                               c/src/qwen.c:2152-2157)
// with separately rounded products (no FMA contraction), on the host-built
// cos/sin table (c/src/qwen.c:531-539), so results are bit-identical to the
// CPU reference; the f16 store is round-to-nearest-even like Metal's half()
// (c/src/metal/metal_kernels.metal.inc:2422-2427).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "te_internal.h"

namespace te {

__device__ __forceinline__ float rope_lo(float a, float b, float c, float s) {
  return __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
}
__device__ __forceinline__ float rope_hi(float a, float b, float c, float s) {
  return __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

// v[i] += b[i] for 8 consecutive fp32 bias values (the reference's te_add_f32,
// c/src/ops.c:408-416: one fp32 addition per element, rounded to nearest).
__device__ __forceinline__ void add_bias8(float (&v)[8], const float* b) {
  const float4 b0 = *reinterpret_cast<const float4*>(b);
  const float4 b1 = *reinterpret_cast<const float4*>(b + 4);
  v[0] = __fadd_rn(v[0], b0.x); v[1] = __fadd_rn(v[1], b0.y); v[2] = __fadd_rn(v[2], b0.z); v[3] = __fadd_rn(v[3], b0.w);
  v[4] = __fadd_rn(v[4], b1.x); v[5] = __fadd_rn(v[5], b1.y); v[6] = __fadd_rn(v[6], b1.z); v[7] = __fadd_rn(v[7], b1.w);
}

// Low part of x in a two-term f16 split: x = hi + lo with hi = f16(x) and lo
// = x - hi (exact in fp32), itself rounded to f16 for the tensor core.  The
// query enters the f16 MMA as hi and lo, so q.k keeps about 22 bits of the
// fp32 query instead of 11.
__device__ __forceinline__ float f16_residual(float x) { return x - __half2float(__float2half_rn(x)); }

__device__ __forceinline__ void f16_residual8(const float (&x)[8], float (&r)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) r[e] = f16_residual(x[e]);
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  return u;
}

// 8 f16 values (one 16-byte word) as fp32.
__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// 8 consecutive values of an fp32 or f16 row as fp32.
__device__ __forceinline__ void load8(const void* base, size_t idx, int f16, float (&v)[8]) {
  if (f16) {
    unpack8(*reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(base) + idx), v);
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

// cos/sin of rotation pairs d..d+7 at one position (two table rows).
__device__ __forceinline__ void load_cs8(const float* cos_row, const float* sin_row, int d, float (&c)[8],
                                         float (&s)[8]) {
  const float4 c0 = *reinterpret_cast<const float4*>(cos_row + d);
  const float4 c1 = *reinterpret_cast<const float4*>(cos_row + d + 4);
  const float4 s0 = *reinterpret_cast<const float4*>(sin_row + d);
  const float4 s1 = *reinterpret_cast<const float4*>(sin_row + d + 4);
  c[0] = c0.x; c[1] = c0.y; c[2] = c0.z; c[3] = c0.w; c[4] = c1.x; c[5] = c1.y; c[6] = c1.z; c[7] = c1.w;
  s[0] = s0.x; s[1] = s0.y; s[2] = s0.z; s[3] = s0.w; s[4] = s1.x; s[5] = s1.y; s[6] = s1.z; s[7] = s1.w;
}

// Rotates 8 pairs (lo[i], hi[i]) in place with the reference expressions.
__device__ __forceinline__ void rope8cs(float (&lo)[8], float (&hi)[8], const float (&c)[8], const float (&s)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = lo[i], b = hi[i];
    lo[i] = rope_lo(a, b, c[i], s[i]);
    hi[i] = rope_hi(a, b, c[i], s[i]);
  }
}

// Rotates 8 pairs (d..d+7, d+half..d+half+7) in place, reading their cos/sin.
__device__ __forceinline__ void rope8(float (&lo)[8], float (&hi)[8], const float* cos_row, const float* sin_row, int d) {
  float c[8], s[8];
  load_cs8(cos_row, sin_row, d, c, s);
  rope8cs(lo, hi, c, s);
}

// Stores dims [d, d+8) and [d+half, d+half+8) of the query row whose unsplit
// offset is `row` (elements, [..][heads][hd] layout): as f16 there, or with
// p.split as the hi row 2r and the lo row 2r + 1 of [..][heads][2][hd].
template <int HD>
__device__ __forceinline__ void store_q8(const QPrepParams& p, size_t row, int d, const float (&lo)[8],
                                         const float (&hi)[8]) {
  constexpr int half = HD / 2;
  if (!p.split) {
    *reinterpret_cast<uint4*>(p.qh + row + d) = pack8(lo);
    *reinterpret_cast<uint4*>(p.qh + row + d + half) = pack8(hi);
    return;
  }
  float rl[8], rh[8];
  f16_residual8(lo, rl);
  f16_residual8(hi, rh);
  __half* hrow = p.qh + 2 * row;
  *reinterpret_cast<uint4*>(hrow + d) = pack8(lo);
  *reinterpret_cast<uint4*>(hrow + d + half) = pack8(hi);
  *reinterpret_cast<uint4*>(hrow + HD + d) = pack8(rl);
  *reinterpret_cast<uint4*>(hrow + HD + d + half) = pack8(rh);
}

}  // namespace te
