// RoPE kernels: the drop-in te_rope_f32, the fused RoPE(k) + f16 append into
// the paged cache, and the prefill query preparation.
//
// All rotations use the reference's exact fp32 expression shapes
//   lo = a*cos - b*sin,  hi = b*cos + a*sin     (c/src/ops.c:313-318,
//                                               c/src/qwen.c:2152-2157)
// with separately rounded products (no FMA contraction), on the host-built
// cos/sin table (c/src/qwen.c:531-539), so results are bit-identical to the
// CPU reference; the f16 store is round-to-nearest-even like Metal's half()
// (c/src/metal/metal_kernels.metal.inc:2422-2427).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "te_internal.h"

namespace te {
namespace {

__device__ __forceinline__ float rope_lo(float a, float b, float c, float s) {
  return __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
}
__device__ __forceinline__ float rope_hi(float a, float b, float c, float s) {
  return __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
}

__global__ void rope_rows_kernel(float* values, const float* cos_row, const float* sin_row, int heads,
                                 int head_dim) {
  const int half = head_dim / 2;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= heads * half) return;
  const int h = i / half, d = i % half;
  float* row = values + (size_t)h * head_dim;
  const float a = row[d], b = row[d + half];
  const float c = cos_row[d], s = sin_row[d];
  row[d] = rope_lo(a, b, c, s);
  row[d + half] = rope_hi(a, b, c, s);
}

// 8 consecutive values of an fp32 or f16 row as fp32.
__device__ __forceinline__ void load8(const void* base, size_t idx, int f16, float (&v)[8]) {
  if (f16) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(base) + idx);
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  return u;
}

// Rotates 8 pairs (d..d+7, d+half..d+half+7) in place with the reference expressions.
__device__ __forceinline__ void rope8(float (&lo)[8], float (&hi)[8], const float* cos_row, const float* sin_row, int d) {
  const float4 c0 = *reinterpret_cast<const float4*>(cos_row + d);
  const float4 c1 = *reinterpret_cast<const float4*>(cos_row + d + 4);
  const float4 s0 = *reinterpret_cast<const float4*>(sin_row + d);
  const float4 s1 = *reinterpret_cast<const float4*>(sin_row + d + 4);
  const float c[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float a = lo[i], b = hi[i];
    lo[i] = rope_lo(a, b, c[i], s[i]);
    hi[i] = rope_hi(a, b, c[i], s[i]);
  }
}

// One thread per (layer, token, kv head, group of 8 rotation pairs).
__global__ void append_rope_kernel(const AppendParams p) {
  const int half = p.head_dim / 2;
  const int groups = half / 8;
  const long long total = (long long)p.n_layers * p.n_tokens * p.kv_heads * groups;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % groups) * 8;
  long long r = i / groups;
  const int kvh = (int)(r % p.kv_heads);
  r /= p.kv_heads;
  const int t = (int)(r % p.n_tokens);
  const int ll = (int)(r / p.n_tokens);
  const size_t in_row = (((size_t)ll * p.n_tokens + t) * p.kv_heads + kvh) * p.head_dim;
  float klo[8], khi[8], vlo[8], vhi[8];
  load8(p.k, in_row + d, p.input_f16, klo);
  load8(p.k, in_row + d + half, p.input_f16, khi);
  load8(p.v, in_row + d, p.input_f16, vlo);
  load8(p.v, in_row + d + half, p.input_f16, vhi);
  if (p.rope) {
    const int pos = p.first_pos + t;
    rope8(klo, khi, p.rope_cos + (size_t)pos * half, p.rope_sin + (size_t)pos * half, d);
  }
  const int idx = p.first_index + t;
  const int page = p.page_row[idx / p.page_tokens];
  const int layer = p.layer_begin + ll;
  const size_t row = ((size_t)(layer * p.num_pages + page) * p.kv_heads + kvh) * p.page_tokens + (idx % p.page_tokens);
  uint16_t* kd = p.k_pool + row * p.head_dim;
  uint16_t* vd = p.v_pool + row * p.head_dim;
  *reinterpret_cast<uint4*>(kd + d) = pack8(klo);
  *reinterpret_cast<uint4*>(kd + d + half) = pack8(khi);
  *reinterpret_cast<uint4*>(vd + d) = pack8(vlo);
  *reinterpret_cast<uint4*>(vd + d + half) = pack8(vhi);
}

// q[n_layers][n_tokens][heads][hd] -> qh[n_layers][heads][n_tokens_padded][hd] (f16, rotated).
// Padding rows (t >= n_tokens) are written as zeros.
__global__ void q_prep_kernel(const QPrepParams p) {
  const int half = p.head_dim / 2;
  const int groups = half / 8;
  const long long total = (long long)p.n_layers * p.n_tokens_padded * p.heads * groups;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % groups) * 8;
  long long r = i / groups;
  const int h = (int)(r % p.heads);
  r /= p.heads;
  const int t = (int)(r % p.n_tokens_padded);
  const int ll = (int)(r / p.n_tokens_padded);
  float lo[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float hi[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (t < p.n_tokens) {
    const size_t in_row = (((size_t)ll * p.n_tokens + t) * p.heads + h) * p.head_dim;
    load8(p.q, in_row + d, p.input_f16, lo);
    load8(p.q, in_row + d + half, p.input_f16, hi);
    if (p.rope) {
      const int pos = p.first_pos + t;
      rope8(lo, hi, p.rope_cos + (size_t)pos * half, p.rope_sin + (size_t)pos * half, d);
    }
  }
  __half* o = p.qh + (((size_t)ll * p.heads + h) * p.n_tokens_padded + t) * p.head_dim;
  *reinterpret_cast<uint4*>(o + d) = pack8(lo);
  *reinterpret_cast<uint4*>(o + d + half) = pack8(hi);
}

}  // namespace

cudaError_t launch_rope_rows(float* values, const float* cos_row, const float* sin_row, int heads, int head_dim,
                             cudaStream_t s) {
  const int n = heads * (head_dim / 2);
  rope_rows_kernel<<<(n + 255) / 256, 256, 0, s>>>(values, cos_row, sin_row, heads, head_dim);
  return cudaGetLastError();
}

cudaError_t launch_append_rope(const AppendParams& p, cudaStream_t s) {
  const long long total = (long long)p.n_layers * p.n_tokens * p.kv_heads * (p.head_dim / 16);
  if (total == 0) return cudaSuccess;
  append_rope_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_q_prep(const QPrepParams& p, cudaStream_t s) {
  const long long total = (long long)p.n_layers * p.n_tokens_padded * p.heads * (p.head_dim / 16);
  if (total == 0) return cudaSuccess;
  q_prep_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace te
