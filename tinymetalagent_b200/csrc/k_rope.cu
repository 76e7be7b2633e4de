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

__device__ __forceinline__ float load_in(const void* base, size_t idx, int f16) {
  return f16 ? __half2float(reinterpret_cast<const __half*>(base)[idx]) : reinterpret_cast<const float*>(base)[idx];
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

// One thread per (layer, token, kv head, rotation pair).
__global__ void append_rope_kernel(const AppendParams p) {
  const int half = p.head_dim / 2;
  const long long total = (long long)p.n_layers * p.n_tokens * p.kv_heads * half;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % half);
  long long r = i / half;
  const int kvh = (int)(r % p.kv_heads);
  r /= p.kv_heads;
  const int t = (int)(r % p.n_tokens);
  const int ll = (int)(r / p.n_tokens);
  const size_t in_row = (((size_t)ll * p.n_tokens + t) * p.kv_heads + kvh) * p.head_dim;
  const float a = load_in(p.k, in_row + d, p.input_f16);
  const float b = load_in(p.k, in_row + d + half, p.input_f16);
  float lo = a, hi = b;
  if (p.rope) {
    const int pos = p.first_pos + t;
    const float c = p.rope_cos[(size_t)pos * half + d];
    const float s = p.rope_sin[(size_t)pos * half + d];
    lo = rope_lo(a, b, c, s);
    hi = rope_hi(a, b, c, s);
  }
  const int idx = p.first_index + t;
  const int page = p.page_row[idx / p.page_tokens];
  const int layer = p.layer_begin + ll;
  const size_t row = ((size_t)(layer * p.num_pages + page) * p.kv_heads + kvh) * p.page_tokens + (idx % p.page_tokens);
  uint16_t* kd = p.k_pool + row * p.head_dim;
  uint16_t* vd = p.v_pool + row * p.head_dim;
  kd[d] = __half_as_ushort(__float2half_rn(lo));
  kd[d + half] = __half_as_ushort(__float2half_rn(hi));
  vd[d] = __half_as_ushort(__float2half_rn(load_in(p.v, in_row + d, p.input_f16)));
  vd[d + half] = __half_as_ushort(__float2half_rn(load_in(p.v, in_row + d + half, p.input_f16)));
}

// q[n_layers][n_tokens][heads][hd] -> qh[n_layers][heads][n_tokens_padded][hd] (f16, rotated).
// Padding rows (t >= n_tokens) are written as zeros.
__global__ void q_prep_kernel(const QPrepParams p) {
  const int half = p.head_dim / 2;
  const long long total = (long long)p.n_layers * p.n_tokens_padded * p.heads * half;
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int d = (int)(i % half);
  long long r = i / half;
  const int h = (int)(r % p.heads);
  r /= p.heads;
  const int t = (int)(r % p.n_tokens_padded);
  const int ll = (int)(r / p.n_tokens_padded);
  float lo = 0.f, hi = 0.f;
  if (t < p.n_tokens) {
    const size_t in_row = (((size_t)ll * p.n_tokens + t) * p.heads + h) * p.head_dim;
    const float a = load_in(p.q, in_row + d, p.input_f16);
    const float b = load_in(p.q, in_row + d + half, p.input_f16);
    lo = a;
    hi = b;
    if (p.rope) {
      const int pos = p.first_pos + t;
      const float c = p.rope_cos[(size_t)pos * half + d];
      const float s = p.rope_sin[(size_t)pos * half + d];
      lo = rope_lo(a, b, c, s);
      hi = rope_hi(a, b, c, s);
    }
  }
  __half* o = p.qh + (((size_t)ll * p.heads + h) * p.n_tokens_padded + t) * p.head_dim;
  o[d] = __float2half_rn(lo);
  o[d + half] = __float2half_rn(hi);
}

}  // namespace

cudaError_t launch_rope_rows(float* values, const float* cos_row, const float* sin_row, int heads, int head_dim,
                             cudaStream_t s) {
  const int n = heads * (head_dim / 2);
  rope_rows_kernel<<<(n + 255) / 256, 256, 0, s>>>(values, cos_row, sin_row, heads, head_dim);
  return cudaGetLastError();
}

cudaError_t launch_append_rope(const AppendParams& p, cudaStream_t s) {
  const long long total = (long long)p.n_layers * p.n_tokens * p.kv_heads * (p.head_dim / 2);
  if (total == 0) return cudaSuccess;
  append_rope_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_q_prep(const QPrepParams& p, cudaStream_t s) {
  const long long total = (long long)p.n_layers * p.n_tokens_padded * p.heads * (p.head_dim / 2);
  if (total == 0) return cudaSuccess;
  q_prep_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace te
