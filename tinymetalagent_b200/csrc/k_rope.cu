// RoPE kernels: the drop-in te_rope_f32, the fused RoPE(k) + f16 append into
// the paged cache, and the prefill query preparation.  Rotation, bias and f16
// conversion arithmetic (bit-identical to the CPU reference) is in
// te_rope.cuh.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "te_internal.h"
#include "te_ptx.cuh"
#include "te_rope.cuh"

namespace te {
namespace {

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

// One thread per (token, kv head, group of 8 rotation pairs); grid.y = layer.
// 32-bit index arithmetic with a compile-time group count.
template <int HD>
__global__ void append_rope_kernel(const AppendParams p) {
  constexpr int half = HD / 2;
  constexpr int groups = half / 8;
  const int ll = blockIdx.y;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (uint32_t)p.n_tokens * (uint32_t)p.kv_heads * groups) return;
  const int d = (int)(i % groups) * 8;
  const uint32_t r = i / groups;
  const int kvh = (int)(r % (uint32_t)p.kv_heads);
  const int t = (int)(r / (uint32_t)p.kv_heads);
  const size_t in_row = (((size_t)ll * p.n_tokens + t) * p.kv_heads + kvh) * HD;
  float klo[8], khi[8], vlo[8], vhi[8];
  load8(p.k, in_row + d, p.input_f16, klo);
  load8(p.k, in_row + d + half, p.input_f16, khi);
  load8(p.v, in_row + d, p.input_f16, vlo);
  load8(p.v, in_row + d + half, p.input_f16, vhi);
  if (p.k_bias) {
    const size_t brow = ((size_t)(p.layer_begin + ll) * p.kv_heads + kvh) * HD;
    add_bias8(klo, p.k_bias + brow + d);
    add_bias8(khi, p.k_bias + brow + d + half);
    add_bias8(vlo, p.v_bias + brow + d);
    add_bias8(vhi, p.v_bias + brow + d + half);
  }
  if (p.rope) {
    const int pos = p.first_pos + t;
    rope8(klo, khi, p.rope_cos + (size_t)pos * half, p.rope_sin + (size_t)pos * half, d);
  }
  const int idx = p.first_index + t;
  const int page = p.page_row[idx / p.page_tokens];
  const int layer = p.layer_begin + ll;
  const size_t row = ((size_t)(layer * p.num_pages + page) * p.kv_heads + kvh) * p.page_tokens + (idx % p.page_tokens);
  uint16_t* kd = p.k_pool + row * HD;
  uint16_t* vd = p.v_pool + row * HD;
  *reinterpret_cast<uint4*>(kd + d) = pack8(klo);
  *reinterpret_cast<uint4*>(kd + d + half) = pack8(khi);
  *reinterpret_cast<uint4*>(vd + d) = pack8(vlo);
  *reinterpret_cast<uint4*>(vd + d + half) = pack8(vhi);
}

// Low parts of a two-term f16 split: lo = f16(x - f16(x)), x - f16(x) exact in fp32.
// Query rows of one token and head: f16 in the same layout, rotated unless
// RoPE is off.
template <int HD>
__device__ __forceinline__ void q_prep_row(const QPrepParams& p, size_t row, int t, int d, const float* bias_row) {
  constexpr int half = HD / 2;
  float lo[8], hi[8];
  load8(p.q, row + d, p.input_f16, lo);
  load8(p.q, row + d + half, p.input_f16, hi);
  if (bias_row) {
    add_bias8(lo, bias_row + d);
    add_bias8(hi, bias_row + d + half);
  }
  if (p.rope) {
    const int pos = p.first_pos + t;
    rope8(lo, hi, p.rope_cos + (size_t)pos * half, p.rope_sin + (size_t)pos * half, d);
  }
  store_q8<HD>(p, row, d, lo, hi);
}

// q[n_layers][n_tokens][heads][hd] -> f16 qh (same layout).  One thread per
// (token, head, group of 8 rotation pairs); grid.y = layer.
template <int HD>
__global__ void q_prep_kernel(const QPrepParams p) {
  constexpr int groups = HD / 16;
  const int ll = blockIdx.y;
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (uint32_t)p.n_tokens * (uint32_t)p.heads * groups) return;
  const uint32_t r = i / groups;
  const float* bias_row =
      p.q_bias ? p.q_bias + ((size_t)(p.layer_begin + ll) * p.heads + (r % (uint32_t)p.heads)) * HD : nullptr;
  q_prep_row<HD>(p, ((size_t)ll * p.n_tokens * p.heads + r) * HD, (int)(r / (uint32_t)p.heads), (int)(i % groups) * 8,
                 bias_row);
}

// A prefill call's inputs in one pass, streamed through shared memory: each
// chunk of kPrepTokens tokens of one layer (its query rows when with_q, its
// K and V rows -- contiguous blocks of the inputs) arrives by bulk copy in a
// ring of kPrepStages stages, so the whole ring's bytes are in flight while
// the warps work on landed chunks.  Warp w handles token w of a chunk: lane
// group g = lane % kGroups owns dims [8g, 8g+8) and their rotation partners
// (the token's cos/sin values are read once per lane) and walks the rows
// lane / kGroups + k * kRowLanes.  Results go straight to global memory.
constexpr int kPrepTokens = 8;
constexpr int kPrepThreads = 32 * kPrepTokens;

template <int HD, bool kF16In>
struct PrepCfg {
  static constexpr int kEl = kF16In ? 2 : 4;
};

template <int HD, bool kF16In>
__global__ void __launch_bounds__(kPrepThreads, 2) prefill_prep_kernel(const AppendParams a, const QPrepParams q,
                                                                      int with_q, int q_stride, int stage_bytes,
                                                                      int stages) {
  using P = PrepCfg<HD, kF16In>;
  constexpr int half = HD / 2;
  constexpr int kGroups = half / 8;
  constexpr int kRowLanes = 32 / kGroups;
  extern __shared__ __align__(128) unsigned char prep_smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(prep_smem + stages * stage_bytes);
  uint64_t* empty = full + stages;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_chunks_layer = (a.n_tokens + kPrepTokens - 1) / kPrepTokens;
  const int n_chunks = n_chunks_layer * a.n_layers;
  const int qrows = with_q ? q.heads : 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kPrepTokens);
    }
    fence_mbarrier_init();
  }
  __syncthreads();
  // chunk c of this CTA: global chunk blockIdx.x + c * gridDim.x
  auto issue = [&](int c, int stage) {
    const int gc = blockIdx.x + c * gridDim.x;
    const int ll = gc / n_chunks_layer;
    const int t0 = (gc % n_chunks_layer) * kPrepTokens;
    const int nt = min(kPrepTokens, a.n_tokens - t0);
    unsigned char* dst = prep_smem + stage * stage_bytes;
    const uint32_t qb = (uint32_t)(nt * qrows * HD * P::kEl);
    const uint32_t kb = (uint32_t)(nt * a.kv_heads * HD * P::kEl);
    mbar_arrive_expect_tx(&full[stage], qb + 2 * kb);
    const size_t tok0 = (size_t)ll * a.n_tokens + t0;
    if (qb) bulk_load(dst, static_cast<const unsigned char*>(q.q) + tok0 * qrows * HD * P::kEl, qb, &full[stage]);
    bulk_load(dst + q_stride, static_cast<const unsigned char*>(a.k) + tok0 * a.kv_heads * HD * P::kEl, kb,
              &full[stage]);
    bulk_load(dst + q_stride + (stage_bytes - q_stride) / 2,
              static_cast<const unsigned char*>(a.v) + tok0 * a.kv_heads * HD * P::kEl, kb, &full[stage]);
  };
  const int my_chunks = blockIdx.x < n_chunks ? (n_chunks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (threadIdx.x == 0) {
    for (int c = 0; c < min(stages, my_chunks); ++c) issue(c, c);
  }
  const int d = (lane % kGroups) * 8;
  const int r0 = lane / kGroups;
  auto load8s = [&](const unsigned char* base, float (&v)[8]) {
    if (kF16In) {
      const uint4 u = *reinterpret_cast<const uint4*>(base);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    } else {
      const float4 x = *reinterpret_cast<const float4*>(base);
      const float4 y = *reinterpret_cast<const float4*>(base + 16);
      v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w; v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
    }
  };
  bool ok = true;
  for (int c = 0; c < my_chunks; ++c) {
    const int stage = c % stages;
    const int gc = blockIdx.x + c * gridDim.x;
    const int ll = gc / n_chunks_layer;
    const int t = (gc % n_chunks_layer) * kPrepTokens + warp;
    // the token's RoPE row and page id, fetched before waiting for the chunk
    const int tc = min(t, a.n_tokens - 1);
    const int pos = a.first_pos + tc;
    float cv[8], sn[8];
    if (a.rope) {
      const float4 c0 = *reinterpret_cast<const float4*>(a.rope_cos + (size_t)pos * half + d);
      const float4 c1 = *reinterpret_cast<const float4*>(a.rope_cos + (size_t)pos * half + d + 4);
      const float4 s0 = *reinterpret_cast<const float4*>(a.rope_sin + (size_t)pos * half + d);
      const float4 s1 = *reinterpret_cast<const float4*>(a.rope_sin + (size_t)pos * half + d + 4);
      cv[0] = c0.x; cv[1] = c0.y; cv[2] = c0.z; cv[3] = c0.w; cv[4] = c1.x; cv[5] = c1.y; cv[6] = c1.z; cv[7] = c1.w;
      sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w; sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
    }
    const int idx = a.first_index + tc;
    const int page = a.page_row[idx / a.page_tokens];
    if (!mbar_wait_warp(&full[stage], (c / stages) & 1)) {
      if (lane == 0) set_error(a.error, 30);
      ok = false;
      break;
    }
    if (t < a.n_tokens) {
      const unsigned char* sq = prep_smem + stage * stage_bytes + (size_t)warp * qrows * HD * P::kEl;
      const unsigned char* sk = prep_smem + stage * stage_bytes + q_stride + (size_t)warp * a.kv_heads * HD * P::kEl;
      const unsigned char* sv = sk + (stage_bytes - q_stride) / 2;
      const size_t qbase = ((size_t)ll * a.n_tokens + t) * qrows * HD;
      constexpr int kQB = 2;  // independent query rows per lane in flight
      for (int rb = r0; rb < qrows; rb += kQB * kRowLanes) {
        float lo[kQB][8], hi[kQB][8];
#pragma unroll
        for (int k = 0; k < kQB; ++k) {
          const int r = rb + k * kRowLanes;
          if (r < qrows) {
            load8s(sq + (size_t)(r * HD + d) * P::kEl, lo[k]);
            load8s(sq + (size_t)(r * HD + d + half) * P::kEl, hi[k]);
          }
        }
#pragma unroll
        for (int k = 0; k < kQB; ++k) {
          const int r = rb + k * kRowLanes;
          if (r < qrows) {
            if (q.q_bias) {
              const float* br = q.q_bias + ((size_t)(q.layer_begin + ll) * qrows + r) * HD;
              add_bias8(lo[k], br + d);
              add_bias8(hi[k], br + d + half);
            }
            if (q.rope) {
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const float x = lo[k][e], y = hi[k][e];
                lo[k][e] = rope_lo(x, y, cv[e], sn[e]);
                hi[k][e] = rope_hi(x, y, cv[e], sn[e]);
              }
            }
            store_q8<HD>(q, qbase + (size_t)r * HD, d, lo[k], hi[k]);
          }
        }
      }
      const int layer = a.layer_begin + ll;
      for (int kvh = r0; kvh < a.kv_heads; kvh += kRowLanes) {
        float klo[8], khi[8], vlo[8], vhi[8];
        load8s(sk + (size_t)(kvh * HD + d) * P::kEl, klo);
        load8s(sk + (size_t)(kvh * HD + d + half) * P::kEl, khi);
        load8s(sv + (size_t)(kvh * HD + d) * P::kEl, vlo);
        load8s(sv + (size_t)(kvh * HD + d + half) * P::kEl, vhi);
        if (a.k_bias) {
          const size_t brow = ((size_t)layer * a.kv_heads + kvh) * HD;
          add_bias8(klo, a.k_bias + brow + d);
          add_bias8(khi, a.k_bias + brow + d + half);
          add_bias8(vlo, a.v_bias + brow + d);
          add_bias8(vhi, a.v_bias + brow + d + half);
        }
        if (a.rope) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float x = klo[e], y = khi[e];
            klo[e] = rope_lo(x, y, cv[e], sn[e]);
            khi[e] = rope_hi(x, y, cv[e], sn[e]);
          }
        }
        const size_t row =
            ((size_t)(layer * a.num_pages + page) * a.kv_heads + kvh) * a.page_tokens + (idx % a.page_tokens);
        uint16_t* kd = a.k_pool + row * HD;
        uint16_t* vd = a.v_pool + row * HD;
        *reinterpret_cast<uint4*>(kd + d) = pack8(klo);
        *reinterpret_cast<uint4*>(kd + d + half) = pack8(khi);
        *reinterpret_cast<uint4*>(vd + d) = pack8(vlo);
        *reinterpret_cast<uint4*>(vd + d + half) = pack8(vhi);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (threadIdx.x == 0 && c + stages < my_chunks) {
      // refill this stage once every warp has read it
      if (!mbar_wait(&empty[stage], (c / stages) & 1)) {
        set_error(a.error, 31);
        ok = false;
      } else {
        issue(c + stages, stage);
      }
    }
  }
  // leave no copy in flight
  if (threadIdx.x == 0) {
    for (int c = max(0, my_chunks - stages); c < my_chunks; ++c) {
      if (!mbar_wait(&full[c % stages], (c / stages) & 1)) set_error(a.error, 32);
    }
  }
  (void)ok;
}

}  // namespace

cudaError_t launch_rope_rows(float* values, const float* cos_row, const float* sin_row, int heads, int head_dim,
                             cudaStream_t s) {
  const int n = heads * (head_dim / 2);
  rope_rows_kernel<<<(n + 255) / 256, 256, 0, s>>>(values, cos_row, sin_row, heads, head_dim);
  return cudaGetLastError();
}

cudaError_t launch_append_rope(const AppendParams& p, cudaStream_t s) {
  const long long per_layer = (long long)p.n_tokens * p.kv_heads * (p.head_dim / 16);
  if (per_layer == 0 || p.n_layers == 0) return cudaSuccess;
  const dim3 grid((unsigned)((per_layer + 255) / 256), (unsigned)p.n_layers);
  if (p.head_dim == 128) append_rope_kernel<128><<<grid, 256, 0, s>>>(p);
  else if (p.head_dim == 64) append_rope_kernel<64><<<grid, 256, 0, s>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

// The same work as two grid-per-row kernels (no shared-memory staging).
cudaError_t launch_prefill_prep_split(const AppendParams& a, const QPrepParams& q, bool with_q, cudaStream_t s) {
  cudaError_t e = launch_append_rope(a, s);
  if (e == cudaSuccess && with_q) e = launch_q_prep(q, s);
  return e;
}

template <int HD, bool kF16In>
cudaError_t launch_prefill_prep_impl(const AppendParams& a, const QPrepParams& q, bool with_q, int sm_count,
                                     cudaStream_t s) {
  using P = PrepCfg<HD, kF16In>;
  const int qrows = with_q ? q.heads : 0;
  const int q_stride = kPrepTokens * qrows * HD * P::kEl;
  const int stage_bytes = q_stride + 2 * kPrepTokens * a.kv_heads * HD * P::kEl;
  const int stages = std::min(4, (100 * 1024) / stage_bytes);  // two CTAs per SM
  if (stages < 2) return launch_prefill_prep_split(a, q, with_q, s);  // chunks too large to double-buffer
  const int smem = stages * stage_bytes + 2 * stages * 8;
  cudaError_t e = cudaFuncSetAttribute(prefill_prep_kernel<HD, kF16In>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const int n_chunks = (a.n_tokens + kPrepTokens - 1) / kPrepTokens * a.n_layers;
  const int grid = std::min(n_chunks, 2 * sm_count);
  prefill_prep_kernel<HD, kF16In><<<grid, kPrepThreads, smem, s>>>(a, q, with_q ? 1 : 0, q_stride, stage_bytes, stages);
  return cudaGetLastError();
}

cudaError_t launch_prefill_prep(const AppendParams& a, const QPrepParams& q, bool with_q, int sm_count,
                                cudaStream_t s) {
  if (a.n_tokens == 0 || a.n_layers == 0) return cudaSuccess;
  if (a.head_dim == 128) {
    return a.input_f16 ? launch_prefill_prep_impl<128, true>(a, q, with_q, sm_count, s)
                       : launch_prefill_prep_impl<128, false>(a, q, with_q, sm_count, s);
  }
  if (a.head_dim == 64) {
    return a.input_f16 ? launch_prefill_prep_impl<64, true>(a, q, with_q, sm_count, s)
                       : launch_prefill_prep_impl<64, false>(a, q, with_q, sm_count, s);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_q_prep(const QPrepParams& p, cudaStream_t s) {
  const long long per_layer = (long long)p.n_tokens * p.heads * (p.head_dim / 16);
  if (per_layer == 0 || p.n_layers == 0) return cudaSuccess;
  const dim3 grid((unsigned)((per_layer + 255) / 256), (unsigned)p.n_layers);
  if (p.head_dim == 128) q_prep_kernel<128><<<grid, 256, 0, s>>>(p);
  else if (p.head_dim == 64) q_prep_kernel<64><<<grid, 256, 0, s>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace te
