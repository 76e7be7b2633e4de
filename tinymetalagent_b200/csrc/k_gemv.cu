// Matrix-vector products with GGUF Q4_0 / Q8_0 weights (HBM-bound).
//
// Reference semantics: te_model_matvec_f32 (c/src/ops.c:177-262) computes,
// for every row of a row-major quantized matrix W [rows][cols], the dot
// product with an fp32 input (te_q4_0_dot_row / te_q8_0_dot_row,
// c/src/ops.c:584-620): 32-weight blocks, each an f16 scale followed by the
// quants -- Q4_0: 16 bytes, byte j holding weight j in its low nibble and
// weight j+16 in its high nibble, both offset by 8; Q8_0: 32 int8 -- and
// weight = quant * scale.  The Metal version is te_metal_matvec_f32
// (c/src/metal/metal_kernels.metal.inc:75-1927).  Here the products are the
// reference's ((q - 8) * scale) * x in fp32; the sums run in another order
// (per-lane partial sums, then a warp tree), so results agree to fp32
// rounding, not bit for bit.
//
// A CTA takes groups of whole rows, a contiguous byte range of W, and copies
// each group into shared memory with 16-byte asynchronous copies (two stages,
// the next group in flight while the current one is reduced); the ragged
// ends of a range (row starts are only 2-byte aligned: 18- and 34-byte
// blocks) are fetched with 2-byte loads.  Warps then take rows, lanes take
// blocks, and a warp reduction produces y[v][row] for up to 8 input vectors.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "te_internal.h"
#include "te_ptx.cuh"

namespace te {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvStageBytes = 24 * 1024;

template <int BLOCK_BYTES, int V>
__global__ void __launch_bounds__(kGemvThreads, V <= 2 ? 2 : 1) gemv_gguf_kernel(const GemvParams p) {
  extern __shared__ __align__(16) unsigned char gsm[];
  const int rb = (p.cols / 32) * BLOCK_BYTES;  // bytes per row
  const int rows_per_group = p.rows_per_group;
  const int n_groups = (p.rows + rows_per_group - 1) / rows_per_group;
  const int stage_bytes = p.stage_bytes;
  const unsigned char* w = static_cast<const unsigned char*>(p.w);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // group g covers bytes [lo, hi) of W; its copy starts at lo rounded down to 16
  auto span = [&](int g, long long& lo16, long long& hi) {
    const long long r0 = (long long)g * rows_per_group;
    const long long r1 = min((long long)p.rows, r0 + rows_per_group);
    lo16 = (r0 * rb) & ~15ll;
    hi = r1 * rb;
  };
  auto issue = [&](int g, int stage) {
    long long lo16, hi;
    span(g, lo16, hi);
    unsigned char* dst = gsm + stage * stage_bytes;
    const long long hi16 = hi & ~15ll;
    const int n16 = (int)((hi16 - lo16) >> 4);
    for (int i = threadIdx.x; i < n16; i += blockDim.x) {
      cp_async_cg16(smem_u32(dst + i * 16), w + lo16 + (long long)i * 16);
    }
    // tail: [max(hi16, lo16), hi) in 2-byte words (row ranges and offsets are even)
    const long long t0 = hi16 > lo16 ? hi16 : lo16;
    const int nt = (int)((hi - t0) >> 1);
    for (int i = threadIdx.x; i < nt; i += blockDim.x) {
      *reinterpret_cast<uint16_t*>(dst + (t0 - lo16) + 2 * i) =
          __ldg(reinterpret_cast<const uint16_t*>(w + t0) + i);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  int g = blockIdx.x;
  if (g < n_groups) issue(g, 0);
  for (int it = 0; g < n_groups; g += gridDim.x, ++it) {
    const int stage = it & 1;
    const int gn = g + gridDim.x;
    if (gn < n_groups) {
      issue(gn, stage ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");  // this group's copies have landed
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    long long lo16, hi;
    span(g, lo16, hi);
    const unsigned char* base = gsm + stage * stage_bytes;
    const int r0 = g * rows_per_group;
    const int r1 = min(p.rows, r0 + rows_per_group);
    for (int row = r0 + warp; row < r1; row += kGemvThreads / 32) {
      const unsigned char* rp = base + ((long long)row * rb - lo16);
      float acc[V];
#pragma unroll
      for (int v = 0; v < V; ++v) acc[v] = 0.f;
      for (int b = lane; b < p.cols / 32; b += 32) {
        const unsigned char* blk = rp + b * BLOCK_BYTES;
        const float scale = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk)));
        constexpr int kWords = (BLOCK_BYTES - 2) / 2;  // 2-byte words of quants: 8 (Q4_0) or 16 (Q8_0)
        uint32_t qw[kWords];
#pragma unroll
        for (int j = 0; j < kWords; ++j) qw[j] = *reinterpret_cast<const uint16_t*>(blk + 2 + 2 * j);
        // weights 16h .. 16h+15 (Q4_0: low nibbles of the 16 bytes, then high
        // nibbles; Q8_0: bytes 16h .. 16h+15)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float wq[16];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (BLOCK_BYTES == 18) {
              const uint32_t q0 = qw[j] & 0xffu, q1 = qw[j] >> 8;
              wq[2 * j] = ((float)(h ? q0 >> 4 : q0 & 0x0fu) - 8.0f) * scale;
              wq[2 * j + 1] = ((float)(h ? q1 >> 4 : q1 & 0x0fu) - 8.0f) * scale;
            } else {
              const uint32_t two = qw[8 * h + j];
              wq[2 * j] = (float)(int8_t)(two & 0xffu) * scale;
              wq[2 * j + 1] = (float)(int8_t)(two >> 8) * scale;
            }
          }
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const float4* xv = reinterpret_cast<const float4*>(p.x + (size_t)v * p.cols + (size_t)b * 32 + 16 * h);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float4 xx = __ldg(xv + k);
              acc[v] = fmaf(wq[4 * k], xx.x, acc[v]);
              acc[v] = fmaf(wq[4 * k + 1], xx.y, acc[v]);
              acc[v] = fmaf(wq[4 * k + 2], xx.z, acc[v]);
              acc[v] = fmaf(wq[4 * k + 3], xx.w, acc[v]);
            }
          }
        }
      }
#pragma unroll
      for (int v = 0; v < V; ++v) {
        float s = acc[v];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) {
          float* yp = p.y + (size_t)v * p.rows + row;
          *yp = p.accumulate ? __fadd_rn(*yp, s) : s;  // the residual add after the projection
        }
      }
    }
    __syncthreads();  // the stage is rewritten by the copy issued two groups later
  }
}

template <int BLOCK_BYTES, int V>
cudaError_t launch_v(const GemvParams& p, int grid, int smem, cudaStream_t s) {
  // the largest staging any accepted shape needs (the host rejects longer rows);
  // each launch still asks for its own size
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemv_gguf_kernel<BLOCK_BYTES, V>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  gemv_gguf_kernel<BLOCK_BYTES, V><<<grid, kGemvThreads, smem, s>>>(p);
  return cudaGetLastError();
}

template <int BLOCK_BYTES>
cudaError_t launch_b(const GemvParams& p, int n_vectors, int grid, int smem, cudaStream_t s) {
  switch (n_vectors) {
    case 1: return launch_v<BLOCK_BYTES, 1>(p, grid, smem, s);
    case 2: return launch_v<BLOCK_BYTES, 2>(p, grid, smem, s);
    case 3: return launch_v<BLOCK_BYTES, 3>(p, grid, smem, s);
    case 4: return launch_v<BLOCK_BYTES, 4>(p, grid, smem, s);
    case 5: return launch_v<BLOCK_BYTES, 5>(p, grid, smem, s);
    case 6: return launch_v<BLOCK_BYTES, 6>(p, grid, smem, s);
    case 7: return launch_v<BLOCK_BYTES, 7>(p, grid, smem, s);
    default: return launch_v<BLOCK_BYTES, 8>(p, grid, smem, s);
  }
}

}  // namespace

cudaError_t launch_gemv_gguf(GemvParams p, int block_bytes, int n_vectors, int sm_count, cudaStream_t s) {
  const int rb = (p.cols / 32) * block_bytes;
  p.rows_per_group = rb >= kGemvStageBytes ? 1 : kGemvStageBytes / rb;
  if (p.rows_per_group > p.rows) p.rows_per_group = p.rows;
  p.stage_bytes = (p.rows_per_group * rb + 15 + 16) & ~15;  // the copy starts up to 14 bytes early
  const int smem = 2 * p.stage_bytes;
  const int n_groups = (p.rows + p.rows_per_group - 1) / p.rows_per_group;
  const int grid = n_groups < 2 * sm_count ? n_groups : 2 * sm_count;
  return block_bytes == 18 ? launch_b<18>(p, n_vectors, grid, smem, s) : launch_b<34>(p, n_vectors, grid, smem, s);
}

}  // namespace te
