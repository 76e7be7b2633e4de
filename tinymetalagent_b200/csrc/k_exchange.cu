// KV-split decode exchange over NVLink: all-gather of the partial records of
// every rank plus their log-sum-exp merge, in one kernel per step.
//
// Each rank decodes its token range with TE_ATTN_PARTIAL into records
// [rows][head_dim + 2] (unnormalised O, then m and l in log2 units).  The
// reference merges nothing (it runs on one device); the merge is that of
// te_attention_merge_partials (the rescale of
// c/src/metal/metal_kernels.metal.inc:2650-2681).
//
// Every rank owns an exchange area in its own HBM, mapped into the other
// ranks' processes through CUDA IPC:
//   data      [2 parities][world][rows][head_dim + 2] fp32
//   arrivals  [2 parities][grid] uint64, counted up by the peers
//   steps     [grid] uint32, this rank's step count per CTA
// CTA c of step s (parity s & 1) stores rows [c*rpc, (c+1)*rpc) of the local
// records into slot `rank` of every rank's data (plain stores over NVLink for
// the peers), makes them visible system-wide, adds 1 to arrivals[parity][c]
// of every peer (a release reduction), then waits (acquire loads) until its
// own arrivals[parity][c] reaches
// (s / 2 + 1) * (world - 1) -- CTA c of every peer has delivered the same rows
// -- and merges those rows from its local data.  A rank runs at most one step
// ahead of any peer (its step s+1 waits for the peers' step s+1 pushes, which
// each peer makes after its step s merge), so the two parities never overlap.
// The step count lives in device memory, so replaying a captured CUDA graph
// continues the sequence.  The wait is bounded (the engine's wait limit, 2 s
// unless te_attn_engine_set_wait_limit changed it); when it runs out the CTA
// sets the engine's error word and leaves without merging.
#include <cuda_runtime.h>

#include <cmath>

#include "te_internal.h"
#include "te_ptx.cuh"

namespace te {
namespace {

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(256) exchange_merge_kernel(const __grid_constant__ ExchangeParams p) {
  const int c = blockIdx.x;
  const int rec = p.head_dim + 2;
  const int r0 = c * p.rows_per_cta;
  const int r1 = min(p.rows, r0 + p.rows_per_cta);
  __shared__ uint32_t s_step;
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_step = p.steps[c];
  __syncthreads();
  const uint32_t step = s_step;
  const int par = (int)(step & 1u);
  const size_t data_floats = (size_t)p.world * p.rows * rec;  // one parity
  if (r0 < r1) {
    // push: rows [r0, r1) into slot `rank` of every rank (records are an even
    // number of floats, so rows start on 8-byte boundaries)
    const float2* src = reinterpret_cast<const float2*>(p.partial + (size_t)r0 * rec);
    const int n2 = (r1 - r0) * rec / 2;
    const size_t off = (size_t)par * data_floats + ((size_t)p.rank * p.rows + r0) * rec;
    for (int w = 0; w < p.world; ++w) {
      float2* dst = reinterpret_cast<float2*>(p.base[w] + off);
      for (int i = threadIdx.x; i < n2; i += blockDim.x) dst[i] = src[i];
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 0; w < p.world; ++w) {
      if (w == p.rank) continue;
      unsigned long long* arr = reinterpret_cast<unsigned long long*>(p.base[w] + 2 * data_floats) + par * p.grid + c;
      asm volatile("red.release.sys.global.add.u64 [%0], 1;" ::"l"(arr) : "memory");
    }
    const unsigned long long target = (unsigned long long)(step / 2u + 1u) * (unsigned long long)(p.world - 1);
    const unsigned long long* mine =
        reinterpret_cast<const unsigned long long*>(p.base[p.rank] + 2 * data_floats) + par * p.grid + c;
    int ok = 1;
    if (ld_acquire_sys(mine) < target) {
      const uint64_t start = globaltimer_ns();
      while (ld_acquire_sys(mine) < target) {
        __nanosleep(64);
        if (globaltimer_ns() - start > p.wait_ns) {
          set_error(p.error, 40);
          ok = 0;
          break;
        }
      }
    }
    p.steps[c] = step + 1u;
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  __threadfence_system();
  // merge: one warp per row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* data = p.base[p.rank] + (size_t)par * data_floats;
  for (int row = r0 + warp; row < r1; row += blockDim.x >> 5) {
    float m = -INFINITY, l = 0.f;
    if (lane < p.world) {
      const float* r = data + ((size_t)lane * p.rows + row) * rec;
      l = r[p.head_dim + 1];
      m = l > 0.f ? r[p.head_dim] : -INFINITY;
    }
    float M = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float wl = (lane < p.world && l > 0.f) ? l * ex2(m - M) : 0.f;
    float L = wl;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    for (int d = lane; d < p.head_dim; d += 32) {
      float O = 0.f;
      for (int k = 0; k < p.world; ++k) {
        const float* r = data + ((size_t)k * p.rows + row) * rec;
        const float lk = r[p.head_dim + 1];
        if (lk > 0.f) O += r[d] * ex2(r[p.head_dim] - M);
      }
      p.out[(size_t)row * p.head_dim + d] = L > 0.f ? O / L : 0.f;
    }
  }
}

}  // namespace

size_t exchange_area_bytes(int world, int rows, int head_dim, int grid) {
  const size_t data = 2ull * world * rows * (head_dim + 2) * sizeof(float);
  return data + 2ull * grid * sizeof(unsigned long long) + (size_t)grid * sizeof(uint32_t);
}

int exchange_grid(int rows) {
  const int g = (rows + 7) / 8;
  return g < 148 ? g : 148;
}

cudaError_t launch_exchange_merge(const ExchangeParams& p, cudaStream_t s) {
  exchange_merge_kernel<<<p.grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

}  // namespace te
