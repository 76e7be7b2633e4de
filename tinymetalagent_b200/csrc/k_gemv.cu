// Matrix-vector products with GGUF Q4_0 / Q8_0 weights (HBM-bound).
//
// Reference semantics: te_model_matvec_f32 (c/src/ops.c:177-262) computes,
// for every row of a row-major quantized matrix W [rows][cols], the dot
// product with an fp32 input (te_q4_0_dot_row / te_q8_0_dot_row,
// c/src/ops.c:584-620): 32-weight blocks, each an f16 scale followed by the
// quants -- Q4_0: 16 bytes, byte j holding weight j in its low nibble and
// weight j+16 in its high nibble, both offset by 8; Q8_0: 32 int8 -- and
// weight = quant * scale.  The Metal version is te_metal_matvec_f32
// (c/src/metal/metal_kernels.metal.inc:75-1927).  Here the weights are the
// same exact values, but the scale multiplies partial sums of 8 weights
// (scale * sum (q - 8) * x) and the sums run in another order (per lane, a
// warp tree, then the 8 warps in order), so results agree to fp32 rounding,
// not bit for bit.
//
// A persistent CTA walks groups of up to R whole rows (a contiguous byte range
// of W).  One thread stages each group into shared memory with a single bulk
// copy (cp.async.bulk, completion on the stage's mbarrier), keeping the next
// stages - 1 groups in flight in a ring; the copy is widened to 16-byte
// boundaries (rows start only 2-byte aligned: 18- and 34-byte blocks), and the
// few bytes past the matrix's last 16-byte boundary are read with plain loads.
// The 8 warps split the columns: a warp step covers 8 blocks (256 weights),
// lane l taking block l / 4 and 8 of its weights (4 or 8 quant bytes), and
// warp w takes steps w, w + 8, ... of every row of the group, so each input
// value a lane loads serves all R rows.  Quant codes become exact floats
// through the 2^23 bit pattern (one byte permute per weight), offsets and
// products run two per f32x2 instruction, and each warp's per-row sums meet
// in shared memory, where y[v][row] is formed.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "te_internal.h"
#include "te_ptx.cuh"

namespace te {
namespace {

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kGemvMaxStages = 4;
constexpr int kGemvHeader = 64;                          // the stages' mbarriers, then the RMSNorm scale
constexpr int kGemvScaleOffset = 8 * kGemvMaxStages;  // up to 8 scales (32 bytes)
constexpr int kGemvPartialFloats = 2 * kGemvWarps * 16;  // [2 parities][warps][R * V <= 16]
constexpr int kGemvStageOffset = kGemvHeader + kGemvPartialFloats * 4;
static_assert(kGemvStageOffset % 16 == 0, "bulk copies land on 16-byte boundaries");

// CTAs per SM the kernel is compiled for (registers): 3 with 1-2 vectors
__host__ __device__ constexpr int gemv_ctas(int v) { return v <= 2 ? 3 : 2; }

// rows per group for V input vectors (R * V <= 16 accumulators per lane);
// Q8_0 groups take half as many rows, so that two CTAs per SM hold three
// stages of typical rows
__host__ __device__ constexpr int gemv_rows(int block_bytes, int v) {
  return (v <= 2 ? 8 : (v <= 4 ? 4 : 2)) / (block_bytes == 34 && v <= 2 ? 2 : 1);
}

// One warp step of a group's dot products: 8 blocks (256 weights), lane l
// taking block l / 4 of it and 8 of its weights -- Q4_0: quant bytes
// 4 (l % 4) .. +3, i.e. weights 4 (l % 4) .. +3 (low nibbles) and
// 16 + 4 (l % 4) .. +3 (high nibbles); Q8_0: weights 8 (l % 4) .. +7 -- for
// every row of the group (FULL: all R rows present, no per-row guard).  Per
// row and vector the lane forms sum (q - offset) * x over its 8 weights
// (exact weights, fp32 products and sums) and adds scale * that to acc.  In a
// step that runs past the row's end (EDGE; cols / 32 not a multiple of 8) a
// lane past it reads the row's last block with input 0 and adds 0.
// The matrix-vector input and its fused prologue: PRO 0 reads x as given;
// PRO 1 (RMSNorm) reads (x[c] * scale) * nw[c], the scale computed once per
// CTA; PRO 2 (SwiGLU) reads x as [gate | up] and forms
// gate[c] / (1 + expf(-gate[c])) * up[c].
struct GemvInput {
  const float* x;
  const float* nw;
  const float* scales;  // shared memory: the RMSNorm scale of each vector
  int cols;
};

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// w: the RMSNorm weights of columns col .. col + 3 (PRO 1), loaded once per
// step for all vectors
template <int PRO>
__device__ __forceinline__ float4 gemv_load(const GemvInput& in, int v, int col, const float4& w) {
  const float* xr = in.x + (size_t)v * (PRO == 2 ? 2 : 1) * in.cols + col;
  float4 a = __ldg(reinterpret_cast<const float4*>(xr));
  if (PRO == 1) {
    const float sc = in.scales[v];
    a = make_float4((a.x * sc) * w.x, (a.y * sc) * w.y, (a.z * sc) * w.z, (a.w * sc) * w.w);
  } else if (PRO == 2) {
    const float4 u = __ldg(reinterpret_cast<const float4*>(xr + in.cols));
    a = make_float4(silu(a.x) * u.x, silu(a.y) * u.y, silu(a.z) * u.z, silu(a.w) * u.w);
  }
  return a;
}

template <int BLOCK_BYTES, int V, int R, bool FULL, bool EDGE, int PRO>
__device__ __forceinline__ void gemv_step(const unsigned char* base, int rb, int nb, int nr, const GemvInput& X,
                                          int b0, int lane, float (&acc)[R][V]) {
  constexpr float kOff = BLOCK_BYTES == 18 ? 8388616.0f : 8388736.0f;  // 2^23 + the quant offset (8 or 128)
  const uint64_t off2 = f2_pack(kOff, kOff);
  const int j = lane & 3;
  const int xo0 = BLOCK_BYTES == 18 ? 4 * j : 8 * j;  // input offsets of the lane's two weight quads
  const int xo1 = BLOCK_BYTES == 18 ? 16 + 4 * j : 8 * j + 4;
  const int qo = BLOCK_BYTES == 18 ? 2 + 4 * j : 2 + 8 * j;  // the lane's quant bytes within a block
  const int b = b0 + (lane >> 2);
  const bool in = !EDGE || b < nb;
  const int bc = in ? b : nb - 1;
  uint64_t xs[V][4];
  float4 wa = make_float4(0.f, 0.f, 0.f, 0.f), wc = wa;
  if (PRO == 1 && in) {
    wa = __ldg(reinterpret_cast<const float4*>(X.nw + b * 32 + xo0));
    wc = __ldg(reinterpret_cast<const float4*>(X.nw + b * 32 + xo1));
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), c = a;
    if (in) {
      a = gemv_load<PRO>(X, v, b * 32 + xo0, wa);
      c = gemv_load<PRO>(X, v, b * 32 + xo1, wc);
    }
    xs[v][0] = f2_pack(a.x, a.y);
    xs[v][1] = f2_pack(a.z, a.w);
    xs[v][2] = f2_pack(c.x, c.y);
    xs[v][3] = f2_pack(c.z, c.w);
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (FULL || r < nr) {
      const unsigned char* blk = base + r * rb + bc * BLOCK_BYTES;
      const float sc = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk)));
      const uint16_t* qp = reinterpret_cast<const uint16_t*>(blk + qo);
      uint32_t lo, hi;  // the lane's 8 codes, one per byte (Q8_0: int8 + 128)
      if (BLOCK_BYTES == 18) {
        const uint32_t q = prmt(qp[0], qp[1], 0x5410u);
        lo = q & 0x0f0f0f0fu;
        hi = (q >> 4) & 0x0f0f0f0fu;
      } else {
        lo = prmt(qp[0], qp[1], 0x5410u) ^ 0x80808080u;
        hi = prmt(qp[2], qp[3], 0x5410u) ^ 0x80808080u;
      }
      // code byte i under the exponent bits of 2^23: the float 2^23 + code,
      // exact; minus the offset, exact
      uint64_t wq[4];
      wq[0] = f2_pack(__uint_as_float(prmt(lo, 0x4B000000u, 0x7440u)), __uint_as_float(prmt(lo, 0x4B000000u, 0x7441u)));
      wq[1] = f2_pack(__uint_as_float(prmt(lo, 0x4B000000u, 0x7442u)), __uint_as_float(prmt(lo, 0x4B000000u, 0x7443u)));
      wq[2] = f2_pack(__uint_as_float(prmt(hi, 0x4B000000u, 0x7440u)), __uint_as_float(prmt(hi, 0x4B000000u, 0x7441u)));
      wq[3] = f2_pack(__uint_as_float(prmt(hi, 0x4B000000u, 0x7442u)), __uint_as_float(prmt(hi, 0x4B000000u, 0x7443u)));
#pragma unroll
      for (int k = 0; k < 4; ++k) wq[k] = f2_sub(wq[k], off2);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        uint64_t d = f2_mul(wq[0], xs[v][0]);
#pragma unroll
        for (int k = 1; k < 4; ++k) d = f2_fma(wq[k], xs[v][k], d);
        float d0, d1;
        f2_unpack(d, d0, d1);
        float part = d0 + d1;
        if (EDGE) part = in ? part : 0.f;
        acc[r][v] = fmaf(sc, part, acc[r][v]);
      }
    }
  }
}

// A group's dot products, per lane: warp w takes steps w, w + 8, ... of the row.
template <int BLOCK_BYTES, int V, int R, bool FULL, int PRO>
__device__ __forceinline__ void gemv_pass(const unsigned char* base, int rb, int nb, int nr, const GemvInput& X,
                                          int warp, int lane, float (&acc)[R][V]) {
  int b0 = 8 * warp;
  for (; b0 + 8 <= nb; b0 += 8 * kGemvWarps) {
    gemv_step<BLOCK_BYTES, V, R, FULL, false, PRO>(base, rb, nb, nr, X, b0, lane, acc);
  }
  if (b0 < nb) gemv_step<BLOCK_BYTES, V, R, FULL, true, PRO>(base, rb, nb, nr, X, b0, lane, acc);
}

template <int BLOCK_BYTES, int V, int PRO>
__global__ void __launch_bounds__(kGemvThreads, gemv_ctas(V)) gemv_gguf_kernel(const GemvParams p) {
  constexpr int R = gemv_rows(BLOCK_BYTES, V);
  extern __shared__ __align__(128) unsigned char gsm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(gsm);
  float* partial = reinterpret_cast<float*>(gsm + kGemvHeader);
  unsigned char* stages = gsm + kGemvStageOffset;
  __shared__ int s_abort;

  const int nb = p.cols / 32;
  const long long rb = (long long)nb * BLOCK_BYTES;  // bytes per row
  const long long total = (long long)p.rows * rb;
  const long long total16 = total & ~15ll;
  const int rows_per_group = p.rows_per_group;
  const int n_groups = (p.rows + rows_per_group - 1) / rows_per_group;
  const int n_stages = p.stages;
  const unsigned char* w = static_cast<const unsigned char*>(p.w);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; ++s) mbar_init(&full[s], 1);
    fence_mbarrier_init();
    s_abort = 0;
  }
  // Launched as a programmatic dependent: until griddep_wait the previous
  // kernel on the stream may still run, so before it this CTA only asks L2
  // for the weight bytes of its first groups (no memory state it could race
  // with); x, y and the staging copies come after.  The next kernel may be
  // scheduled as soon as every CTA has started.
  if (threadIdx.x == 0) {
    for (int s = 0; s + 1 < n_stages; ++s) {
      const int g = blockIdx.x + s * gridDim.x;
      if (g >= n_groups) break;
      const long long lo16 = ((long long)g * rows_per_group * rb) & ~15ll;
      const long long hi16 = min(((long long)min(p.rows, (g + 1) * rows_per_group) * rb + 15) & ~15ll, total16);
      if (hi16 > lo16) bulk_prefetch_l2(w + lo16, (uint32_t)(hi16 - lo16));
    }
  }
  griddep_launch_dependents();
  griddep_wait();
  // one thread: stage group g; the copy covers [lo rounded down to 16, hi
  // rounded up to 16) clipped to the matrix's last 16-byte boundary, and the
  // bytes past that boundary (last group only) arrive by plain loads before
  // the mbarrier arrival that publishes them
  auto issue = [&](int g, int stage) {
    const long long lo = (long long)g * rows_per_group * rb;
    const long long hi = min((long long)p.rows, (long long)(g + 1) * rows_per_group) * rb;
    const long long lo16 = lo & ~15ll;
    const long long hi16 = min((hi + 15) & ~15ll, total16);
    unsigned char* dst = stages + (size_t)stage * p.stage_bytes;
    for (long long t = hi16 > lo16 ? hi16 : lo16; t < hi; t += 2) {
      *reinterpret_cast<uint16_t*>(dst + (t - lo16)) = __ldg(reinterpret_cast<const uint16_t*>(w + t));
    }
    if (hi16 > lo16) {
      mbar_arrive_expect_tx(&full[stage], (uint32_t)(hi16 - lo16));
      bulk_load(dst, w + lo16, (uint32_t)(hi16 - lo16), &full[stage]);
    } else {
      mbar_arrive(&full[stage]);
    }
  };

  // the first stages' copies start before the input's prologue runs
  if (threadIdx.x == 0) {
    for (int s = 0; s + 1 < n_stages; ++s) {
      const int g = blockIdx.x + s * gridDim.x;
      if (g < n_groups) issue(g, s);
    }
  }

  float* scales = reinterpret_cast<float*>(gsm + kGemvScaleOffset);
  const GemvInput X{p.x, p.norm_w, scales, p.cols};
  if (PRO == 1) {
    // RMSNorm scale of each input vector, as te_rmsnorm_f32 forms it
    // (c/src/ops.c:283-288): the squares summed in double, then
    // 1 / sqrtf((float)(sum / cols) + eps) in fp32; each CTA computes them
    // for itself (the vectors are a few KB), the partial-sum area holding the
    // per-warp sums before the first group uses it
    double ss[V];
#pragma unroll
    for (int v = 0; v < V; ++v) ss[v] = 0.0;
    for (int c = threadIdx.x * 4; c < p.cols; c += kGemvThreads * 4) {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(p.x + (size_t)v * p.cols + c));
        ss[v] += (double)t.x * (double)t.x + (double)t.y * (double)t.y + (double)t.z * (double)t.z +
                 (double)t.w * (double)t.w;
      }
    }
    double* red = reinterpret_cast<double*>(partial);  // [V][warps]
#pragma unroll
    for (int v = 0; v < V; ++v) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss[v] += __shfl_xor_sync(0xffffffffu, ss[v], o);
      if (lane == 0) red[v * kGemvWarps + warp] = ss[v];
    }
    __syncthreads();
    if (threadIdx.x < V) {
      double tot = 0.0;
      for (int k = 0; k < kGemvWarps; ++k) tot += red[threadIdx.x * kGemvWarps + k];
      scales[threadIdx.x] = 1.0f / sqrtf((float)(tot / (double)p.cols) + p.eps);
    }
  }
  __syncthreads();


  int it = 0;
  for (int g = blockIdx.x; g < n_groups; g += gridDim.x, ++it) {
    // the stage of iteration it - 1 was released by the barrier that ended it
    if (threadIdx.x == 0) {
      const int gi = g + (n_stages - 1) * gridDim.x;
      if (gi < n_groups) issue(gi, (it + n_stages - 1) % n_stages);
    }
    const int stage = it % n_stages;
    if (!mbar_wait(&full[stage], (uint32_t)(it / n_stages) & 1u)) {
      set_error(p.error, 50);
      s_abort = 1;  // every thread leaves after this iteration's barrier
    }
    const int r0 = g * rows_per_group;
    const int nr = min(p.rows - r0, rows_per_group);
    const long long lo16 = ((long long)r0 * rb) & ~15ll;
    const unsigned char* base = stages + (size_t)stage * p.stage_bytes + (int)((long long)r0 * rb - lo16);

    float acc[R][V];
#pragma unroll
    for (int r = 0; r < R; ++r) {
#pragma unroll
      for (int v = 0; v < V; ++v) acc[r][v] = 0.f;
    }
    if (nr == R) {
      gemv_pass<BLOCK_BYTES, V, R, true, PRO>(base, (int)rb, nb, nr, X, warp, lane, acc);
    } else {
      gemv_pass<BLOCK_BYTES, V, R, false, PRO>(base, (int)rb, nb, nr, X, warp, lane, acc);
    }
    float* part = partial + (it & 1) * (kGemvWarps * 16);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r < nr) {
#pragma unroll
        for (int v = 0; v < V; ++v) {
          float s = acc[r][v];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
          if (lane == 0) part[(warp * R + r) * V + v] = s;
        }
      }
    }
    __syncthreads();  // partial sums complete; this iteration's stage is free again
    if (threadIdx.x < nr * V) {
      const int r = threadIdx.x / V, v = threadIdx.x % V;
      float s = part[r * V + v];
#pragma unroll
      for (int k = 1; k < kGemvWarps; ++k) s += part[(k * R + r) * V + v];
      float* yp = p.y + (size_t)v * p.rows + r0 + r;
      *yp = p.accumulate ? __fadd_rn(*yp, s) : s;  // the residual add after the projection
    }
    if (s_abort) {  // read after the barrier: the same decision in every thread
      // before leaving, let the copies this CTA still has in flight land (bounded)
      if (threadIdx.x == 0) {
        for (int j = it; j < it + n_stages; ++j) {
          if (blockIdx.x + j * gridDim.x < n_groups) mbar_wait(&full[j % n_stages], (uint32_t)(j / n_stages) & 1u);
        }
      }
      break;
    }
  }
}

template <int BLOCK_BYTES, int V, int PRO = 0>
cudaError_t launch_v(const GemvParams& p, int ctas_per_sm, int sm_count, int smem, cudaStream_t s) {
  // the largest staging any accepted shape needs (the host rejects longer
  // rows); each launch still asks for its own size
  static std::atomic<uint64_t> configured{0};  // one bit per device
  const cudaError_t e =
      set_smem_limit_once(configured, (const void*)gemv_gguf_kernel<BLOCK_BYTES, V, PRO>, 227 * 1024 - 128);
  if (e != cudaSuccess) return e;
  const int n_groups = (p.rows + p.rows_per_group - 1) / p.rows_per_group;
  const int slots = ctas_per_sm * sm_count;
  const int grid = n_groups < slots ? n_groups : slots;
  // programmatic dependent launch (the kernel waits before touching any
  // memory the previous kernel may write)
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_gguf_kernel<BLOCK_BYTES, V, PRO>, p);
}

template <int BLOCK_BYTES, int PRO>
cudaError_t launch_p(const GemvParams& p, int n_vectors, int ctas_per_sm, int sm_count, int smem, cudaStream_t s) {
  switch (n_vectors) {
    case 1: return launch_v<BLOCK_BYTES, 1, PRO>(p, ctas_per_sm, sm_count, smem, s);
    case 2: return launch_v<BLOCK_BYTES, 2, PRO>(p, ctas_per_sm, sm_count, smem, s);
    case 3: return launch_v<BLOCK_BYTES, 3, PRO>(p, ctas_per_sm, sm_count, smem, s);
    case 4: return launch_v<BLOCK_BYTES, 4, PRO>(p, ctas_per_sm, sm_count, smem, s);
    case 5: return launch_v<BLOCK_BYTES, 5, PRO>(p, ctas_per_sm, sm_count, smem, s);
    case 6: return launch_v<BLOCK_BYTES, 6, PRO>(p, ctas_per_sm, sm_count, smem, s);
    case 7: return launch_v<BLOCK_BYTES, 7, PRO>(p, ctas_per_sm, sm_count, smem, s);
    default: return launch_v<BLOCK_BYTES, 8, PRO>(p, ctas_per_sm, sm_count, smem, s);
  }
}

template <int BLOCK_BYTES>
cudaError_t launch_b(const GemvParams& p, int n_vectors, int ctas_per_sm, int sm_count, int smem, cudaStream_t s) {
  if (p.prologue == 1) return launch_p<BLOCK_BYTES, 1>(p, n_vectors, ctas_per_sm, sm_count, smem, s);
  if (p.prologue == 2) return launch_p<BLOCK_BYTES, 2>(p, n_vectors, ctas_per_sm, sm_count, smem, s);
  return launch_p<BLOCK_BYTES, 0>(p, n_vectors, ctas_per_sm, sm_count, smem, s);
}

}  // namespace

cudaError_t launch_gemv_gguf(GemvParams p, int block_bytes, int n_vectors, int sm_count, cudaStream_t s) {
  const long long rb = (long long)(p.cols / 32) * block_bytes;
  // R rows per group (the kernel's compile-time count, no per-row guards),
  // fewer only when two stages of R rows would not fit one CTA; a stage holds
  // the group widened to 16-byte boundaries at both ends
  int rpg = gemv_rows(block_bytes, n_vectors);
  while (rpg > 1 && 2 * ((rpg * rb + 45) & ~15ll) + kGemvStageOffset + 128 > 227 * 1024) --rpg;
  if (rpg > p.rows) rpg = p.rows;
  p.rows_per_group = rpg;
  p.stage_bytes = (int)((rpg * rb + 30 + 15) & ~15ll);
  // the most CTAs per SM (up to gemv_ctas) whose shares of the SM's 228 KiB
  // (less the static word and the per-CTA reserve) hold at least two stages;
  // then as many stages as fit the share, up to 4
  int ctas_per_sm = gemv_ctas(n_vectors);
  int stages = 0;
  for (; ctas_per_sm >= 1; --ctas_per_sm) {
    const int share = ctas_per_sm == 1 ? 227 * 1024 - 128 : (228 * 1024) / ctas_per_sm - 1024 - 128;
    stages = (share - kGemvStageOffset) / p.stage_bytes;
    if (stages >= 2) break;
  }
  if (stages > kGemvMaxStages) stages = kGemvMaxStages;
  p.stages = stages;
  const int smem = kGemvStageOffset + stages * p.stage_bytes;
  return block_bytes == 18 ? launch_b<18>(p, n_vectors, ctas_per_sm, sm_count, smem, s)
                           : launch_b<34>(p, n_vectors, ctas_per_sm, sm_count, smem, s);
}

}  // namespace te
