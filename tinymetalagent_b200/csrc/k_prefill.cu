// Causal flash-attention prefill on 5th-generation tensor cores (sm_100a).
//
// Reference semantics: the CPU prefill calls te_attention_decode_f32 once per
// prompt token t with position t over the cache filled so far
// (c/src/qwen.c:810-824; c/src/ops.c:323-395): query t attends keys 0..t,
// scale 1/sqrt(head_dim), softmax, weighted V sum.  The Metal analogue is the
// 8x16-tile simdgroup-MMA kernel te_attention_flash_mma_t_f32_kernel
// (c/src/metal/metal_kernels.metal.inc:2693-2836, causal test
// c/tests/kernel_ops.c:678-741).
//
// One work item = (layer, query head, 128-query tile); items are ordered by
// decreasing causal length and dealt round-robin to a persistent grid of one
// CTA per SM.  Warp roles (192 threads):
//   warp 0     TMA producer: Q tiles (double-buffered, so the next item's Q
//              is prefetched), K/V tiles (128 keys) into a 2-stage ring
//   warp 1     TMEM owner; lane 0 issues tcgen05.mma:
//                S[sb] = Q K^T   (M=128 queries, N=128 keys, K=128 dims, f16 -> f32 in TMEM)
//                O    += P V     (M=128 queries, N=128 dims,  K=128 keys)
//   warps 2-5  softmax + epilogue, one query row per thread (TMEM lane): read S
//              with tcgen05.ld, causal mask, online softmax in exp2 domain, P
//              (f16) to shared memory in the 128B-swizzled K-major layout the
//              MMA reads; O is rescaled in TMEM only when the running max grows
//              by more than 2^8 (exact: l uses the same reference max).
// S is double-buffered in TMEM so Q K^T of tile j+1 overlaps the softmax of
// tile j, and P V of tile j overlaps the softmax of tile j+1.
// Operands are staged by TMA with 128-byte swizzle (no multicast).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "te_internal.h"
#include "te_ptx.cuh"

namespace te {
namespace {

constexpr int BM = 128;                     // queries per tile
constexpr int BN = 128;                     // keys per tile
constexpr int HD = 128;                     // head dim
constexpr int kTile = BM * HD * 2;          // 32 KiB: 128 rows x 128 f16, as two 64-column halves
constexpr int kHalf = kTile / 2;            // 16 KiB: 128 rows x 128 B
constexpr int kBox = 64 * 128;              // 8 KiB TMA box: 64 rows x 64 f16
constexpr int kThreads = 192;

constexpr int OFF_Q = 0;                    // two Q buffers (the next item's Q is prefetched)
constexpr int OFF_KV = OFF_Q + 2 * kTile;   // stage s: K at OFF_KV + s*2*kTile, V at + kTile
constexpr int OFF_P = OFF_KV + 4 * kTile;
constexpr int OFF_BAR = OFF_P + kTile;      // 229376
constexpr int kSmemBytes = OFF_BAR + 256 + 1024;

enum Bar {
  Q_FULL0 = 0, Q_FULL1, Q_EMPTY0, Q_EMPTY1, K_FULL0, K_FULL1, V_FULL0, V_FULL1, KV_EMPTY0, KV_EMPTY1,
  S_FULL0, S_FULL1, S_EMPTY0, S_EMPTY1, P_FULL, PV_DONE, O_EMPTY, DRAIN, kNumBars
};

constexpr uint32_t kTmemCols = 512;         // S0 [0,128), S1 [128,256), O [256,384)
constexpr uint32_t kColO = 256;

struct Item {
  int layer_local, head, qt, n_kv;
};

__device__ __forceinline__ Item item_of(const PrefillParams& p, int it) {
  const int per_qt = p.n_layers * p.heads;
  const int n_qt = p.n_tokens_padded / BM;
  Item I;
  I.qt = n_qt - 1 - it / per_qt;            // longest causal rows first
  const int r = it % per_qt;
  I.layer_local = r / p.heads;
  I.head = r % p.heads;
  const int total = p.q_offset + p.n_tokens;
  const int last_key = min(p.q_offset + (I.qt + 1) * BM, total);  // keys [0, last_key)
  I.n_kv = (last_key + BN - 1) / BN;
  return I;
}

__device__ __forceinline__ bool aborted(volatile int* flag) { return *flag != 0; }

__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[Q_FULL0 + s], 1);
      mbar_init(&bar[Q_EMPTY0 + s], 1);
      mbar_init(&bar[K_FULL0 + s], 1);
      mbar_init(&bar[V_FULL0 + s], 1);
      mbar_init(&bar[KV_EMPTY0 + s], 1);
      mbar_init(&bar[S_FULL0 + s], 1);
      mbar_init(&bar[S_EMPTY0 + s], 4);
    }
    mbar_init(&bar[P_FULL], 4);
    mbar_init(&bar[PV_DONE], 1);
    mbar_init(&bar[O_EMPTY], 4);
    mbar_init(&bar[DRAIN], 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int total = p.q_offset + p.n_tokens;
  const int G = p.heads / p.kv_heads;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the items (page-table entries are read one per lane
    // and shuffled); lane 0 issues every TMA copy.
    if (lane == 0) {
      prefetch_tmap(&p.tmap_q);
      prefetch_tmap(&p.tmap_k);
      prefetch_tmap(&p.tmap_v);
    }
    uint32_t qc = 0, kc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      // one lane reads the abort flag so the whole warp takes the same branch
      if (__shfl_sync(0xffffffffu, lane == 0 && aborted(abort_flag) ? 1 : 0, 0)) break;
      const Item I = item_of(p, it);
      const int qs = qc & 1;
      if (lane == 0) {
        if (!mbar_wait(&bar[Q_EMPTY0 + qs], ((qc >> 1) & 1) ^ 1)) {
          set_error(p.error, 11);
          ok = false;
        } else {
          mbar_arrive_expect_tx(&bar[Q_FULL0 + qs], kTile);
          const int qrow = (I.layer_local * p.heads + I.head) * p.n_tokens_padded + I.qt * BM;
#pragma unroll
          for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < 2; ++c)
              tma_load_2d(smem + OFF_Q + qs * kTile + c * kHalf + h * kBox, &p.tmap_q, &bar[Q_FULL0 + qs], c * 64,
                          qrow + h * 64);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      ++qc;
      const int layer = p.layer_begin + I.layer_local;
      const int kvh = I.head / G;
      int pg_batch = -1, pg_reg = 0;
      for (int j = 0; j < I.n_kv; ++j, ++kc) {
        const int s = kc & 1;
        int pages[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int idx = min((j * BN + h * 64) / p.page_tokens, p.n_pages_mapped - 1);  // rows past the end are masked
          if ((idx >> 5) != pg_batch) {
            pg_batch = idx >> 5;
            const int e = pg_batch * 32 + lane;
            pg_reg = e < p.n_pages_mapped ? p.page_table_row[e] : 0;
          }
          pages[h] = __shfl_sync(0xffffffffu, pg_reg, idx & 31);
        }
        if (lane == 0) {
          if (!mbar_wait(&bar[KV_EMPTY0 + s], ((kc >> 1) & 1) ^ 1)) {
            set_error(p.error, 12);
            ok = false;
          } else {
            unsigned char* ks = smem + OFF_KV + s * 2 * kTile;
            unsigned char* vs = ks + kTile;
            mbar_arrive_expect_tx(&bar[K_FULL0 + s], kTile);
            mbar_arrive_expect_tx(&bar[V_FULL0 + s], kTile);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int tok = j * BN + h * 64;
              const int row = ((layer * p.num_pages + pages[h]) * p.kv_heads + kvh) * p.page_tokens + (tok % p.page_tokens);
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                tma_load_2d(ks + c * kHalf + h * kBox, &p.tmap_k, &bar[K_FULL0 + s], c * 64, row);
                tma_load_2d(vs + c * kHalf + h * kBox, &p.tmap_v, &bar[V_FULL0 + s], c * 64, row);
              }
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
    }
    if (!ok) *abort_flag = 1;
    // Leave no copy in flight: the last Q and K/V stages have landed (immediate when consumed).
    if (lane == 0) {
      for (uint32_t j = qc >= 2 ? qc - 2 : 0; j < qc; ++j) {
        if (!mbar_wait(&bar[Q_FULL0 + (j & 1)], (j >> 1) & 1)) set_error(p.error, 13);
      }
      for (uint32_t k = (kc >= 2 ? kc - 2 : 0); k < kc; ++k) {
        if (!mbar_wait(&bar[K_FULL0 + (k & 1)], (k >> 1) & 1)) set_error(p.error, 14);
        if (!mbar_wait(&bar[V_FULL0 + (k & 1)], (k >> 1) & 1)) set_error(p.error, 14);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = idesc_f16_f32(BM, BN, false, false);
      constexpr uint32_t idesc_pv = idesc_f16_f32(BM, HD, false, true);
      const uint32_t sp = smem_u32(smem + OFF_P);
      uint32_t qc = 0, kc = 0, sc = 0, pc = 0, oc = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < p.n_items && ok && !aborted(abort_flag); it += gridDim.x) {
        const Item I = item_of(p, it);
        const int qs = qc & 1;
        if (!mbar_wait(&bar[Q_FULL0 + qs], (qc >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sq = smem_u32(smem + OFF_Q + qs * kTile);
        const uint32_t kc0 = kc;
        auto do_pv = [&](int jj) -> bool {
          const uint32_t k_idx = kc0 + jj;
          const int s = k_idx & 1;
          if (!mbar_wait(&bar[P_FULL], pc & 1)) return false;
          if (jj == 0 && !mbar_wait(&bar[O_EMPTY], (oc & 1) ^ 1)) return false;
          if (!mbar_wait(&bar[V_FULL0 + s], (k_idx >> 1) & 1)) return false;
          tc_fence_after();
          const uint32_t sv = smem_u32(smem + OFF_KV + s * 2 * kTile + kTile);
#pragma unroll
          for (int k = 0; k < BN / 16; ++k) {
            const uint64_t a = smem_desc_sw128(sp + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
            const uint64_t b = smem_desc_sw128(sv + k * 2048, kHalf, 1024);
            umma_f16(tmem + kColO, a, b, idesc_pv, (jj > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&bar[PV_DONE]);
          umma_commit(&bar[KV_EMPTY0 + s]);
          ++pc;
          return true;
        };
        for (int j = 0; j < I.n_kv && ok; ++j) {
          const uint32_t k_idx = kc0 + j;
          const int s = k_idx & 1;
          const int sb = sc & 1;
          if (!mbar_wait(&bar[K_FULL0 + s], (k_idx >> 1) & 1) ||
              !mbar_wait(&bar[S_EMPTY0 + sb], ((sc >> 1) & 1) ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sk = smem_u32(smem + OFF_KV + s * 2 * kTile);
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint64_t a = smem_desc_sw128(sq + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
            const uint64_t b = smem_desc_sw128(sk + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
            umma_f16(tmem + sb * BN, a, b, idesc_qk, k > 0 ? 1u : 0u);
          }
          umma_commit(&bar[S_FULL0 + sb]);
          ++sc;
          if (j == I.n_kv - 1) umma_commit(&bar[Q_EMPTY0 + qs]);
          if (j >= 1 && !do_pv(j - 1)) ok = false;
        }
        if (ok && !do_pv(I.n_kv - 1)) ok = false;
        kc = kc0 + I.n_kv;
        ++qc;
        ++oc;
      }
      if (!ok) { set_error(p.error, 15); *abort_flag = 1; }
      // Every MMA this thread issued has completed before TMEM is released.
      umma_commit(&bar[DRAIN]);
      if (!mbar_wait(&bar[DRAIN], 0)) set_error(p.error, 16);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const uint32_t sp = smem_u32(smem + OFF_P);
    const float sl = p.scale_log2;
    uint32_t sc = 0, pc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      if (__any_sync(0xffffffffu, aborted(abort_flag))) break;
      const Item I = item_of(p, it);
      const int q_pos = p.q_offset + I.qt * BM + row;
      const int key_limit = min(q_pos, total - 1);
      const int first_row_limit = min(p.q_offset + I.qt * BM, total - 1);
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < I.n_kv; ++j) {
        const int sb = sc & 1;
        if (!mbar_wait_warp(&bar[S_FULL0 + sb], (sc >> 1) & 1)) { ok = false; break; }
        tc_fence_after();
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          tmem_ld32(tmem + lane_addr + sb * BN + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
        }
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[S_EMPTY0 + sb]);
        ++sc;
        const bool need_mask = (j + 1) * BN - 1 > first_row_limit;
        if (need_mask) {
#pragma unroll
          for (int c = 0; c < BN; ++c) {
            if (j * BN + c > key_limit) s[c] = -INFINITY;
          }
        }
        // row max of the raw scores: 8 independent partial maxima, then a tree
        float pm[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = s[u];
#pragma unroll
        for (int c = 8; c < BN; ++c) pm[c & 7] = fmaxf(pm[c & 7], s[c]);
        const float tmax_raw = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])),
                                     fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
        const float m_new = fmaxf(m, tmax_raw * sl);  // scaling by sl > 0 preserves the max
        if (pc > 0) {  // P buffer free and O stable: the previous P V finished
          if (!mbar_wait_warp(&bar[PV_DONE], (pc - 1) & 1)) { ok = false; break; }
          tc_fence_after();
        }
        if (j == 0) {
          m = m_new;
        } else if (m_new > m + 8.f) {
          const float alpha = ex2(m - m_new);
          l *= alpha;
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_addr + kColO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(tmem + lane_addr + kColO + c * 32, o);
          }
          tmem_wait_st();
          m = m_new;
        }
        // p = 2^(s*scale - m): one FFMA + one SFU op per score; 8 partial sums
        const float neg_m = -m;
        float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          const float e = ex2(fmaf(s[c], sl, neg_m));
          s[c] = e;
          ps[c & 7] += e;
        }
        const float rs = ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        l += rs;
        // P row -> shared memory, 128B-swizzled K-major (two 64-key halves).
#pragma unroll
        for (int ch = 0; ch < BN / 8; ++ch) {
          const uint32_t addr = sp + (ch >> 3) * kHalf + row * 128 + ((((ch & 7) ^ (row & 7))) << 4);
          sts128(addr, pack_half2(s[ch * 8 + 0], s[ch * 8 + 1]), pack_half2(s[ch * 8 + 2], s[ch * 8 + 3]),
                 pack_half2(s[ch * 8 + 4], s[ch * 8 + 5]), pack_half2(s[ch * 8 + 6], s[ch * 8 + 7]));
        }
        fence_proxy_async_shared();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[P_FULL]);
        ++pc;
      }
      if (!ok) break;
      // epilogue: O / l -> out[layer][token][head][:]
      if (!mbar_wait_warp(&bar[PV_DONE], (pc - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      const int tok = I.qt * BM + row;
      const float inv = 1.f / l;
      float* dst = p.out + (((size_t)I.layer_local * p.n_tokens + tok) * p.heads + I.head) * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_addr + kColO + c * 32, o);
        tmem_wait_ld();
        if (tok < p.n_tokens) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            *reinterpret_cast<float4*>(dst + c * 32 + e) =
                make_float4(o[e] * inv, o[e + 1] * inv, o[e + 2] * inv, o[e + 3] * inv);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[O_EMPTY]);
    }
    if (!ok) { set_error(p.error, 17); *abort_flag = 1; }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

cudaError_t launch_prefill_tc(const PrefillParams& p, int sm_count, cudaStream_t s) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int grid = p.n_items < sm_count ? p.n_items : sm_count;
  prefill_tc_kernel<<<grid, kThreads, kSmemBytes, s>>>(p);
  return cudaGetLastError();
}

}  // namespace te
