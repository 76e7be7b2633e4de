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
// One work item = (layer, kv head, pair of query heads of that GQA group,
// 128-query tile).  Both heads attend exactly the same keys, so every K/V tile
// staged by TMA feeds four MMAs (an odd group's last head is a single-head
// item).  Items are ordered by decreasing causal length and dealt round-robin
// to a persistent grid of one CTA per SM.
//
// Template parameters: HD = 128 or 64 (the reference's only MMA prefill is the
// head_dim-64 kernel above); SPLIT = the query enters the tensor cores as two
// f16 tiles, hi = f16(q) and lo = f16(q - hi), both multiplied by the same K
// tile into the same S accumulator, so q.k keeps about 22 bits of the fp32
// query.  A SPLIT item is one head: its lo tile takes the second query slot
// and the second softmax warpgroup idles.
//
// Warp roles (384 threads):
//   warp 0      TMA producer: the Q tiles, then K and V tiles (128 keys) into
//               two 2-stage rings (K released after its tile's last Q K^T, V
//               after its last P V)
//   warp 1      TMEM owner; lane 0 issues tcgen05.mma in the order
//                 QK_A(0) QK_B(0) | PV_A(j) QK_A(j+1) PV_B(j) QK_B(j+1) | ...
//               (S = Q K^T: M=128 queries, N=128 keys, K=128 dims, A/B from shared
//                memory; O += P V: A = P from tensor memory, B = V from shared memory)
//   warps 2-3   idle (they complete warpgroup 0, whose registers go to the softmax)
//   warps 4-7   softmax + epilogue of head A, one query row per thread (TMEM lane)
//   warps 8-11  softmax + epilogue of head B
// Tensor memory: S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512) columns;
// P (f16, two per 32-bit column) overwrites the first 64 columns of its S once
// S has been read.  tcgen05.mma operations of one thread execute in issue
// order, so the next Q K^T into S starts only after the P V that reads P
// there.  O is rescaled in TMEM only when a row's running max grows by more
// than 2^8 (exact: l uses the same reference max).
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>

#include "te_internal.h"
#include "te_ptx.cuh"

namespace te {
namespace {

constexpr int BM = 128;                     // queries per tile
constexpr int BN = 128;                     // keys per tile
constexpr int kHalf = 128 * 128;            // 16 KiB: 128 rows x 128 B (one 64-column chunk of a tile)
constexpr int kBox = 64 * 128;              // 8 KiB TMA box: 64 rows x 64 f16
constexpr int kThreads = 384;               // three warpgroups
constexpr int kRegsLow = 120;                // per thread, warpgroup 0 (producer, MMA issuer)
constexpr int kRegsHigh = 184;              // per thread, the two softmax warpgroups
static_assert(128 * (kRegsLow + 2 * kRegsHigh) <= 65536, "register split exceeds the launch's registers");

// Shared-memory plan for head dim HD: query slots A and B, a 2-stage ring of K
// and V tiles, output staging (4 KiB per softmax warp), barriers.
template <int HD>
struct Plan {
  static constexpr int kChunks = HD / 64;    // 64-column chunks per tile row
  static constexpr int kTile = BM * HD * 2;  // one Q, K or V tile (BM == BN)
  static constexpr int OFF_QA = 0;
  static constexpr int OFF_QB = kTile;
  static constexpr int OFF_KV = 2 * kTile;   // stage s: K at OFF_KV + s*2*kTile, V at + kTile
  static constexpr int OFF_OST = OFF_KV + 4 * kTile;
  static constexpr int OFF_BAR = OFF_OST + 8 * 4096;
  static constexpr int kSmemBytes = OFF_BAR + 256 + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory plan exceeds the per-CTA limit");
};

enum Bar {
  Q_FULL = 0, Q_EMPTY, K_FULL0, K_FULL1, V_FULL0, V_FULL1, K_EMPTY0, K_EMPTY1, V_EMPTY0, V_EMPTY1,
  S_FULL_A, S_FULL_B, P_FULL_A, P_FULL_B, O_FULL_A, O_FULL_B, O_EMPTY_A, O_EMPTY_B, DRAIN, kNumBars
};

// Tensor memory: S_A [0,128) S_B [128,256) O_A [256,256+HD) O_B [256+HD,256+2HD).
constexpr uint32_t kTmemCols = 512;
__device__ __forceinline__ uint32_t col_s(int t) { return t ? 128u : 0u; }
template <int HD>
__device__ __forceinline__ uint32_t col_o(int t) { return 256u + (uint32_t)(t * HD); }

struct Item {
  int layer_local, kvh, head_a, has_b, qt, n_kv;
};

// Items of one (layer, kv head, 128-query tile): pairs of heads, or single
// heads when SPLIT (the second query slot holds the low part).
template <bool SPLIT>
__device__ __forceinline__ int units_per_group(int G) { return SPLIT ? G : (G + 1) / 2; }

template <bool SPLIT>
__device__ __forceinline__ Item item_of(const PrefillParams& p, int it) {
  const int G = p.heads / p.kv_heads;
  const int pairs = units_per_group<SPLIT>(G);
  const int per_qt = p.n_layers * p.kv_heads * pairs;
  const int n_qt = p.n_tokens_padded / BM;
  Item I;
  I.qt = n_qt - 1 - it / per_qt;  // longest causal rows first
  int r = it % per_qt;
  const int pr = r % pairs;
  r /= pairs;
  I.kvh = r % p.kv_heads;
  I.layer_local = r / p.kv_heads;
  I.head_a = I.kvh * G + (SPLIT ? pr : 2 * pr);
  I.has_b = SPLIT ? 0 : (2 * pr + 1 < G);
  const int total = p.q_offset + p.n_tokens;
  const int last_key = min(p.q_offset + (I.qt + 1) * BM, total);  // keys [0, last_key)
  I.n_kv = (last_key + BN - 1) / BN;
  return I;
}

__device__ __forceinline__ bool aborted(volatile int* flag) { return *flag != 0; }

// tcgen05.st of 16 packed f16 pairs to this thread's lane.
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t (&u)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]),
        "r"(u[8]), "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15])
      : "memory");
}

// O (+)= P V with P (f16) in tensor memory as the A operand.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <int HD, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) prefill_tc_kernel(const __grid_constant__ PrefillParams p) {
  using PL = Plan<HD>;
  constexpr int kTile = PL::kTile;
  constexpr int OFF_QA = PL::OFF_QA, OFF_QB = PL::OFF_QB, OFF_KV = PL::OFF_KV, OFF_OST = PL::OFF_OST;
  constexpr int OFF_BAR = PL::OFF_BAR;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&bar[Q_FULL], 1);
    mbar_init(&bar[Q_EMPTY], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar[K_FULL0 + s], 1);
      mbar_init(&bar[V_FULL0 + s], 1);
      mbar_init(&bar[K_EMPTY0 + s], 1);
      mbar_init(&bar[V_EMPTY0 + s], 1);
      mbar_init(&bar[S_FULL_A + s], 1);
      mbar_init(&bar[P_FULL_A + s], 4);
      mbar_init(&bar[O_FULL_A + s], 1);
      mbar_init(&bar[O_EMPTY_A + s], 4);
    }
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
  // Register split: warpgroup 0 (producer, MMA issuer, two idle warps) gives
  // registers to the softmax warpgroups, which hold a 128-score row each.
  // 128 x (kRegsLow + 2 * kRegsHigh) <= 65536 registers of the launch.
  if (warp < 4) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow) : "memory");
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the items (page-table entries are read one per lane
    // and shuffled); lane 0 issues every TMA copy.
    if (lane == 0) {
      prefetch_tmap(&p.tmap_q);
      prefetch_tmap(&p.tmap_k);
      prefetch_tmap(&p.tmap_v);
    }
    // L2 priorities: K/V tiles are re-read by every item of their (layer, kv
    // head) -- keep them; query tiles are read once -- stream them.
    const uint64_t keep = policy_evict_last();
    const uint64_t stream_once = policy_evict_first();
    uint32_t ic = 0, kc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x, ++ic) {
      if (__shfl_sync(0xffffffffu, lane == 0 && aborted(abort_flag) ? 1 : 0, 0)) break;
      const Item I = item_of<SPLIT>(p, it);
      if (lane == 0) {
        if (!mbar_wait(&bar[Q_EMPTY], (ic & 1) ^ 1)) {
          set_error(p.error, 11);
          ok = false;
        } else {
          // query tiles: heads A (and B), or head A's hi and lo parts (query
          // rows 2h and 2h + 1 of the split layout)
          const int n_q = SPLIT ? 2 : 1 + I.has_b;
          mbar_arrive_expect_tx(&bar[Q_FULL], (uint32_t)(n_q * kTile));
          for (int t = 0; t < n_q; ++t) {
            const int qrow = SPLIT ? 2 * I.head_a + t : I.head_a + t;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int c = 0; c < PL::kChunks; ++c)
                tma_load_4d_hint(smem + (t ? OFF_QB : OFF_QA) + c * kHalf + h * kBox, &p.tmap_q, &bar[Q_FULL],
                                 c * 64, qrow, I.qt * BM + h * 64, I.layer_local, stream_once);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      const int layer = p.layer_begin + I.layer_local;
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
        // K and V of a stage are released separately: K after the tile's last
        // Q K^T, V after its last P V.  V(j) needs the stage of V(j-2), whose
        // last P V completes before the last Q K^T of K(j-1) that K(j+1)
        // waits for, so loading K(j) then V(j) never holds a K load behind a
        // V load.
        if (lane == 0) {
          int rows[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int tok = j * BN + h * 64;
            rows[h] = ((layer * p.num_pages + pages[h]) * p.kv_heads + I.kvh) * p.page_tokens + (tok % p.page_tokens);
          }
          unsigned char* ks = smem + OFF_KV + s * 2 * kTile;
          unsigned char* vs = ks + kTile;
          if (!mbar_wait(&bar[K_EMPTY0 + s], ((kc >> 1) & 1) ^ 1)) {
            set_error(p.error, 12);
            ok = false;
          } else {
            mbar_arrive_expect_tx(&bar[K_FULL0 + s], kTile);
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int c = 0; c < PL::kChunks; ++c)
                tma_load_2d_hint(ks + c * kHalf + h * kBox, &p.tmap_k, &bar[K_FULL0 + s], c * 64, rows[h], keep);
          }
          if (ok && !mbar_wait(&bar[V_EMPTY0 + s], ((kc >> 1) & 1) ^ 1)) {
            set_error(p.error, 12);
            ok = false;
          } else if (ok) {
            mbar_arrive_expect_tx(&bar[V_FULL0 + s], kTile);
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int c = 0; c < PL::kChunks; ++c)
                tma_load_2d_hint(vs + c * kHalf + h * kBox, &p.tmap_v, &bar[V_FULL0 + s], c * 64, rows[h], keep);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
      }
    }
    if (!ok) *abort_flag = 1;
    // Leave no copy in flight: the last Q and K/V stages have landed (immediate when consumed).
    if (lane == 0) {
      if (ic > 0 && !mbar_wait(&bar[Q_FULL], (ic - 1) & 1)) set_error(p.error, 13);
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
      const uint32_t sq[2] = {smem_u32(smem + OFF_QA), smem_u32(smem + OFF_QB)};
      uint32_t ic = 0, kc = 0;
      uint32_t pc[2] = {0, 0};  // P tiles consumed per head slot
      uint32_t oc[2] = {0, 0};  // items (with that head slot) started
      bool ok = true;
      auto wait = [&](int b, uint32_t parity) -> bool {
        if (!mbar_wait(&bar[b], parity)) return false;
        tc_fence_after();
        return true;
      };
      auto qk = [&](int t, uint32_t k_idx) {
        const uint32_t sk = smem_u32(smem + OFF_KV + (k_idx & 1) * 2 * kTile);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t a = smem_desc_sw128(sq[t] + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
          const uint64_t b = smem_desc_sw128(sk + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
          umma_f16(tmem + col_s(t), a, b, idesc_qk, k > 0 ? 1u : 0u);
        }
        if (SPLIT) {
          // the query's low part (slot B) times the same K tile, into the same S
#pragma unroll
          for (int k = 0; k < HD / 16; ++k) {
            const uint64_t a = smem_desc_sw128(sq[1] + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
            const uint64_t b = smem_desc_sw128(sk + (k >> 2) * kHalf + (k & 3) * 32, 16, 1024);
            umma_f16(tmem + col_s(t), a, b, idesc_qk, 1u);
          }
        }
        umma_commit(&bar[S_FULL_A + t]);
      };
      auto pv = [&](int t, uint32_t k_idx, int j) {
        const uint32_t sv = smem_u32(smem + OFF_KV + (k_idx & 1) * 2 * kTile + kTile);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t b = smem_desc_sw128(sv + k * 2048, kHalf, 1024);
          umma_f16_ts(tmem + col_o<HD>(t), tmem + col_s(t) + k * 8, b, idesc_pv, (j > 0 || k > 0) ? 1u : 0u);
        }
      };
      for (int it = blockIdx.x; it < p.n_items && ok && !aborted(abort_flag); it += gridDim.x, ++ic) {
        const Item I = item_of<SPLIT>(p, it);
        const int nt = 1 + I.has_b;
        const uint32_t kc0 = kc;
        if (!wait(Q_FULL, ic & 1) || !wait(K_FULL0 + (kc0 & 1), (kc0 >> 1) & 1)) { ok = false; break; }
        for (int t = 0; t < nt; ++t) qk(t, kc0);
        umma_commit(&bar[K_EMPTY0 + (kc0 & 1)]);  // every Q K^T of tile 0 issued: K stage free on completion
        if (I.n_kv == 1) umma_commit(&bar[Q_EMPTY]);
        for (int j = 0; j < I.n_kv && ok; ++j) {
          const uint32_t k_idx = kc0 + j;
          const int s = k_idx & 1;
          for (int t = 0; t < nt; ++t) {
            // Waits that are normally complete come first (V of this tile, K
            // of the next), so that the unit's P is the last wait before its
            // MMAs are issued.
            if ((t == 0 && !wait(V_FULL0 + s, (k_idx >> 1) & 1)) ||
                (t == 0 && j + 1 < I.n_kv && !wait(K_FULL0 + ((k_idx + 1) & 1), ((k_idx + 1) >> 1) & 1)) ||
                (j == 0 && !wait(O_EMPTY_A + t, (oc[t] & 1) ^ 1)) || !wait(P_FULL_A + t, pc[t] & 1)) {
              ok = false;
              break;
            }
            ++pc[t];
            pv(t, k_idx, j);
            if (t == nt - 1) umma_commit(&bar[V_EMPTY0 + s]);  // every P V of tile j issued: V stage free on completion
            if (j + 1 < I.n_kv) {
              qk(t, k_idx + 1);
              if (t == nt - 1) umma_commit(&bar[K_EMPTY0 + ((k_idx + 1) & 1)]);  // K stage of tile j+1 free on completion
              if (j + 2 == I.n_kv && t == nt - 1) umma_commit(&bar[Q_EMPTY]);
            } else {
              umma_commit(&bar[O_FULL_A + t]);
              ++oc[t];
            }
          }
        }
        kc = kc0 + I.n_kv;
      }
      if (!ok) { set_error(p.error, 15); *abort_flag = 1; }
      // Every MMA this thread issued has completed before TMEM is released.
      umma_commit(&bar[DRAIN]);
      if (!mbar_wait(&bar[DRAIN], 0)) set_error(p.error, 16);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh) : "memory");
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >= 8 ? 1 : 0;  // which head of the pair
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    const uint32_t s_addr = tmem + lane_addr + col_s(t);
    const uint32_t o_addr = tmem + lane_addr + col_o<HD>(t);
    const float sl = p.scale_log2;
    uint32_t sc = 0, oc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      if (__any_sync(0xffffffffu, aborted(abort_flag))) break;
      const Item I = item_of<SPLIT>(p, it);
      if (t == 1 && !I.has_b) continue;
      const int q_pos = p.q_offset + I.qt * BM + row;
      const int key_limit = min(q_pos, total - 1);
      const int first_row_limit = min(p.q_offset + I.qt * BM, total - 1);
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < I.n_kv; ++j) {
        if (!mbar_wait_warp(&bar[S_FULL_A + t], sc & 1)) { ok = false; break; }
        ++sc;
        tc_fence_after();
        const bool need_mask = (j + 1) * BN - 1 > first_row_limit;
        // the row's 128 scores: four loads in flight, one wait
        float x[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(s_addr + c * 32, *reinterpret_cast<float(*)[32]>(&x[c * 32]));
        tmem_wait_ld();
        if (need_mask) {
#pragma unroll
          for (int e = 0; e < BN; ++e) {
            if (j * BN + e > key_limit) x[e] = -INFINITY;
          }
        }
        // row max of the raw scores (8 independent partial maxima, 3-input max)
        float pm[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) pm[u] = fmax3(x[u], x[u + 8], x[u + 16]);
#pragma unroll
        for (int e = 24; e < BN; e += 16) {
#pragma unroll
          for (int u = 0; u < 8; ++u) pm[u] = fmax3(pm[u], x[e + u], e + 8 + u < BN ? x[e + 8 + u] : x[e + u]);
        }
        const float tmax_raw = fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]), fmaxf(pm[6], pm[7]));
        const float m_new = fmaxf(m, tmax_raw * sl);  // scaling by sl > 0 preserves the max
        // lazy rescale: keep the old reference max unless the row max grew by > 2^8.
        // The decision is per row; the TMEM rescale of O below is
        // warp-collective, so a warp runs it when any of its rows needs it
        // (alpha = 1 for the others).
        const bool rescale = j > 0 && m_new > m + 8.f;
        const bool warp_rescale = __any_sync(0xffffffffu, rescale);
        const float alpha = rescale ? ex2(m - m_new) : 1.f;
        if (j == 0 || rescale) m = m_new;
        // p = 2^(s*scale - m) -> f16 pairs over the first half of S's columns
        // (S is entirely in registers, so overwriting its columns is safe).
        // Scale, bias and row sum take two elements per f32x2 instruction.
        const uint64_t sl2 = f2_pack(sl, sl);
        const uint64_t nm2 = f2_pack(-m, -m);
        uint64_t ps2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const uint64_t y = f2_fma(f2_pack(x[c * 32 + e], x[c * 32 + e + 1]), sl2, nm2);
            float y0, y1;
            f2_unpack(y, y0, y1);
            const uint64_t ev = f2_pack(ex2(y0), ex2(y1));
            ps2[(e >> 1) & 3] = f2_add(ps2[(e >> 1) & 3], ev);
            float e0, e1;
            f2_unpack(ev, e0, e1);
            pk[e >> 1] = pack_half2(e0, e1);
          }
          tmem_st16u(s_addr + c * 16, pk);
        }
        float ps[8];
#pragma unroll
        for (int u = 0; u < 4; ++u) f2_unpack(ps2[u], ps[2 * u], ps[2 * u + 1]);
        l = l * alpha + (((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7])));
        if (warp_rescale) {
          // O is stable: the commit that signalled this S tracks the previous P V too
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            float o[32];
            tmem_ld32(o_addr + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] *= alpha;
            tmem_st32(o_addr + c * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar[P_FULL_A + t]);
      }
      if (!ok) break;
      // epilogue: O / l -> out[layer][token][head][:].  Each warp moves its 32
      // rows in four 32-column blocks: TMEM -> registers (one row per lane)
      // -> a 128B-swizzled 4 KiB staging block -> read back four rows per
      // instruction -> coalesced 128-byte row segments to global memory.
      if (!mbar_wait_warp(&bar[O_FULL_A + t], oc & 1)) { ok = false; break; }
      ++oc;
      tc_fence_after();
      const float inv = 1.f / l;
      const uint32_t stg = smem_u32(smem + OFF_OST + (warp - 4) * 4096);
      const int tok0 = I.qt * BM + quad * 32;
      float* out_base = p.out + (((size_t)I.layer_local * p.n_tokens + tok0) * p.heads + I.head_a + t) * HD;
      const size_t row_stride = (size_t)p.heads * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        float o[32];
        tmem_ld32(o_addr + c * 32, o);
        tmem_wait_ld();
        __syncwarp();  // the previous block's read-back is done
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          sts128(stg + lane * 128 + ((k ^ (lane & 7)) << 4), __float_as_uint(o[4 * k] * inv),
                 __float_as_uint(o[4 * k + 1] * inv), __float_as_uint(o[4 * k + 2] * inv),
                 __float_as_uint(o[4 * k + 3] * inv));
        }
        __syncwarp();
        const int k = lane & 7;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int r = 4 * i + (lane >> 3);
          const uint4 v = lds128(stg + r * 128 + ((k ^ (r & 7)) << 4));
          if (tok0 + r < p.n_tokens) {
            *reinterpret_cast<uint4*>(out_base + (size_t)r * row_stride + c * 32 + 4 * k) = v;
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar[O_EMPTY_A + t]);
    }
    if (!ok) { set_error(p.error, 17); *abort_flag = 1; }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

template <int HD, bool SPLIT>
cudaError_t launch_prefill_impl(const PrefillParams& p, int sm_count, cudaStream_t s) {
  static std::atomic<uint64_t> configured{0};  // one bit per device
  const cudaError_t e = set_smem_limit_once(configured, (const void*)prefill_tc_kernel<HD, SPLIT>, Plan<HD>::kSmemBytes);
  if (e != cudaSuccess) return e;
  const int grid = p.n_items < sm_count ? p.n_items : sm_count;
  prefill_tc_kernel<HD, SPLIT><<<grid, kThreads, Plan<HD>::kSmemBytes, s>>>(p);
  return cudaGetLastError();
}

}  // namespace

int prefill_items(int n_layers, int heads, int kv_heads, int n_tokens_padded, bool split) {
  const int G = heads / kv_heads;
  return n_layers * kv_heads * (split ? G : (G + 1) / 2) * (n_tokens_padded / BM);
}

cudaError_t launch_prefill_tc(const PrefillParams& p, int sm_count, cudaStream_t s) {
  if (p.head_dim == 128) {
    return p.split ? launch_prefill_impl<128, true>(p, sm_count, s) : launch_prefill_impl<128, false>(p, sm_count, s);
  }
  if (p.head_dim == 64) {
    return p.split ? launch_prefill_impl<64, true>(p, sm_count, s) : launch_prefill_impl<64, false>(p, sm_count, s);
  }
  return cudaErrorInvalidValue;
}

}  // namespace te
