// C-ABI layer of libtinyengine.so: argument validation with the reference's
// status codes, the device-resident engine and paged f16 KV cache, work
// decomposition for the kernels, and the two drop-in CPU-API functions.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/tinyengine.h"
#include "../../include/tinyengine_attn.h"
#include "te_internal.h"

extern "C" void te_host_rope_table(float* cos_table, float* sin_table, size_t first_position, size_t positions,
                                   size_t head_dim, float theta);

using namespace te;

struct te_attn_engine {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int sm_count = 148;
  uint32_t decode_chunk = 0;
  float* partials = nullptr;
  size_t partials_bytes = 0;
  uint32_t* counters = nullptr;
  size_t counters_count = 0;
  int* d_error = nullptr;
  void* io = nullptr;  // device staging for TE_ATTN_HOST_BUFFERS
  size_t io_bytes = 0;
  void* qh = nullptr;  // prefill: rotated f16 queries
  size_t qh_bytes = 0;
  uint32_t* tile_counter = nullptr;
  uint64_t launches = 0;
  std::string last_error;
  bool time_kernels = false;  // te_attn_engine_time_kernels
  bool kernel_timed = false;
  cudaEvent_t ev_k0 = nullptr, ev_k1 = nullptr;
  uint64_t wait_ns = 2000000000ull;  // bound of the exchange kernel's waits for other GPUs

  // Per-kernel device-time profile (te_attn_engine_profile, TINYENGINE_PROFILE=1):
  // an event pair around every launch, resolved when the engine synchronises.
  bool profile = false;
  bool profile_env = false;  // enabled by TINYENGINE_PROFILE: printed to stderr when the engine is freed
  struct ProfPair {
    int kind;
    cudaEvent_t a, b;
  };
  std::vector<ProfPair> prof_pending;
  std::vector<ProfPair> prof_free;
  double prof_ms[8] = {};  // per ProfKind
  uint64_t prof_calls[8] = {};
};

struct te_kv_cache {
  te_attn_engine* eng = nullptr;
  te_kv_cache_desc d{};
  uint32_t pages_per_seq = 0;
  uint16_t* k_pool = nullptr;
  uint16_t* v_pool = nullptr;
  int32_t* d_page_table = nullptr;
  std::vector<int32_t> h_page_table;  // [max_seqs][pages_per_seq], -1 = unmapped
  std::vector<uint32_t> contig;       // per sequence: leading pages that are consecutive in the pool
  std::vector<int64_t> len, offset;
  std::vector<int32_t> free_pages;
  float* d_cos = nullptr;
  float* d_sin = nullptr;
  CUtensorMap tmap_k{}, tmap_v{};
  // projection biases (te_kv_cache_set_qkv_bias): [layers][bias_heads * hd] for q,
  // [layers][kv_heads * hd] for k and v; null until set
  float* d_qb = nullptr;
  float* d_kb = nullptr;
  float* d_vb = nullptr;
  uint32_t bias_heads = 0;
};

struct te_attn_exchange {
  te_attn_engine* eng = nullptr;
  int world = 0, rank = 0, rows = 0, hd = 0, grid = 0;
  float* local = nullptr;                  // this rank's exchange area
  float* base[kMaxExchangeRanks] = {};     // every rank's area as mapped in this process
  bool connected = false;
};

namespace {

// Switches to a device for the duration of a call and restores the caller's.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

te_status fail(te_attn_engine* e, te_status st, const std::string& msg) {
  if (e) e->last_error = msg;
  return st;
}

te_status cuda_fail(te_attn_engine* e, cudaError_t err, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorString(err);
  if (e) e->last_error = m;
  return err == cudaErrorMemoryAllocation ? TE_STATUS_OUT_OF_MEMORY : TE_STATUS_RUNTIME_ERROR;
}

bool cuda_device_available() {
  int n = 0;
  return cudaGetDeviceCount(&n) == cudaSuccess && n > 0;
}

// Kernel families of the profile, in report order.
enum ProfKind {
  PK_DECODE = 0, PK_APPEND, PK_MERGE, PK_PREFILL_PREP, PK_PREFILL_ATTN, PK_MATVEC, PK_EXCHANGE, PK_STEP, PK_COUNT
};
const char* const kProfNames[PK_COUNT] = {"decode",       "append", "merge",   "prefill_prep",
                                          "prefill_attn", "matvec", "exchange", "step"};

// Opens a profiled launch: records the first event of a pair on the engine's
// stream and returns its slot, or -1 when profiling is off or the stream is
// being captured into a graph (event timing does not apply to replays).
int prof_begin(te_attn_engine* e, int kind) {
  if (!e->profile) return -1;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(e->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return -1;
  te_attn_engine::ProfPair pp;
  if (!e->prof_free.empty()) {
    pp = e->prof_free.back();
    e->prof_free.pop_back();
  } else if (cudaEventCreate(&pp.a) != cudaSuccess || cudaEventCreate(&pp.b) != cudaSuccess) {
    return -1;
  }
  pp.kind = kind;
  cudaEventRecord(pp.a, e->stream);
  e->prof_pending.push_back(pp);
  return (int)e->prof_pending.size() - 1;
}

void prof_end(te_attn_engine* e, int slot) {
  if (slot >= 0) cudaEventRecord(e->prof_pending[(size_t)slot].b, e->stream);
}

// Folds every completed pair into the per-kind totals (waits for none).
void prof_collect(te_attn_engine* e) {
  std::vector<te_attn_engine::ProfPair> keep;
  for (const auto& pp : e->prof_pending) {
    if (cudaEventQuery(pp.b) != cudaSuccess) {
      keep.push_back(pp);
      continue;
    }
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, pp.a, pp.b) == cudaSuccess) {
      e->prof_ms[pp.kind] += ms;
      e->prof_calls[pp.kind] += 1;
    }
    e->prof_free.push_back(pp);
  }
  e->prof_pending.swap(keep);
  (void)cudaGetLastError();  // a query of a not-yet-complete event is not an error
}

std::string prof_line(const te_attn_engine* e) {
  double total = 0.0;
  for (int k = 0; k < PK_COUNT; ++k) total += e->prof_ms[k];
  std::string out;
  char buf[96];
  std::snprintf(buf, sizeof(buf), "tinyengine_profile: device_ms=%.3f", total);
  out += buf;
  for (int k = 0; k < PK_COUNT; ++k) {
    std::snprintf(buf, sizeof(buf), " %s=%.3f/%llu", kProfNames[k], e->prof_ms[k],
                  (unsigned long long)e->prof_calls[k]);
    out += buf;
  }
  return out;
}

// Grows a device buffer; the stream is drained first so no queued kernel uses the old one.
cudaError_t grow(te_attn_engine* e, void** buf, size_t* cap, size_t need, bool zero) {
  if (need <= *cap) return cudaSuccess;
  cudaError_t err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return err;
  if (*buf) cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  // geometric growth: a call that needs slightly more never reallocates each time
  size_t sz = std::max(std::max(2 * need, 2 * *cap), (size_t)1 << 20);
  err = cudaMalloc(buf, sz);
  if (err != cudaSuccess) return err;
  if (zero) {
    err = cudaMemset(*buf, 0, sz);
    if (err != cudaSuccess) return err;
  }
  *cap = sz;
  return cudaSuccess;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

// 2-D f16 tensor map over [rows][cols] with a box of box_rows x 64 columns, 128B swizzle.
bool make_tmap_f16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Prefill queries [layers][tokens][heads][hd] f16 as a 4-D tensor map: one box
// is 64 tokens x 64 dims of one head (128B swizzle); tokens past the end read
// as zeros.
bool make_tmap_q_f16(CUtensorMap* m, const void* base, uint64_t hd, uint64_t heads, uint64_t tokens, uint64_t layers) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {hd, heads, tokens, layers};
  cuuint64_t strides[3] = {hd * 2, heads * hd * 2, tokens * heads * hd * 2};
  cuuint32_t box[4] = {64, 1, 64, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

size_t pool_row(const te_kv_cache* c, size_t layer, int32_t page, size_t kvh, size_t tok_in_page) {
  return ((layer * c->d.total_pages + (size_t)page) * c->d.kv_heads + kvh) * c->d.page_tokens + tok_in_page;
}

// Maps pages so that sequence `seq` can hold `tokens` tokens.
te_status ensure_pages(te_kv_cache* c, size_t seq, size_t tokens) {
  if (tokens > c->d.max_tokens_per_seq) {
    return fail(c->eng, TE_STATUS_INVALID_ARGUMENT, "sequence would exceed max_tokens_per_seq");
  }
  const size_t need = (tokens + c->d.page_tokens - 1) / c->d.page_tokens;
  int32_t* row = c->h_page_table.data() + seq * c->pages_per_seq;
  size_t first_new = need, last_new = 0;
  for (size_t i = 0; i < need; ++i) {
    if (row[i] >= 0) continue;
    if (c->free_pages.empty()) return fail(c->eng, TE_STATUS_OUT_OF_MEMORY, "KV page pool exhausted");
    row[i] = c->free_pages.back();
    c->free_pages.pop_back();
    first_new = std::min(first_new, i);
    last_new = i;
  }
  if (first_new < need) {
    cudaError_t err = cudaMemcpyAsync(c->d_page_table + seq * c->pages_per_seq + first_new, row + first_new,
                                      (last_new - first_new + 1) * sizeof(int32_t), cudaMemcpyHostToDevice,
                                      c->eng->stream);
    if (err != cudaSuccess) return cuda_fail(c->eng, err, "page table upload");
  }
  uint32_t& run = c->contig[seq];
  while (run < need && row[run] == row[0] + (int32_t)run) ++run;
  return TE_STATUS_OK;
}

// First page of `seq` when its pages covering `tokens` are consecutive in the
// pool (the kernel then computes page ids instead of reading the table), or -1.
int32_t contiguous_base(const te_kv_cache* c, size_t seq, size_t tokens) {
  const size_t need = (tokens + c->d.page_tokens - 1) / c->d.page_tokens;
  return need > 0 && c->contig[seq] >= need ? c->h_page_table[seq * c->pages_per_seq] : -1;
}

// Copies rows [n][kv_heads][hd] between a flat buffer and the paged pool.
te_status copy_rows(te_kv_cache* c, size_t layer, size_t seq, size_t t0, size_t n, uint16_t* pool, void* flat,
                    bool to_pool) {
  const size_t hd = c->d.head_dim, hkv = c->d.kv_heads, P = c->d.page_tokens;
  const int32_t* row = c->h_page_table.data() + seq * c->pages_per_seq;
  size_t t = t0;
  while (t < t0 + n) {
    const size_t pg = t / P, in_pg = t % P;
    const size_t m = std::min(P - in_pg, t0 + n - t);
    if (row[pg] < 0) return fail(c->eng, TE_STATUS_INVALID_ARGUMENT, "tokens outside the sequence's pages");
    for (size_t h = 0; h < hkv; ++h) {
      uint16_t* dev = pool + pool_row(c, layer, row[pg], h, in_pg) * hd;
      uint16_t* fl = reinterpret_cast<uint16_t*>(flat) + ((t - t0) * hkv + h) * hd;
      cudaError_t err = to_pool ? cudaMemcpy2DAsync(dev, hd * 2, fl, hkv * hd * 2, hd * 2, m, cudaMemcpyDefault,
                                                    c->eng->stream)
                                : cudaMemcpy2DAsync(fl, hkv * hd * 2, dev, hd * 2, hd * 2, m, cudaMemcpyDefault,
                                                    c->eng->stream);
      if (err != cudaSuccess) return cuda_fail(c->eng, err, "KV row copy");
    }
    t += m;
  }
  return TE_STATUS_OK;
}

}  // namespace

namespace te {
bool encode_tmap_f16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  return make_tmap_f16(m, base, rows, cols, box_rows);
}
}  // namespace te

// ===========================================================================
// tinyengine.h: version, status strings, drop-in CPU-API functions
// ===========================================================================

extern "C" {

TE_API const char* te_version(void) { return "0.1.0-b200-attn"; }

TE_API const char* te_strerror(te_status status) {
  switch (status) {
    case TE_STATUS_OK: return "ok";
    case TE_STATUS_INVALID_ARGUMENT: return "invalid argument";
    case TE_STATUS_IO_ERROR: return "I/O error";
    case TE_STATUS_UNSUPPORTED: return "unsupported";
    case TE_STATUS_OUT_OF_MEMORY: return "out of memory";
    case TE_STATUS_RUNTIME_ERROR: return "runtime error";
    default: return "unknown error";
  }
}

TE_API te_status te_rope_f32(float* values, size_t heads, size_t head_dim, size_t position, float theta) {
  // Validation order and codes: c/src/ops.c:302-304.
  if (values == NULL || heads == 0u || head_dim == 0u || (head_dim % 2u) != 0u || !(theta > 0.0f)) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  if (!cuda_device_available()) return TE_STATUS_UNSUPPORTED;
  const size_t half = head_dim / 2;
  std::vector<float> tab(2 * half);
  te_host_rope_table(tab.data(), tab.data() + half, position, 1, head_dim, theta);
  cudaStream_t s = cudaStreamPerThread;
  const size_t vbytes = heads * head_dim * sizeof(float);
  float* d = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void**>(&d), vbytes + 2 * half * sizeof(float), s) != cudaSuccess) {
    return TE_STATUS_OUT_OF_MEMORY;
  }
  float* dtab = d + heads * head_dim;
  te_status st = TE_STATUS_OK;
  if (cudaMemcpyAsync(d, values, vbytes, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaMemcpyAsync(dtab, tab.data(), 2 * half * sizeof(float), cudaMemcpyHostToDevice, s) != cudaSuccess ||
      launch_rope_rows(d, dtab, dtab + half, (int)heads, (int)head_dim, s) != cudaSuccess ||
      cudaMemcpyAsync(values, d, vbytes, cudaMemcpyDeviceToHost, s) != cudaSuccess) {
    st = TE_STATUS_RUNTIME_ERROR;
  }
  cudaFreeAsync(d, s);
  if (cudaStreamSynchronize(s) != cudaSuccess) st = TE_STATUS_RUNTIME_ERROR;
  return st;
}

TE_API te_status te_attention_decode_f32(const float* query, const float* key_cache, const float* value_cache,
                                         size_t position, size_t heads, size_t kv_heads, size_t head_dim,
                                         float* out) {
  // Validation order and codes: c/src/ops.c:333-339.
  if (query == NULL || key_cache == NULL || value_cache == NULL || out == NULL || heads == 0u || kv_heads == 0u ||
      head_dim == 0u || (heads % kv_heads) != 0u) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  if (position == SIZE_MAX) return TE_STATUS_UNSUPPORTED;
  if (!cuda_device_available()) return TE_STATUS_UNSUPPORTED;
  const size_t n = position + 1;
  if (n > (size_t)INT32_MAX || heads > 65535u) return TE_STATUS_UNSUPPORTED;
  cudaStream_t s = cudaStreamPerThread;
  const size_t qb = heads * head_dim * sizeof(float);
  const size_t kvb = n * kv_heads * head_dim * sizeof(float);
  const size_t scb = heads * n * sizeof(float);
  char* d = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void**>(&d), 2 * qb + 2 * kvb + scb, s) != cudaSuccess) {
    return TE_STATUS_OUT_OF_MEMORY;
  }
  float* dq = reinterpret_cast<float*>(d);
  float* dout = reinterpret_cast<float*>(d + qb);
  float* dk = reinterpret_cast<float*>(d + 2 * qb);
  float* dv = reinterpret_cast<float*>(d + 2 * qb + kvb);
  float* dsc = reinterpret_cast<float*>(d + 2 * qb + 2 * kvb);
  te_status st = TE_STATUS_OK;
  if (cudaMemcpyAsync(dq, query, qb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaMemcpyAsync(dk, key_cache, kvb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaMemcpyAsync(dv, value_cache, kvb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      launch_decode_f32_generic(dq, dk, dv, dsc, dout, n, (int)heads, (int)kv_heads, (int)head_dim, s) !=
          cudaSuccess ||
      cudaMemcpyAsync(out, dout, qb, cudaMemcpyDeviceToHost, s) != cudaSuccess) {
    st = TE_STATUS_RUNTIME_ERROR;
  }
  cudaFreeAsync(d, s);
  if (cudaStreamSynchronize(s) != cudaSuccess) st = TE_STATUS_RUNTIME_ERROR;
  return st;
}

// ===========================================================================
// tinyengine_attn.h: engine
// ===========================================================================

TE_API te_attn_options te_attn_default_options(void) {
  te_attn_options o;
  std::memset(&o, 0, sizeof(o));
  o.abi_version = TE_ATTN_ABI_VERSION;
  return o;
}

TE_API te_status te_attn_engine_create(const te_attn_options* options, te_attn_engine** out_engine) {
  if (options == NULL || out_engine == NULL) return TE_STATUS_INVALID_ARGUMENT;
  *out_engine = nullptr;
  if (options->abi_version != TE_ATTN_ABI_VERSION) return TE_STATUS_UNSUPPORTED;
  if (options->decode_chunk_tokens % kStageTokens != 0) return TE_STATUS_INVALID_ARGUMENT;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return TE_STATUS_UNSUPPORTED;
  if (options->device < 0 || options->device >= n) return TE_STATUS_INVALID_ARGUMENT;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, options->device) != cudaSuccess) return TE_STATUS_RUNTIME_ERROR;
  if (prop.major != 10) return TE_STATUS_UNSUPPORTED;  // built for sm_100a only
  DeviceGuard dg(options->device);
  te_attn_engine* e = new te_attn_engine();
  e->device = options->device;
  e->sm_count = prop.multiProcessorCount;
  e->decode_chunk = options->decode_chunk_tokens;
  if (options->stream) {
    e->stream = reinterpret_cast<cudaStream_t>(options->stream);
  } else {
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
      delete e;
      return TE_STATUS_RUNTIME_ERROR;
    }
    e->own_stream = true;
  }
  if (cudaMalloc(reinterpret_cast<void**>(&e->d_error), 64) != cudaSuccess ||
      cudaMemset(e->d_error, 0, 64) != cudaSuccess) {
    te_attn_engine_free(e);
    return TE_STATUS_OUT_OF_MEMORY;
  }
  e->tile_counter = reinterpret_cast<uint32_t*>(e->d_error + 4);
  const char* prof = std::getenv("TINYENGINE_PROFILE");
  if (prof && prof[0] && std::strcmp(prof, "0") != 0) e->profile = e->profile_env = true;
  *out_engine = e;
  return TE_STATUS_OK;
}

TE_API void te_attn_engine_free(te_attn_engine* e) {
  if (!e) return;
  {
    DeviceGuard dg(e->device);
    if (e->stream) cudaStreamSynchronize(e->stream);
    cudaFree(e->partials);
    cudaFree(e->counters);
    cudaFree(e->d_error);
    cudaFree(e->io);
    cudaFree(e->qh);
    if (e->ev_k0) cudaEventDestroy(e->ev_k0);
    if (e->ev_k1) cudaEventDestroy(e->ev_k1);
    prof_collect(e);
    if (e->profile_env) std::fprintf(stderr, "%s\n", prof_line(e).c_str());
    for (const auto& pp : e->prof_pending) {
      cudaEventDestroy(pp.a);
      cudaEventDestroy(pp.b);
    }
    for (const auto& pp : e->prof_free) {
      cudaEventDestroy(pp.a);
      cudaEventDestroy(pp.b);
    }
    if (e->own_stream && e->stream) cudaStreamDestroy(e->stream);
  }
  delete e;
}

TE_API te_status te_attn_engine_set_stream(te_attn_engine* e, void* stream) {
  if (!e) return TE_STATUS_INVALID_ARGUMENT;
  DeviceGuard dg(e->device);
  cudaStreamSynchronize(e->stream);
  if (e->own_stream) cudaStreamDestroy(e->stream);
  e->own_stream = false;
  e->stream = reinterpret_cast<cudaStream_t>(stream);
  if (!stream) {
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) return TE_STATUS_RUNTIME_ERROR;
    e->own_stream = true;
  }
  return TE_STATUS_OK;
}

TE_API void* te_attn_engine_stream(const te_attn_engine* e) { return e ? reinterpret_cast<void*>(e->stream) : nullptr; }

TE_API te_status te_attn_engine_synchronize(te_attn_engine* e) {
  if (!e) return TE_STATUS_INVALID_ARGUMENT;
  DeviceGuard dg(e->device);
  cudaError_t err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return cuda_fail(e, err, "stream synchronize");
  if (e->profile) prof_collect(e);
  int code = 0;
  err = cudaMemcpy(&code, e->d_error, sizeof(int), cudaMemcpyDeviceToHost);
  if (err != cudaSuccess) return cuda_fail(e, err, "error word read");
  if (code != 0) {
    cudaMemset(e->d_error, 0, sizeof(int));
    char buf[128];
    std::snprintf(buf, sizeof(buf), "device-side error %d (a bounded wait expired or a capacity check failed)", code);
    return fail(e, TE_STATUS_RUNTIME_ERROR, buf);
  }
  return TE_STATUS_OK;
}

TE_API const char* te_attn_engine_last_error(const te_attn_engine* e) {
  return e ? e->last_error.c_str() : "no engine";
}

TE_API uint64_t te_attn_engine_launch_count(const te_attn_engine* e) { return e ? e->launches : 0; }

TE_API te_status te_attn_engine_time_kernels(te_attn_engine* e, int enable) {
  if (!e) return TE_STATUS_INVALID_ARGUMENT;
  if (enable && !e->ev_k0) {
    DeviceGuard dg(e->device);
    if (cudaEventCreate(&e->ev_k0) != cudaSuccess || cudaEventCreate(&e->ev_k1) != cudaSuccess) {
      return fail(e, TE_STATUS_RUNTIME_ERROR, "event creation");
    }
  }
  e->time_kernels = enable != 0;
  e->kernel_timed = false;
  return TE_STATUS_OK;
}

TE_API te_status te_attn_engine_set_wait_limit(te_attn_engine* e, uint32_t milliseconds) {
  if (!e || milliseconds == 0 || milliseconds > 60000) return TE_STATUS_INVALID_ARGUMENT;
  e->wait_ns = (uint64_t)milliseconds * 1000000ull;
  return TE_STATUS_OK;
}

TE_API te_status te_attn_engine_profile(te_attn_engine* e, int enable) {
  if (!e) return TE_STATUS_INVALID_ARGUMENT;
  e->profile = enable != 0;
  return TE_STATUS_OK;
}

TE_API te_status te_attn_engine_profile_report(te_attn_engine* e, char* buf, size_t len) {
  if (!e || !buf || len == 0) return TE_STATUS_INVALID_ARGUMENT;
  DeviceGuard dg(e->device);
  cudaError_t err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return cuda_fail(e, err, "stream synchronize");
  prof_collect(e);
  const std::string line = prof_line(e);
  std::snprintf(buf, len, "%s", line.c_str());
  return line.size() < len ? TE_STATUS_OK : TE_STATUS_INVALID_ARGUMENT;
}

TE_API te_status te_attn_engine_last_kernel_ms(te_attn_engine* e, float* ms) {
  if (!e || !ms || !e->kernel_timed) return TE_STATUS_INVALID_ARGUMENT;
  DeviceGuard dg(e->device);
  cudaError_t err = cudaEventSynchronize(e->ev_k1);
  if (err == cudaSuccess) err = cudaEventElapsedTime(ms, e->ev_k0, e->ev_k1);
  return err == cudaSuccess ? TE_STATUS_OK : cuda_fail(e, err, "kernel timing");
}

// ===========================================================================
// KV cache
// ===========================================================================

TE_API te_kv_cache_desc te_kv_cache_default_desc(void) {
  te_kv_cache_desc d;
  std::memset(&d, 0, sizeof(d));
  d.abi_version = TE_ATTN_ABI_VERSION;
  d.layers = 1;
  d.max_seqs = 1;
  d.max_tokens_per_seq = 4096;
  d.kv_heads = 2;
  d.head_dim = 128;
  d.page_tokens = 128;
  d.rope_theta = 1000000.0f;
  return d;
}

TE_API te_status te_kv_cache_create(te_attn_engine* e, const te_kv_cache_desc* desc, te_kv_cache** out_cache) {
  if (!e || !desc || !out_cache) return TE_STATUS_INVALID_ARGUMENT;
  *out_cache = nullptr;
  if (desc->abi_version != TE_ATTN_ABI_VERSION) return fail(e, TE_STATUS_UNSUPPORTED, "cache desc ABI version");
  te_kv_cache_desc d = *desc;
  if (d.page_tokens == 0) d.page_tokens = 128;
  if (d.layers == 0 || d.max_seqs == 0 || d.max_tokens_per_seq == 0 || d.kv_heads == 0 ||
      !(d.rope_theta > 0.0f) || d.page_tokens % kStageTokens != 0) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "invalid cache description");
  }
  if (d.head_dim != 64 && d.head_dim != 128) return fail(e, TE_STATUS_UNSUPPORTED, "head_dim must be 64 or 128");
  const uint32_t pps = (d.max_tokens_per_seq + d.page_tokens - 1) / d.page_tokens;
  if (d.total_pages == 0) d.total_pages = d.max_seqs * pps;
  if (d.max_position == 0) d.max_position = d.max_tokens_per_seq;
  const uint64_t rows = (uint64_t)d.layers * d.total_pages * d.kv_heads * d.page_tokens;
  if (rows >= (1ull << 31)) return fail(e, TE_STATUS_UNSUPPORTED, "pool too large for 32-bit row coordinates");
  DeviceGuard dg(e->device);
  te_kv_cache* c = new te_kv_cache();
  c->eng = e;
  c->d = d;
  c->pages_per_seq = pps;
  const size_t pool_bytes = rows * d.head_dim * sizeof(uint16_t);
  const size_t half = d.head_dim / 2;
  cudaError_t err = cudaMalloc(reinterpret_cast<void**>(&c->k_pool), pool_bytes);
  if (err == cudaSuccess) err = cudaMalloc(reinterpret_cast<void**>(&c->v_pool), pool_bytes);
  if (err == cudaSuccess) err = cudaMemsetAsync(c->k_pool, 0, pool_bytes, e->stream);
  if (err == cudaSuccess) err = cudaMemsetAsync(c->v_pool, 0, pool_bytes, e->stream);
  if (err == cudaSuccess)
    err = cudaMalloc(reinterpret_cast<void**>(&c->d_page_table), (size_t)d.max_seqs * pps * sizeof(int32_t));
  if (err == cudaSuccess)
    err = cudaMalloc(reinterpret_cast<void**>(&c->d_cos), 2 * (size_t)d.max_position * half * sizeof(float));
  if (err != cudaSuccess) {
    te_kv_cache_free(c);
    return cuda_fail(e, err, "KV cache allocation");
  }
  c->d_sin = c->d_cos + (size_t)d.max_position * half;
  c->h_page_table.assign((size_t)d.max_seqs * pps, -1);
  c->contig.assign(d.max_seqs, 0);
  c->len.assign(d.max_seqs, 0);
  c->offset.assign(d.max_seqs, 0);
  c->free_pages.resize(d.total_pages);
  for (uint32_t i = 0; i < d.total_pages; ++i) c->free_pages[i] = (int32_t)(d.total_pages - 1 - i);
  std::vector<float> tab(2 * (size_t)d.max_position * half);
  te_host_rope_table(tab.data(), tab.data() + (size_t)d.max_position * half, 0, d.max_position, d.head_dim,
                     d.rope_theta);
  err = cudaMemcpy(c->d_cos, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice);
  if (err == cudaSuccess)
    err = cudaMemcpy(c->d_page_table, c->h_page_table.data(), c->h_page_table.size() * sizeof(int32_t),
                     cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) {
    te_kv_cache_free(c);
    return cuda_fail(e, err, "KV cache initialisation");
  }
  if (!make_tmap_f16(&c->tmap_k, c->k_pool, rows, d.head_dim, kStageTokens) ||
      !make_tmap_f16(&c->tmap_v, c->v_pool, rows, d.head_dim, kStageTokens)) {
    te_kv_cache_free(c);
    return fail(e, TE_STATUS_RUNTIME_ERROR, "cuTensorMapEncodeTiled failed");
  }
  *out_cache = c;
  return TE_STATUS_OK;
}

TE_API void te_kv_cache_free(te_kv_cache* c) {
  if (!c) return;
  {
    DeviceGuard dg(c->eng->device);
    cudaStreamSynchronize(c->eng->stream);
    cudaFree(c->k_pool);
    cudaFree(c->v_pool);
    cudaFree(c->d_page_table);
    cudaFree(c->d_cos);
    cudaFree(c->d_kb);  // the bias allocation (d_vb and d_qb point into it)
  }
  delete c;
}

TE_API te_status te_kv_cache_seq_reset(te_kv_cache* c, size_t seq, size_t position_offset) {
  if (!c || seq >= c->d.max_seqs) return TE_STATUS_INVALID_ARGUMENT;
  int32_t* row = c->h_page_table.data() + seq * c->pages_per_seq;
  for (uint32_t i = 0; i < c->pages_per_seq; ++i) {
    if (row[i] >= 0) c->free_pages.push_back(row[i]);
    row[i] = -1;
  }
  c->contig[seq] = 0;
  c->len[seq] = 0;
  c->offset[seq] = (int64_t)position_offset;
  // Device rows of unmapped entries are never read (reads stop at the length).
  return TE_STATUS_OK;
}

TE_API te_status te_kv_cache_seq_truncate(te_kv_cache* c, size_t seq, size_t length) {
  if (!c || seq >= c->d.max_seqs || length > (size_t)c->len[seq]) return TE_STATUS_INVALID_ARGUMENT;
  c->len[seq] = (int64_t)length;  // pages stay mapped; later appends overwrite the dropped tokens
  return TE_STATUS_OK;
}

TE_API te_status te_kv_cache_reserve(te_kv_cache* c, size_t seq, size_t tokens) {
  if (!c || seq >= c->d.max_seqs) return TE_STATUS_INVALID_ARGUMENT;
  DeviceGuard dg(c->eng->device);
  return ensure_pages(c, seq, tokens);
}

TE_API te_status te_kv_cache_seq_length(const te_kv_cache* c, size_t seq, size_t* out_length) {
  if (!c || !out_length || seq >= c->d.max_seqs) return TE_STATUS_INVALID_ARGUMENT;
  *out_length = (size_t)c->len[seq];
  return TE_STATUS_OK;
}

TE_API te_status te_kv_cache_write_f16(te_kv_cache* c, size_t layer, size_t seq, size_t token_begin,
                                       size_t n_tokens, const uint16_t* k, const uint16_t* v) {
  if (!c || !k || !v || layer >= c->d.layers || seq >= c->d.max_seqs || n_tokens == 0) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  DeviceGuard dg(c->eng->device);
  te_status st = ensure_pages(c, seq, token_begin + n_tokens);
  if (st != TE_STATUS_OK) return st;
  st = copy_rows(c, layer, seq, token_begin, n_tokens, c->k_pool, const_cast<uint16_t*>(k), true);
  if (st == TE_STATUS_OK) st = copy_rows(c, layer, seq, token_begin, n_tokens, c->v_pool, const_cast<uint16_t*>(v), true);
  if (st != TE_STATUS_OK) return st;
  c->len[seq] = std::max<int64_t>(c->len[seq], (int64_t)(token_begin + n_tokens));
  return TE_STATUS_OK;
}

TE_API te_status te_kv_cache_read_f16(te_kv_cache* c, size_t layer, size_t seq, size_t token_begin,
                                      size_t n_tokens, uint16_t* k, uint16_t* v) {
  if (!c || !k || !v || layer >= c->d.layers || seq >= c->d.max_seqs || n_tokens == 0) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  if (token_begin + n_tokens > (size_t)c->len[seq]) return fail(c->eng, TE_STATUS_INVALID_ARGUMENT, "read past length");
  DeviceGuard dg(c->eng->device);
  te_status st = copy_rows(c, layer, seq, token_begin, n_tokens, c->k_pool, k, false);
  if (st == TE_STATUS_OK) st = copy_rows(c, layer, seq, token_begin, n_tokens, c->v_pool, v, false);
  if (st != TE_STATUS_OK) return st;
  cudaError_t err = cudaStreamSynchronize(c->eng->stream);
  return err == cudaSuccess ? TE_STATUS_OK : cuda_fail(c->eng, err, "KV read");
}

TE_API te_status te_kv_cache_set_qkv_bias(te_kv_cache* c, size_t layer_begin, size_t n_layers, size_t heads,
                                          const float* q_bias, const float* k_bias, const float* v_bias) {
  if (!c || n_layers == 0 || heads == 0 || layer_begin + n_layers > c->d.layers) return TE_STATUS_INVALID_ARGUMENT;
  te_attn_engine* e = c->eng;
  const size_t hkv = c->d.kv_heads, hd = c->d.head_dim;
  if (heads % hkv != 0) return fail(e, TE_STATUS_INVALID_ARGUMENT, "heads must be a multiple of kv_heads");
  if (c->bias_heads != 0 && c->bias_heads != heads) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "heads differs from the first te_kv_cache_set_qkv_bias call");
  }
  DeviceGuard dg(e->device);
  const size_t L = c->d.layers;
  if (!c->d_qb) {
    // one allocation: q biases, then k, then v; zeros until set
    const size_t bytes = L * (heads + 2 * hkv) * hd * sizeof(float);
    cudaError_t err = cudaMalloc(&c->d_kb, bytes);
    if (err == cudaSuccess) err = cudaMemsetAsync(c->d_kb, 0, bytes, e->stream);
    if (err != cudaSuccess) {
      cudaFree(c->d_kb);
      c->d_kb = nullptr;
      return cuda_fail(e, err, "bias allocation");
    }
    c->d_vb = c->d_kb + L * hkv * hd;
    c->d_qb = c->d_vb + L * hkv * hd;
    c->bias_heads = (uint32_t)heads;
  }
  struct Part {
    float* dst;
    const float* src;
    size_t row;
  } parts[3] = {{c->d_qb, q_bias, heads * hd}, {c->d_kb, k_bias, hkv * hd}, {c->d_vb, v_bias, hkv * hd}};
  for (const Part& pt : parts) {
    float* dst = pt.dst + layer_begin * pt.row;
    const size_t bytes = n_layers * pt.row * sizeof(float);
    const cudaError_t err = pt.src ? cudaMemcpyAsync(dst, pt.src, bytes, cudaMemcpyDefault, e->stream)
                                   : cudaMemsetAsync(dst, 0, bytes, e->stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "bias upload");
  }
  const cudaError_t err = cudaStreamSynchronize(e->stream);
  return err == cudaSuccess ? TE_STATUS_OK : cuda_fail(e, err, "bias upload");
}

// ===========================================================================
// Compute
// ===========================================================================

TE_API te_status te_kv_append_rope(te_kv_cache* c, size_t layer_begin, size_t n_layers, size_t seq, const void* k,
                                   const void* v, size_t n_tokens, uint32_t flags) {
  if (!c || !k || !v || n_layers == 0 || n_tokens == 0 || layer_begin + n_layers > c->d.layers ||
      seq >= c->d.max_seqs) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  if (flags & ~(TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16 | TE_ATTN_NO_ROPE | TE_ATTN_QKV_BIAS)) {
    return fail(c->eng, TE_STATUS_INVALID_ARGUMENT, "unsupported flags for te_kv_append_rope");
  }
  if ((flags & TE_ATTN_QKV_BIAS) && !c->d_kb) {
    return fail(c->eng, TE_STATUS_INVALID_ARGUMENT, "TE_ATTN_QKV_BIAS before te_kv_cache_set_qkv_bias");
  }
  te_attn_engine* e = c->eng;
  if ((reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15u) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "k and v must be 16-byte aligned");
  }
  DeviceGuard dg(e->device);
  const int64_t first = c->len[seq];
  if ((uint64_t)(c->offset[seq] + first + n_tokens) > c->d.max_position) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "RoPE position beyond max_position");
  }
  te_status st = ensure_pages(c, seq, (size_t)first + n_tokens);
  if (st != TE_STATUS_OK) return st;
  AppendParams p{};
  p.k = k;
  p.v = v;
  p.k_pool = c->k_pool;
  p.v_pool = c->v_pool;
  p.page_row = c->d_page_table + seq * c->pages_per_seq;
  p.rope_cos = c->d_cos;
  p.rope_sin = c->d_sin;
  if (flags & TE_ATTN_QKV_BIAS) {
    p.k_bias = c->d_kb;
    p.v_bias = c->d_vb;
  }
  p.input_f16 = (flags & TE_ATTN_INPUT_F16) ? 1 : 0;
  p.rope = (flags & TE_ATTN_NO_ROPE) ? 0 : 1;
  p.n_layers = (int32_t)n_layers;
  p.layer_begin = (int32_t)layer_begin;
  p.n_tokens = (int32_t)n_tokens;
  p.first_index = (int32_t)first;
  p.first_pos = (int32_t)(c->offset[seq] + first);
  p.kv_heads = (int32_t)c->d.kv_heads;
  p.head_dim = (int32_t)c->d.head_dim;
  p.num_pages = (int32_t)c->d.total_pages;
  p.page_tokens = (int32_t)c->d.page_tokens;
  const int prof = prof_begin(e, PK_APPEND);
  cudaError_t err = launch_append_rope(p, e->stream);
  prof_end(e, prof);
  if (err != cudaSuccess) return cuda_fail(e, err, "append kernel launch");
  e->launches++;
  if (flags & TE_ATTN_ADVANCE) c->len[seq] = first + (int64_t)n_tokens;
  return TE_STATUS_OK;
}

// The decode call; with an exchange x (one sequence, no host buffers or
// public partial records) the records go to x's area and the kernel runs the
// fused KV-split exchange.
static te_status decode_call(te_kv_cache* c, size_t layer_begin, size_t n_layers, const uint32_t* seq_ids,
                             size_t n_seqs, const int64_t* q_positions, const float* q, const float* k_new,
                             const float* v_new, size_t heads, float* out, uint32_t flags, te_attn_exchange* x) {
  if (!c || !seq_ids || !q || !out || n_layers == 0 || n_seqs == 0 || heads == 0 ||
      layer_begin + n_layers > c->d.layers || (k_new == NULL) != (v_new == NULL)) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  te_attn_engine* e = c->eng;
  if (flags & ~(TE_ATTN_ADVANCE | TE_ATTN_PARTIAL | TE_ATTN_NO_ROPE | TE_ATTN_HOST_BUFFERS | TE_ATTN_QKV_BIAS)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "unsupported flags for te_attention_decode");
  }
  const size_t hkv = c->d.kv_heads, hd = c->d.head_dim;
  if (heads % hkv != 0) return fail(e, TE_STATUS_INVALID_ARGUMENT, "heads must be a multiple of kv_heads");
  if ((flags & TE_ATTN_QKV_BIAS) && (!c->d_qb || c->bias_heads != heads)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "TE_ATTN_QKV_BIAS needs te_kv_cache_set_qkv_bias with these heads");
  }
  const size_t G = heads / hkv;
  if (G > 16) return fail(e, TE_STATUS_UNSUPPORTED, "more than 16 query heads per kv head");
  if (n_seqs > c->d.max_seqs) return TE_STATUS_INVALID_ARGUMENT;
  const bool append = k_new != NULL;
  if (!(flags & TE_ATTN_HOST_BUFFERS) &&
      ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) &
       15u)) {
    // the kernel copies query and new k/v rows with 16-byte bulk copies
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "q, k_new and v_new must be 16-byte aligned");
  }
  DeviceGuard dg(e->device);

  // Per-sequence work, validated before anything is queued.
  std::vector<SeqEntry> ent(n_seqs);
  std::vector<char> seen(c->d.max_seqs, 0);
  size_t max_len = 0;
  for (size_t i = 0; i < n_seqs; ++i) {
    const uint32_t s = seq_ids[i];
    if (s >= c->d.max_seqs || seen[s]) return fail(e, TE_STATUS_INVALID_ARGUMENT, "bad or repeated sequence id");
    seen[s] = 1;
    const int64_t len = c->len[s] + (append ? 1 : 0);
    if (len <= 0) return fail(e, TE_STATUS_INVALID_ARGUMENT, "decode over an empty sequence");
    if ((uint64_t)len > c->d.max_tokens_per_seq) return fail(e, TE_STATUS_INVALID_ARGUMENT, "sequence full");
    const int64_t qpos = q_positions ? q_positions[i] : c->offset[s] + len - 1;
    const int64_t npos = append ? c->offset[s] + len - 1 : -1;
    if (qpos < 0 || (uint64_t)qpos >= c->d.max_position || (uint64_t)(npos + 1) > c->d.max_position) {
      return fail(e, TE_STATUS_INVALID_ARGUMENT, "RoPE position beyond max_position");
    }
    ent[i].slot = (int32_t)s;
    ent[i].len = (int32_t)len;
    ent[i].q_pos = (int32_t)qpos;
    ent[i].new_pos = (int32_t)npos;
    max_len = std::max(max_len, (size_t)len);
  }
  if (append) {
    for (size_t i = 0; i < n_seqs; ++i) {
      te_status st = ensure_pages(c, seq_ids[i], (size_t)ent[i].len);
      if (st != TE_STATUS_OK) return st;
    }
  }
  for (size_t i = 0; i < n_seqs; ++i) ent[i].page_base = contiguous_base(c, seq_ids[i], (size_t)ent[i].len);

  // Device staging for host buffers.
  const size_t q_elems = n_layers * n_seqs * heads * hd;
  const size_t kv_elems = n_layers * n_seqs * hkv * hd;
  const size_t out_elems = n_layers * n_seqs * heads * (hd + ((flags & TE_ATTN_PARTIAL) ? 2 : 0));
  const float* dq = q;
  const float* dk = k_new;
  const float* dv = v_new;
  float* dout = out;
  // With host buffers, an `out` in pinned host memory that the device can
  // address (cudaHostAlloc / cudaMallocHost memory, under unified addressing)
  // is written by the kernel directly: no device-to-host copy afterwards.
  bool out_mapped = false;
  if (flags & TE_ATTN_HOST_BUFFERS) {
    cudaPointerAttributes pa{};
    if (cudaPointerGetAttributes(&pa, out) == cudaSuccess && pa.type == cudaMemoryTypeHost && pa.devicePointer &&
        (reinterpret_cast<uintptr_t>(pa.devicePointer) & 15u) == 0) {
      out_mapped = true;
    }
    (void)cudaGetLastError();  // an unregistered (pageable) pointer is not an error here
    const size_t need = (q_elems + 2 * kv_elems + out_elems) * sizeof(float);
    cudaError_t err = grow(e, &e->io, &e->io_bytes, need, false);
    if (err != cudaSuccess) return cuda_fail(e, err, "staging allocation");
    float* base = reinterpret_cast<float*>(e->io);
    float* sq = base;
    float* sk = sq + q_elems;
    float* sv = sk + kv_elems;
    dout = sv + kv_elems;
    // Inputs in pinned host memory the device can address, 16-byte aligned and
    // sized: one gather kernel reads them over PCIe (instead of one copy
    // operation per buffer); otherwise ordinary copies.
    GatherParams gp{};
    const void* srcs[3] = {q, k_new, v_new};
    float* dsts[3] = {sq, sk, sv};
    const size_t bytes[3] = {q_elems * sizeof(float), kv_elems * sizeof(float), kv_elems * sizeof(float)};
    bool mapped = true;
    for (int i = 0; i < (append ? 3 : 1) && mapped; ++i) {
      cudaPointerAttributes pa{};
      mapped = cudaPointerGetAttributes(&pa, srcs[i]) == cudaSuccess && pa.type == cudaMemoryTypeHost &&
               pa.devicePointer && ((reinterpret_cast<uintptr_t>(pa.devicePointer) | bytes[i]) & 15u) == 0;
      if (mapped) {
        gp.src[gp.n] = pa.devicePointer;
        gp.dst[gp.n] = dsts[i];
        gp.chunks[gp.n] = bytes[i] / 16;
        ++gp.n;
      }
    }
    (void)cudaGetLastError();  // an unregistered (pageable) pointer is not an error here
    if (mapped) {
      err = launch_gather_host(gp, e->stream);
      if (err == cudaSuccess) e->launches++;
    } else {
      err = cudaMemcpyAsync(sq, q, q_elems * sizeof(float), cudaMemcpyHostToDevice, e->stream);
      if (err == cudaSuccess && append) err = cudaMemcpyAsync(sk, k_new, kv_elems * sizeof(float), cudaMemcpyHostToDevice, e->stream);
      if (err == cudaSuccess && append) err = cudaMemcpyAsync(sv, v_new, kv_elems * sizeof(float), cudaMemcpyHostToDevice, e->stream);
    }
    if (err != cudaSuccess) return cuda_fail(e, err, "input upload");
    dq = sq;
    dk = append ? sk : nullptr;
    dv = append ? sv : nullptr;
    if (out_mapped) {
      cudaPointerAttributes pa{};
      cudaPointerGetAttributes(&pa, out);
      dout = static_cast<float*>(pa.devicePointer);
    }
  }

  DecodeParams p;
  std::memset(&p, 0, sizeof(p));
  p.tmap_k = c->tmap_k;
  p.tmap_v = c->tmap_v;
  p.page_table = c->d_page_table;
  p.q = dq;
  p.k_new = dk;
  p.v_new = dv;
  p.out = dout;
  p.k_pool = c->k_pool;
  p.v_pool = c->v_pool;
  p.rope_cos = c->d_cos;
  p.rope_sin = c->d_sin;
  if (flags & TE_ATTN_QKV_BIAS) {
    p.q_bias = c->d_qb;
    p.k_bias = c->d_kb;
    p.v_bias = c->d_vb;
  }
  p.error = e->d_error;
  p.seq_total = (int32_t)n_seqs;
  p.layer_begin = (int32_t)layer_begin;
  p.n_layers = (int32_t)n_layers;
  p.kv_heads = (int32_t)hkv;
  p.group = (int32_t)G;
  p.num_pages = (int32_t)c->d.total_pages;
  p.page_tokens = (int32_t)c->d.page_tokens;
  p.max_pages_per_seq = (int32_t)c->pages_per_seq;
  p.rope = (flags & TE_ATTN_NO_ROPE) ? 0 : 1;
  p.partial_out = (flags & TE_ATTN_PARTIAL) ? 1 : 0;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)hd));
  if (x) {
    const size_t push = exchange_area_bytes(x->world, x->rows, x->hd, x->grid);
    const FusedLayout f = fused_layout(push, x->world, x->rows, x->hd);
    p.partial_out = 2;
    p.out = reinterpret_cast<float*>(reinterpret_cast<char*>(x->local) + f.rec);
    p.xch_world = x->world;
    p.xch_rank = x->rank;
    p.xch_rows = x->rows;
    p.xch_wait_ns = e->wait_ns;
    for (int w = 0; w < x->world; ++w) {
      char* b = reinterpret_cast<char*>(x->base[w]);
      p.xch_rec[w] = reinterpret_cast<float*>(b + f.rec);
      p.xch_cnt[w] = reinterpret_cast<uint32_t*>(b + f.cnt);
    }
    p.xch_out = reinterpret_cast<float*>(reinterpret_cast<char*>(x->local) + f.out);
    p.xch_done = reinterpret_cast<uint32_t*>(reinterpret_cast<char*>(x->local) + f.done);
  }

  // Stream-K split over at most one CTA per SM, or over ranges of about
  // decode_chunk_tokens tokens when the engine was given that hint.
  for (size_t base = 0; base < n_seqs; base += kMaxParamSeqs) {
    const size_t nb = std::min<size_t>(kMaxParamSeqs, n_seqs - base);
    for (size_t i = 0; i < nb; ++i) p.seqs[i] = ent[base + i];
    p.n_seqs = (int32_t)nb;
    p.seq_base = (int32_t)base;
    long long max_grid = e->sm_count;
    if (e->decode_chunk) {
      long long tokens = 0;
      for (size_t i = 0; i < nb; ++i) tokens += p.seqs[i].len;
      tokens *= (long long)(n_layers * hkv);
      max_grid = std::min<long long>(max_grid, std::max<long long>(1, (tokens + e->decode_chunk - 1) / e->decode_chunk));
    }
    plan_stream_k(p, max_grid);
    if (!e->decode_chunk) plan_cluster(p, e->sm_count);
    auto launch = [&]() -> te_status {
      const size_t part_bytes = (size_t)p.grid * p.max_segs * G * decode_scratch_rec((int)hd) * sizeof(float);
      cudaError_t err = grow(e, reinterpret_cast<void**>(&e->partials), &e->partials_bytes, part_bytes, false);
      if (err == cudaSuccess) {
        size_t bytes = e->counters_count * sizeof(uint32_t);
        err = grow(e, reinterpret_cast<void**>(&e->counters), &bytes, n_layers * hkv * nb * sizeof(uint32_t), true);
        e->counters_count = bytes / sizeof(uint32_t);
      }
      if (err != cudaSuccess) return cuda_fail(e, err, "decode scratch allocation");
      p.partials = e->partials;
      p.counters = e->counters;
      const int prof = prof_begin(e, PK_DECODE);
      err = launch_decode_f16(p, (int)hd, e->stream);
      prof_end(e, prof);
      if (err != cudaSuccess) return cuda_fail(e, err, "decode kernel launch");
      return TE_STATUS_OK;
    };
    te_status st = launch();
    if (st != TE_STATUS_OK && p.cluster_k > 1) {
      // The device could not schedule the clusters (a launch-time, non-sticky
      // error): the stream-K split instead.
      (void)cudaGetLastError();
      plan_stream_k(p, max_grid);
      p.cluster_k = 0;
      st = launch();
    }
    if (st != TE_STATUS_OK) return st;
    e->launches++;
  }

  if (flags & TE_ATTN_HOST_BUFFERS) {
    cudaError_t err = out_mapped ? cudaSuccess
                                 : cudaMemcpyAsync(out, dout, out_elems * sizeof(float), cudaMemcpyDeviceToHost,
                                                   e->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "output download");
  }
  if (append && (flags & TE_ATTN_ADVANCE)) {
    for (size_t i = 0; i < n_seqs; ++i) c->len[seq_ids[i]] += 1;
  }
  return TE_STATUS_OK;
}

TE_API te_status te_attention_decode(te_kv_cache* c, size_t layer_begin, size_t n_layers, const uint32_t* seq_ids,
                                     size_t n_seqs, const int64_t* q_positions, const float* q, const float* k_new,
                                     const float* v_new, size_t heads, float* out, uint32_t flags) {
  return decode_call(c, layer_begin, n_layers, seq_ids, n_seqs, q_positions, q, k_new, v_new, heads, out, flags,
                     nullptr);
}

TE_API te_status te_attention_decode_kv_split(te_attn_exchange* x, te_kv_cache* c, size_t layer_begin,
                                              size_t n_layers, size_t seq, int64_t q_position, const float* q,
                                              const float* k_new, const float* v_new, size_t heads,
                                              uint32_t flags) {
  if (!x || !c || c->eng != x->eng || !q) return TE_STATUS_INVALID_ARGUMENT;
  te_attn_engine* e = x->eng;
  if (!x->connected) return fail(e, TE_STATUS_INVALID_ARGUMENT, "exchange not connected");
  if (flags & ~(TE_ATTN_ADVANCE | TE_ATTN_NO_ROPE | TE_ATTN_QKV_BIAS)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "unsupported flags for te_attention_decode_kv_split");
  }
  if (n_layers * heads != (size_t)x->rows || c->d.head_dim != (uint32_t)x->hd) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "the exchange was created for other rows or head_dim");
  }
  if (seq > UINT32_MAX) return TE_STATUS_INVALID_ARGUMENT;
  const uint32_t sid = (uint32_t)seq;
  const int64_t qp = q_position;
  float* rec = reinterpret_cast<float*>(x->local);  // placeholder: decode_call writes to the exchange's records
  return decode_call(c, layer_begin, n_layers, &sid, 1, q_position >= 0 ? &qp : nullptr, q, k_new, v_new, heads,
                     rec, flags, x);
}

TE_API te_status te_attn_exchange_output(te_attn_exchange* x, float** out) {
  if (!x || !out) return TE_STATUS_INVALID_ARGUMENT;
  const size_t push = exchange_area_bytes(x->world, x->rows, x->hd, x->grid);
  *out = reinterpret_cast<float*>(reinterpret_cast<char*>(x->local) + fused_layout(push, x->world, x->rows, x->hd).out);
  return TE_STATUS_OK;
}

TE_API te_status te_attention_merge_partials(te_attn_engine* e, const float* partials, size_t n_parts, size_t rows,
                                             size_t head_dim, float* out, uint32_t flags) {
  if (!e || !partials || !out || n_parts == 0 || rows == 0 || head_dim == 0) return TE_STATUS_INVALID_ARGUMENT;
  if (flags & ~TE_ATTN_PARTIAL) return fail(e, TE_STATUS_INVALID_ARGUMENT, "unsupported flags for merge");
  if (rows > (size_t)INT32_MAX) return TE_STATUS_UNSUPPORTED;
  DeviceGuard dg(e->device);
  const int prof = prof_begin(e, PK_MERGE);
  cudaError_t err = launch_merge_partials(partials, (int)n_parts, (int)rows, (int)head_dim, out,
                                          (flags & TE_ATTN_PARTIAL) ? 1 : 0, e->stream);
  prof_end(e, prof);
  if (err != cudaSuccess) return cuda_fail(e, err, "merge kernel launch");
  e->launches++;
  return TE_STATUS_OK;
}

TE_API te_status te_matvec_gguf(te_attn_engine* e, uint32_t quant, const void* w, size_t rows, size_t cols,
                                const float* x, size_t n_vectors, float* y, uint32_t flags) {
  if (!e || !w || !x || !y || rows == 0 || cols == 0 || cols % 32 != 0 || n_vectors == 0 || n_vectors > 8 ||
      (quant != TE_ATTN_QUANT_GGUF_Q4_0 && quant != TE_ATTN_QUANT_GGUF_Q8_0) || (flags & ~TE_ATTN_ACCUMULATE)) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15u) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "w and x must be 16-byte aligned");
  }
  const int block_bytes = quant == TE_ATTN_QUANT_GGUF_Q4_0 ? 18 : 34;
  const size_t rb = cols / 32 * block_bytes;
  if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX || 2 * (rb + 48) + 1280 > 227 * 1024) {  // two stages of one row
    return fail(e, TE_STATUS_UNSUPPORTED, "matrix rows too long to stage");
  }
  DeviceGuard dg(e->device);
  GemvParams p{};
  p.w = w;
  p.x = x;
  p.y = y;
  p.rows = (int32_t)rows;
  p.cols = (int32_t)cols;
  p.accumulate = (flags & TE_ATTN_ACCUMULATE) ? 1 : 0;
  p.error = e->d_error;
  const int prof = prof_begin(e, PK_MATVEC);
  const cudaError_t err = launch_gemv_gguf(p, block_bytes, (int)n_vectors, e->sm_count, e->stream);
  prof_end(e, prof);
  if (err != cudaSuccess) return cuda_fail(e, err, "matvec kernel launch");
  e->launches++;
  return TE_STATUS_OK;
}

TE_API te_status te_matvec_gguf_fused(te_attn_engine* e, uint32_t quant, const void* w, size_t rows, size_t cols,
                                      const float* x, size_t n_vectors, const float* norm_weight, float eps, float* y,
                                      uint32_t flags) {
  const uint32_t pro = flags & (TE_ATTN_RMSNORM_INPUT | TE_ATTN_SWIGLU_INPUT);
  if (!e || !w || !x || !y || rows == 0 || cols == 0 || cols % 32 != 0 || n_vectors == 0 || n_vectors > 8 ||
      (quant != TE_ATTN_QUANT_GGUF_Q4_0 && quant != TE_ATTN_QUANT_GGUF_Q8_0) ||
      (flags & ~(TE_ATTN_ACCUMULATE | TE_ATTN_RMSNORM_INPUT | TE_ATTN_SWIGLU_INPUT)) ||
      (pro != TE_ATTN_RMSNORM_INPUT && pro != TE_ATTN_SWIGLU_INPUT)) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  if (pro == TE_ATTN_RMSNORM_INPUT && (!norm_weight || !(eps > 0.0f))) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "RMSNorm input needs its weight and eps > 0");
  }
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) |
       (pro == TE_ATTN_RMSNORM_INPUT ? reinterpret_cast<uintptr_t>(norm_weight) : 0u)) & 15u) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "w, x and norm_weight must be 16-byte aligned");
  }
  const int block_bytes = quant == TE_ATTN_QUANT_GGUF_Q4_0 ? 18 : 34;
  const size_t rb = cols / 32 * block_bytes;
  if (rows > (size_t)INT32_MAX || cols > (size_t)INT32_MAX / 2 || 2 * (rb + 48) + 1280 > 227 * 1024) {
    return fail(e, TE_STATUS_UNSUPPORTED, "matrix rows too long to stage");
  }
  DeviceGuard dg(e->device);
  GemvParams p{};
  p.w = w;
  p.x = x;
  p.y = y;
  p.rows = (int32_t)rows;
  p.cols = (int32_t)cols;
  p.accumulate = (flags & TE_ATTN_ACCUMULATE) ? 1 : 0;
  p.error = e->d_error;
  p.prologue = pro == TE_ATTN_RMSNORM_INPUT ? 1 : 2;
  p.norm_w = norm_weight;
  p.eps = eps;
  const int prof = prof_begin(e, PK_MATVEC);
  const cudaError_t err = launch_gemv_gguf(p, block_bytes, (int)n_vectors, e->sm_count, e->stream);
  prof_end(e, prof);
  if (err != cudaSuccess) return cuda_fail(e, err, "matvec kernel launch");
  e->launches++;
  return TE_STATUS_OK;
}

static_assert(sizeof(cudaIpcMemHandle_t) == TE_ATTN_IPC_HANDLE_BYTES, "IPC handle size");

TE_API te_status te_attn_exchange_create(te_attn_engine* e, size_t world, size_t rank, size_t rows, size_t head_dim,
                                         te_attn_exchange** out, unsigned char* ipc_handle) {
  if (!e || !out || !ipc_handle || world < 2 || world > (size_t)kMaxExchangeRanks || rank >= world || rows == 0 ||
      rows > (1u << 20) || (head_dim != 64 && head_dim != 128)) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  DeviceGuard dg(e->device);
  te_attn_exchange* x = new te_attn_exchange();
  x->eng = e;
  x->world = (int)world;
  x->rank = (int)rank;
  x->rows = (int)rows;
  x->hd = (int)head_dim;
  x->grid = exchange_grid((int)rows);
  const size_t bytes = fused_layout(exchange_area_bytes(x->world, x->rows, x->hd, x->grid), x->world, x->rows, x->hd).end;
  cudaError_t err = cudaMalloc(&x->local, bytes);
  if (err == cudaSuccess) err = cudaMemset(x->local, 0, bytes);
  cudaIpcMemHandle_t h;
  if (err == cudaSuccess) err = cudaIpcGetMemHandle(&h, x->local);
  if (err != cudaSuccess) {
    cudaFree(x->local);
    delete x;
    return cuda_fail(e, err, "exchange area");
  }
  std::memcpy(ipc_handle, &h, sizeof(h));
  x->base[x->rank] = x->local;
  *out = x;
  return TE_STATUS_OK;
}

TE_API te_status te_attn_exchange_connect(te_attn_exchange* x, const unsigned char* handles) {
  if (!x || !handles || x->connected) return TE_STATUS_INVALID_ARGUMENT;
  DeviceGuard dg(x->eng->device);
  for (int w = 0; w < x->world; ++w) {
    if (w == x->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles + (size_t)w * TE_ATTN_IPC_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    const cudaError_t err = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) {
      for (int v = 0; v < w; ++v) {
        if (v != x->rank && x->base[v]) cudaIpcCloseMemHandle(x->base[v]);
        if (v != x->rank) x->base[v] = nullptr;
      }
      return cuda_fail(x->eng, err, "exchange peer mapping");
    }
    x->base[w] = static_cast<float*>(ptr);
  }
  x->connected = true;
  return TE_STATUS_OK;
}

TE_API te_status te_attn_exchange_merge(te_attn_exchange* x, const float* partial, float* out) {
  if (!x || !partial || !out) return TE_STATUS_INVALID_ARGUMENT;
  if (!x->connected) return fail(x->eng, TE_STATUS_INVALID_ARGUMENT, "exchange not connected");
  if ((reinterpret_cast<uintptr_t>(partial) | reinterpret_cast<uintptr_t>(out)) & 7u) {
    return fail(x->eng, TE_STATUS_INVALID_ARGUMENT, "partial and out must be 8-byte aligned");
  }
  te_attn_engine* e = x->eng;
  DeviceGuard dg(e->device);
  ExchangeParams p{};
  p.partial = partial;
  p.out = out;
  for (int w = 0; w < x->world; ++w) p.base[w] = x->base[w];
  const size_t data_floats = 2ull * x->world * x->rows * (x->hd + 2);
  p.steps = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned long long*>(x->local + data_floats) + 2 * x->grid);
  p.error = e->d_error;
  p.world = x->world;
  p.rank = x->rank;
  p.rows = x->rows;
  p.head_dim = x->hd;
  p.grid = x->grid;
  p.rows_per_cta = (x->rows + x->grid - 1) / x->grid;
  p.wait_ns = e->wait_ns;
  const int prof = prof_begin(e, PK_EXCHANGE);
  const cudaError_t err = launch_exchange_merge(p, e->stream);
  prof_end(e, prof);
  if (err != cudaSuccess) return cuda_fail(e, err, "exchange kernel launch");
  e->launches++;
  return TE_STATUS_OK;
}

TE_API void te_attn_exchange_free(te_attn_exchange* x) {
  if (!x) return;
  {
    DeviceGuard dg(x->eng->device);
    cudaStreamSynchronize(x->eng->stream);
    for (int w = 0; w < x->world; ++w) {
      if (w != x->rank && x->base[w]) cudaIpcCloseMemHandle(x->base[w]);
    }
    cudaFree(x->local);
  }
  delete x;
}

TE_API te_status te_attention_prefill(te_kv_cache* c, size_t layer_begin, size_t n_layers, size_t seq,
                                      const void* q, const void* k, const void* v, size_t n_tokens, size_t heads,
                                      float* out, uint32_t flags) {
  if (!c || !q || !k || !v || !out || n_layers == 0 || n_tokens == 0 || heads == 0 ||
      layer_begin + n_layers > c->d.layers || seq >= c->d.max_seqs) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  te_attn_engine* e = c->eng;
  if (flags & ~(TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16 | TE_ATTN_HOST_BUFFERS | TE_ATTN_NO_ROPE | TE_ATTN_QKV_BIAS |
                TE_ATTN_EXACT_Q)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "unsupported flags for te_attention_prefill");
  }
  const size_t hkv = c->d.kv_heads, hd = c->d.head_dim;
  if (heads % hkv != 0) return fail(e, TE_STATUS_INVALID_ARGUMENT, "heads must be a multiple of kv_heads");
  const bool bias = (flags & TE_ATTN_QKV_BIAS) != 0;
  if (bias && (!c->d_qb || c->bias_heads != heads)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "TE_ATTN_QKV_BIAS needs te_kv_cache_set_qkv_bias with these heads");
  }
  if (!(flags & TE_ATTN_HOST_BUFFERS) &&
      ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
        reinterpret_cast<uintptr_t>(out)) & 15u)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "q, k, v and out must be 16-byte aligned");
  }
  const size_t q_offset = (size_t)c->len[seq];
  const size_t total = q_offset + n_tokens;
  if (total > c->d.max_tokens_per_seq) return fail(e, TE_STATUS_INVALID_ARGUMENT, "sequence would exceed max_tokens_per_seq");
  if ((uint64_t)(c->offset[seq] + total) > c->d.max_position) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "RoPE position beyond max_position");
  }
  // The kernel multiplies f16 queries.  f16 inputs without RoPE or bias are
  // read as they are (exact); otherwise the prepared query is fp32 and enters
  // the tensor cores as hi + lo f16 parts (split) -- always for fp32 inputs,
  // for f16 inputs when TE_ATTN_EXACT_Q asks -- or rounded once to f16.
  const bool input_f16 = (flags & TE_ATTN_INPUT_F16) != 0;
  const bool with_q = !(input_f16 && (flags & TE_ATTN_NO_ROPE) && !bias);
  const bool split = with_q && (!input_f16 || (flags & TE_ATTN_EXACT_Q));
  const size_t q_rows_per_token = heads * (split ? 2 : 1);
  const size_t n_pad = (n_tokens + 127) / 128 * 128;
  const size_t items = (size_t)prefill_items((int)n_layers, (int)heads, (int)hkv, (int)n_pad, split);
  const size_t qh_rows = n_layers * q_rows_per_token * n_pad;
  if (items > (size_t)INT32_MAX || qh_rows >= (1ull << 31)) return fail(e, TE_STATUS_UNSUPPORTED, "prefill too large");
  DeviceGuard dg(e->device);
  te_status st = ensure_pages(c, seq, total);
  if (st != TE_STATUS_OK) return st;

  const size_t in_el = (flags & TE_ATTN_INPUT_F16) ? 2 : 4;
  const size_t q_bytes = n_layers * n_tokens * heads * hd * in_el;
  const size_t kv_bytes = n_layers * n_tokens * hkv * hd * in_el;
  const size_t out_bytes = n_layers * n_tokens * heads * hd * sizeof(float);
  const void* dq = q;
  const void* dk = k;
  const void* dv = v;
  float* dout = out;
  cudaError_t err;
  if (flags & TE_ATTN_HOST_BUFFERS) {
    err = grow(e, &e->io, &e->io_bytes, q_bytes + 2 * kv_bytes + out_bytes + 256, false);
    if (err != cudaSuccess) return cuda_fail(e, err, "staging allocation");
    char* base = reinterpret_cast<char*>(e->io);
    char* sq = base;
    char* sk = sq + q_bytes;
    char* sv = sk + kv_bytes;
    dout = reinterpret_cast<float*>(sv + kv_bytes);
    err = cudaMemcpyAsync(sq, q, q_bytes, cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = cudaMemcpyAsync(sk, k, kv_bytes, cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = cudaMemcpyAsync(sv, v, kv_bytes, cudaMemcpyHostToDevice, e->stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "input upload");
    dq = sq;
    dk = sk;
    dv = sv;
  }

  // 1) RoPE(k) + f16 append of the new tokens for every layer (launched with 2)
  AppendParams a{};
  a.k = dk;
  a.v = dv;
  a.k_pool = c->k_pool;
  a.v_pool = c->v_pool;
  a.page_row = c->d_page_table + seq * c->pages_per_seq;
  a.rope_cos = c->d_cos;
  a.rope_sin = c->d_sin;
  if (bias) {
    a.k_bias = c->d_kb;
    a.v_bias = c->d_vb;
  }
  a.input_f16 = (flags & TE_ATTN_INPUT_F16) ? 1 : 0;
  a.rope = (flags & TE_ATTN_NO_ROPE) ? 0 : 1;
  a.n_layers = (int32_t)n_layers;
  a.layer_begin = (int32_t)layer_begin;
  a.n_tokens = (int32_t)n_tokens;
  a.first_index = (int32_t)q_offset;
  a.first_pos = (int32_t)(c->offset[seq] + q_offset);
  a.kv_heads = (int32_t)hkv;
  a.head_dim = (int32_t)hd;
  a.num_pages = (int32_t)c->d.total_pages;
  a.page_tokens = (int32_t)c->d.page_tokens;
  // 2) f16 queries for the kernel: f16 inputs without RoPE or bias are read
  // as they are; otherwise they are biased, rotated and converted into
  // scratch in the same layout, in one pass with the append.
  const void* qf16 = dq;
  QPrepParams qp{};
  if (with_q) {
    err = grow(e, &e->qh, &e->qh_bytes, n_layers * n_tokens * q_rows_per_token * hd * sizeof(__half), false);
    if (err != cudaSuccess) return cuda_fail(e, err, "prefill query scratch allocation");
    qp.q = dq;
    qp.qh = reinterpret_cast<__half*>(e->qh);
    qp.rope_cos = c->d_cos;
    qp.rope_sin = c->d_sin;
    qp.q_bias = bias ? c->d_qb : nullptr;
    qp.input_f16 = a.input_f16;
    qp.rope = a.rope;
    qp.n_layers = (int32_t)n_layers;
    qp.layer_begin = (int32_t)layer_begin;
    qp.n_tokens = (int32_t)n_tokens;
    qp.heads = (int32_t)heads;
    qp.head_dim = (int32_t)hd;
    qp.first_pos = a.first_pos;
    qp.split = split ? 1 : 0;
    qf16 = e->qh;
  }
  a.error = e->d_error;
  int prof = prof_begin(e, PK_PREFILL_PREP);
  err = launch_prefill_prep(a, qp, with_q, e->sm_count, e->stream);
  prof_end(e, prof);
  if (err != cudaSuccess) return cuda_fail(e, err, "append / query preparation launch");
  e->launches++;

  // 3) causal flash attention on tcgen05
  PrefillParams p;
  std::memset(&p, 0, sizeof(p));
  if (!make_tmap_q_f16(&p.tmap_q, qf16, hd, q_rows_per_token, n_tokens, n_layers)) {
    return fail(e, TE_STATUS_RUNTIME_ERROR, "query tensor map");
  }
  p.tmap_k = c->tmap_k;
  p.tmap_v = c->tmap_v;
  p.page_table_row = c->d_page_table + seq * c->pages_per_seq;
  p.out = dout;
  p.error = e->d_error;
  p.n_layers = (int32_t)n_layers;
  p.layer_begin = (int32_t)layer_begin;
  p.heads = (int32_t)heads;
  p.kv_heads = (int32_t)hkv;
  p.n_tokens = (int32_t)n_tokens;
  p.n_tokens_padded = (int32_t)n_pad;
  p.q_offset = (int32_t)q_offset;
  p.num_pages = (int32_t)c->d.total_pages;
  p.page_tokens = (int32_t)c->d.page_tokens;
  p.n_pages_mapped = (int32_t)((total + c->d.page_tokens - 1) / c->d.page_tokens);
  p.n_items = (int32_t)items;
  p.head_dim = (int32_t)hd;
  p.split = split ? 1 : 0;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)hd));
  if (e->time_kernels) cudaEventRecord(e->ev_k0, e->stream);
  prof = prof_begin(e, PK_PREFILL_ATTN);
  err = launch_prefill_tc(p, e->sm_count, e->stream);
  prof_end(e, prof);
  if (err != cudaSuccess) return cuda_fail(e, err, "prefill kernel launch");
  if (e->time_kernels) {
    cudaEventRecord(e->ev_k1, e->stream);
    e->kernel_timed = true;
  }
  e->launches++;

  if (flags & TE_ATTN_HOST_BUFFERS) {
    err = cudaMemcpyAsync(out, dout, out_bytes, cudaMemcpyDeviceToHost, e->stream);
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    if (err != cudaSuccess) return cuda_fail(e, err, "output download");
  }
  if (flags & TE_ATTN_ADVANCE) c->len[seq] = (int64_t)total;
  return TE_STATUS_OK;
}


// ===========================================================================
// Whole-token qwen2 decode step (k_step.cu)
// ===========================================================================

struct te_qwen_step {
  te_kv_cache* cache = nullptr;
  te_attn_engine* eng = nullptr;
  StepParams p{};           // everything but the per-call fields
  unsigned char* wpack = nullptr;
  long long* d_off = nullptr;
  float* scratch = nullptr;
  uint32_t* sync = nullptr;
  int grid = 0, smem = 0;
  uint32_t heads = 0;
};

TE_API void te_qwen_step_free(te_qwen_step* st) {
  if (!st) return;
  if (st->eng) {
    DeviceGuard dg(st->eng->device);
    cudaStreamSynchronize(st->eng->stream);
    cudaFree(st->wpack);
    cudaFree(st->d_off);
    cudaFree(st->scratch);
    cudaFree(st->sync);
  }
  delete st;
}

TE_API te_status te_qwen_step_create(te_kv_cache* c, const te_qwen_step_desc* d, te_qwen_step** out) {
  if (!c || !d || !out) return TE_STATUS_INVALID_ARGUMENT;
  *out = nullptr;
  te_attn_engine* e = c->eng;
  if (d->abi_version != TE_ATTN_ABI_VERSION) return fail(e, TE_STATUS_INVALID_ARGUMENT, "abi_version mismatch");
  const uint32_t L = d->layers, H = d->hidden, NH = d->heads, F = d->ffn, V = d->vocab;
  const uint32_t kvh = c->d.kv_heads, hd = c->d.head_dim;
  if (L == 0 || L != c->d.layers || NH == 0 || NH % kvh != 0 || NH * hd != H || H % 32 != 0 || F == 0 ||
      F % 32 != 0 || V == 0 || !(d->eps > 0.0f)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "model shape does not match the cache (heads * head_dim == hidden, "
                                               "hidden and ffn multiples of 32)");
  }
  if (NH / kvh > 16) return fail(e, TE_STATUS_UNSUPPORTED, "more than 16 query heads per kv head");
  if (L > (uint32_t)kStepMaxLayers || (H + e->sm_count - 1) / e->sm_count > (uint32_t)kStepMaxOwnRows) {
    return fail(e, TE_STATUS_UNSUPPORTED, "more layers or hidden rows per SM than the step kernel takes");
  }
  if (H > (1u << 24) || F > (1u << 24) || V > (uint32_t)INT32_MAX) return TE_STATUS_INVALID_ARGUMENT;
  const uint32_t quants[kStepKinds] = {d->quant_qkv, d->quant_o, d->quant_gu, d->quant_down, d->quant_head};
  for (uint32_t q : quants) {
    if (q != TE_ATTN_QUANT_GGUF_Q4_0 && q != TE_ATTN_QUANT_GGUF_Q8_0) return TE_STATUS_INVALID_ARGUMENT;
  }
  if (!d->w_qkv || !d->w_o || !d->w_gu || !d->w_down || !d->w_head || !d->attn_norm || !d->ffn_norm ||
      !d->out_norm || !d->embedding) {
    return TE_STATUS_INVALID_ARGUMENT;
  }
  const void* const* per_layer[4] = {d->w_qkv, d->w_o, d->w_gu, d->w_down};
  for (int k = 0; k < 4; ++k) {
    for (uint32_t l = 0; l < L; ++l) {
      if (!per_layer[k][l] || (reinterpret_cast<uintptr_t>(per_layer[k][l]) & 1u)) {
        return fail(e, TE_STATUS_INVALID_ARGUMENT, "projection pointers must be non-null and 2-byte aligned");
      }
    }
  }
  if ((reinterpret_cast<uintptr_t>(d->w_head) & 1u) ||
      ((reinterpret_cast<uintptr_t>(d->attn_norm) | reinterpret_cast<uintptr_t>(d->ffn_norm) |
        reinterpret_cast<uintptr_t>(d->out_norm) | reinterpret_cast<uintptr_t>(d->embedding)) & 15u)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "norm weights and the embedding table must be 16-byte aligned");
  }
  if ((uint64_t)c->d.layers * c->d.total_pages * kvh * c->d.page_tokens >= (1ull << 31)) {
    return fail(e, TE_STATUS_UNSUPPORTED, "KV pool too large for the step kernel's 32-bit row ids");
  }
  DeviceGuard dg(e->device);
  const int G = e->sm_count;
  const uint32_t kv = kvh * hd;
  const uint32_t rows[kStepKinds] = {H + 2 * kv, H, F, H, V};  // gate/up: F rows of (gate row, up row)
  const uint32_t cols[kStepKinds] = {H, H, H, F, H};
  int max_row = 0;
  for (int k = 0; k < kStepKinds; ++k) {
    const int bb = quants[k] == TE_ATTN_QUANT_GGUF_Q4_0 ? 18 : 34;
    max_row = std::max(max_row, (int)(cols[k] / 32 * bb) * (k == kStepGU ? 2 : 1));  // a gate/up stage: two rows
  }
  // stages of up to 64 KiB (at least 32 KiB, or one row, or one gate/up pair), in a byte ring of the rest
  // of shared memory that holds at least two of them
  const int attn_bytes = step_attn_bytes((int)hd);
  // work area: the ffn-sized input vector, the attention buffers, or x with its RMSNorm weights
  const int union_bytes = (std::max(std::max((int)std::max(H, F) * 4, attn_bytes), (int)H * 8) + 127) & ~127;
  const int ring_bytes = (227 * 1024 - step_fixed_smem() - union_bytes) & ~15;
  const int stage_min = std::max(32768, (max_row + 15) & ~15);
  const int stage_max = std::max(stage_min, std::min(65536, (ring_bytes / 2) & ~15));
  if (ring_bytes < 2 * stage_max) return fail(e, TE_STATUS_UNSUPPORTED, "rows or vectors too long for the step kernel's ring");
  const int smem = step_smem_bytes(ring_bytes, union_bytes);
  cudaError_t err = step_configure();
  if (err != cudaSuccess) return cuda_fail(e, err, "step kernel shared-memory limit");
  if (step_max_ctas_per_sm(smem) < 1) return fail(e, TE_STATUS_UNSUPPORTED, "step kernel does not fit an SM");

  StepParams p{};
  for (int k = 0; k < kStepKinds; ++k) {
    plan_step_mat(p.mat[k], (int)rows[k], (int)cols[k], quants[k] == TE_ATTN_QUANT_GGUF_Q4_0 ? 18 : 34, G,
                  stage_max, k == kStepGU ? 1 : 0);
  }
  // each CTA's stream: its stages of every layer's four projections, then the head's
  std::vector<long long> off((size_t)G + 1);
  std::vector<StepPackSeg> segs;
  long long pos = 0;
  auto add = [&](int k, const void* w, int b) {
    const StepMat& m = p.mat[k];
    int r0;
    const int n = step_cta_rows(m, b, r0);
    const int ns = step_n_stages(n, m.rps);
    for (int s = 0; s < ns; ++s) {
      const int lo = step_stage_lo(s, n, ns), hi = step_stage_lo(s + 1, n, ns);
      StepPackSeg sg;
      sg.src0 = static_cast<const unsigned char*>(w) + (size_t)(r0 + lo) * m.row_bytes;
      // gate/up: the same rows of the second half (up rows follow the F gate rows)
      sg.src1 = m.pair ? static_cast<const unsigned char*>(w) + (size_t)(m.rows + r0 + lo) * m.row_bytes : sg.src0;
      sg.dst_off = pos;
      sg.rows = (m.pair ? 2 : 1) * (hi - lo);
      sg.split = hi - lo;
      sg.nb = m.cols / 32;
      sg.block_bytes = m.block_bytes;
      segs.push_back(sg);
      pos += step_stage_bytes(sg.rows, sg.nb, m.block_bytes);
    }
  };
  for (int b = 0; b < G; ++b) {
    off[(size_t)b] = pos;
    for (uint32_t l = 0; l < L; ++l) {
      for (int k = 0; k < 4; ++k) add(k, per_layer[k][l], b);
    }
    add(kStepHead, d->w_head, b);
  }
  off[(size_t)G] = pos;
  if (segs.size() > (size_t)INT32_MAX) return TE_STATUS_UNSUPPORTED;

  auto* st = new te_qwen_step();
  st->cache = c;
  st->eng = e;
  st->grid = G;
  st->smem = smem;
  st->heads = NH;
  const int max_chunks = (int)((c->d.max_tokens_per_seq + kStepChunk - 1) / kStepChunk);
  const size_t group = NH / kvh;
  auto up4 = [](size_t n) { return (n + 3) & ~size_t(3); };  // 16-byte aligned sub-buffers
  // tagged words (8 bytes each): q|k|v, attention, SwiGLU output, two x vectors
  const size_t n_ll = up4(H + 2 * kv) + up4(H) + up4(F) + 2 * up4(H);
  const size_t n_rec = up4((size_t)kvh * max_chunks * group * (hd + 2)), n_cand = up4(2 * (size_t)G);
  StepPackSeg* d_segs = nullptr;
  err = cudaMalloc(&st->wpack, (size_t)std::max(pos, 16ll));
  if (err == cudaSuccess) err = cudaMalloc(&st->d_off, off.size() * sizeof(long long));
  if (err == cudaSuccess) err = cudaMalloc(&st->scratch, 2 * n_ll * sizeof(float) + (n_rec + n_cand) * sizeof(float));
  if (err == cudaSuccess) err = cudaMemsetAsync(st->scratch, 0, 2 * n_ll * sizeof(float), e->stream);
  if (err == cudaSuccess) err = cudaMalloc(&st->sync, (4 + kvh) * sizeof(uint32_t));
  if (err == cudaSuccess) err = cudaMalloc(&d_segs, std::max<size_t>(segs.size(), 1) * sizeof(StepPackSeg));
  if (err == cudaSuccess) err = cudaMemsetAsync(st->wpack, 0, (size_t)std::max(pos, 16ll), e->stream);
  if (err == cudaSuccess) err = cudaMemsetAsync(st->sync, 0, (4 + kvh) * sizeof(uint32_t), e->stream);
  if (err == cudaSuccess) {
    err = cudaMemcpyAsync(st->d_off, off.data(), off.size() * sizeof(long long), cudaMemcpyHostToDevice, e->stream);
  }
  if (err == cudaSuccess && !segs.empty()) {
    err = cudaMemcpyAsync(d_segs, segs.data(), segs.size() * sizeof(StepPackSeg), cudaMemcpyHostToDevice, e->stream);
  }
  if (err == cudaSuccess) err = launch_step_pack(d_segs, (int)segs.size(), st->wpack, e->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (d_segs) cudaFree(d_segs);
  if (err != cudaSuccess) {
    te_qwen_step_free(st);
    return cuda_fail(e, err, "step set-up");
  }
  p.wpack = st->wpack;
  p.cta_off = st->d_off;
  p.layers = (int32_t)L;
  p.hidden = (int32_t)H;
  p.heads = (int32_t)NH;
  p.kv_heads = (int32_t)kvh;
  p.head_dim = (int32_t)hd;
  p.ffn = (int32_t)F;
  p.vocab = (int32_t)V;
  p.group = (int32_t)group;
  p.eps = d->eps;
  p.scale_log2 = (float)(1.4426950408889634 / std::sqrt((double)hd));
  p.k_pool = c->k_pool;
  p.v_pool = c->v_pool;
  p.num_pages = (int32_t)c->d.total_pages;
  p.page_tokens = (int32_t)c->d.page_tokens;
  p.rope_cos = c->d_cos;
  p.rope_sin = c->d_sin;
  p.attn_norm = d->attn_norm;
  p.ffn_norm = d->ffn_norm;
  p.out_norm = d->out_norm;
  p.emb = d->embedding;
  auto* ll = reinterpret_cast<unsigned long long*>(st->scratch);
  p.ll_qkv = ll;
  p.ll_attn = p.ll_qkv + up4(H + 2 * kv);
  p.ll_h = p.ll_attn + up4(H);
  p.ll_x[0] = p.ll_h + up4(F);
  p.ll_x[1] = p.ll_x[0] + up4(H);
  p.rec = st->scratch + 2 * n_ll;
  p.cand = p.rec + n_rec;
  p.sync = st->sync;
  p.error = e->d_error;
  p.ring_bytes = ring_bytes;
  p.union_bytes = union_bytes;
  st->p = p;
  *out = st;
  return TE_STATUS_OK;
}

TE_API te_status te_qwen_step_run(te_qwen_step* st, size_t seq, const int64_t* token, float* hidden, float* logits,
                                  int64_t* next_token, uint32_t flags) {
  if (!st || !token || !hidden) return TE_STATUS_INVALID_ARGUMENT;
  te_kv_cache* c = st->cache;
  te_attn_engine* e = st->eng;
  if (flags & ~(TE_ATTN_ADVANCE | TE_ATTN_QKV_BIAS | TE_ATTN_STEP_HEAD)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "unsupported flags for te_qwen_step_run");
  }
  const bool head = (flags & TE_ATTN_STEP_HEAD) != 0;
  if (head && (!logits || !next_token)) return fail(e, TE_STATUS_INVALID_ARGUMENT, "the head needs logits and next_token");
  if ((reinterpret_cast<uintptr_t>(hidden) & 15u) || (reinterpret_cast<uintptr_t>(token) & 7u) ||
      (head && ((reinterpret_cast<uintptr_t>(logits) & 3u) || (reinterpret_cast<uintptr_t>(next_token) & 7u)))) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "hidden must be 16-byte aligned, token and next_token 8-byte aligned");
  }
  if (seq >= c->d.max_seqs) return TE_STATUS_INVALID_ARGUMENT;
  if ((flags & TE_ATTN_QKV_BIAS) && (!c->d_qb || c->bias_heads != st->heads)) {
    return fail(e, TE_STATUS_INVALID_ARGUMENT, "TE_ATTN_QKV_BIAS needs te_kv_cache_set_qkv_bias with these heads");
  }
  const int64_t len = c->len[seq] + 1;
  if ((uint64_t)len > c->d.max_tokens_per_seq) return fail(e, TE_STATUS_INVALID_ARGUMENT, "sequence full");
  const int64_t pos = c->offset[seq] + len - 1;
  if ((uint64_t)pos >= c->d.max_position) return fail(e, TE_STATUS_INVALID_ARGUMENT, "RoPE position beyond max_position");
  DeviceGuard dg(e->device);
  te_status sts = ensure_pages(c, seq, (size_t)len);
  if (sts != TE_STATUS_OK) return sts;
  StepParams p = st->p;
  p.page_row = c->d_page_table + seq * c->pages_per_seq;
  p.page_base = contiguous_base(c, seq, (size_t)len);
  p.n_tokens = (int32_t)len;
  p.rope_pos = (int32_t)pos;
  if (flags & TE_ATTN_QKV_BIAS) {
    p.q_bias = c->d_qb;
    p.k_bias = c->d_kb;
    p.v_bias = c->d_vb;
  }
  p.token_in = token;
  p.x = hidden;
  p.logits = logits;
  p.token_out = next_token;
  p.head = head ? 1 : 0;
  const int prof = prof_begin(e, PK_STEP);
  const cudaError_t err = launch_step(p, st->grid, st->smem, e->stream);
  prof_end(e, prof);
  if (err != cudaSuccess) return cuda_fail(e, err, "step kernel launch");
  e->launches++;
  if (flags & TE_ATTN_ADVANCE) c->len[seq] = len;
  return TE_STATUS_OK;
}

}  // extern "C"
