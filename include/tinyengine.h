/*
 * TinyEngine C ABI -- attention-stage subset, B200 build.
 *
 * The status codes, export macro, ABI version and the two attention-stage
 * entry points keep the exact names, signatures and error behaviour of
 * TinyEngine's c/include/tinyengine.h so that existing callers (qwen.c's
 * decode/prefill loops, kernel tests, ctypes bindings) link unchanged:
 *   TE_API / TE_ABI_VERSION    c/include/tinyengine.h:15-25
 *   te_status                  c/include/tinyengine.h:28-35
 *   te_version, te_strerror    c/include/tinyengine.h:214-215 (c/src/tinyengine.c:13-34)
 *   te_rope_f32                c/include/tinyengine.h:293-299 (c/src/ops.c:295-321)
 *   te_attention_decode_f32    c/include/tinyengine.h:300-309 (c/src/ops.c:323-395)
 * The Apple-only #error of the original header is gone; everything else that
 * header declares (GGUF models, tokenizer, generation) is outside this build.
 *
 * In this build both functions run on the current CUDA device of the calling
 * thread.  They keep the original contract: host fp32 buffers in and out,
 * caller-owned memory, no state kept between calls, reentrant.  Each call
 * copies its inputs to the device, runs a CUDA kernel and copies the result
 * back before returning; they exist for drop-in parity, while the
 * device-resident engine in tinyengine_attn.h is the fast path.  With no
 * usable CUDA device they return TE_STATUS_UNSUPPORTED; there is no CPU
 * fallback.
 */
#ifndef TINYENGINE_H
#define TINYENGINE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#  if defined(TINYENGINE_BUILD)
#    define TE_API __declspec(dllexport)
#  else
#    define TE_API __declspec(dllimport)
#  endif
#else
#  define TE_API __attribute__((visibility("default")))
#endif

#define TE_ABI_VERSION 3u

typedef enum te_status {
    TE_STATUS_OK = 0,
    TE_STATUS_INVALID_ARGUMENT = 1,
    TE_STATUS_IO_ERROR = 2,
    TE_STATUS_UNSUPPORTED = 3,
    TE_STATUS_OUT_OF_MEMORY = 4,
    TE_STATUS_RUNTIME_ERROR = 5
} te_status;

/* Replaces te_version, c/include/tinyengine.h:214. */
TE_API const char *te_version(void);
/* Replaces te_strerror, c/include/tinyengine.h:215; same strings as c/src/tinyengine.c:17-34. */
TE_API const char *te_strerror(te_status status);

/*
 * Replaces te_rope_f32, c/include/tinyengine.h:293-299.
 * In-place rotary embedding of values[heads][head_dim] at `position`
 * (half-split pairs (i, i + head_dim/2), frequency theta^(-2i/head_dim)).
 * INVALID_ARGUMENT for NULL, zero or odd head_dim, zero heads, theta <= 0.
 * Result is bit-identical to the reference CPU function.
 */
TE_API te_status te_rope_f32(
    float *values,
    size_t heads,
    size_t head_dim,
    size_t position,
    float theta
);

/*
 * Replaces te_attention_decode_f32, c/include/tinyengine.h:300-309.
 * Single-query grouped-query attention over position+1 cached tokens:
 * query[heads][head_dim], key_cache/value_cache[position+1][kv_heads][head_dim]
 * (token-major, heads interleaved), out[heads][head_dim]; q head h reads KV
 * head h / (heads / kv_heads); scale 1/sqrt(head_dim).
 * INVALID_ARGUMENT for NULL pointers, zero sizes or heads % kv_heads != 0;
 * UNSUPPORTED for position == SIZE_MAX (as the reference).
 */
TE_API te_status te_attention_decode_f32(
    const float *query,
    const float *key_cache,
    const float *value_cache,
    size_t position,
    size_t heads,
    size_t kv_heads,
    size_t head_dim,
    float *out
);

#ifdef __cplusplus
}
#endif

#endif
