/*
 * CPU oracle for the attention stage (TEST INFRASTRUCTURE ONLY).
 *
 * This is a plain-C restatement of TinyEngine's CPU attention path, used by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker.  The product library never links, loads or calls it.
 *
 * Each function names the reference file:line it restates (paths are relative
 * to the TinyEngine project root).  Loop order and fp32 expression shapes are
 * kept identical so that, built with the same flags as the reference
 * (gcc -O2, x86-64 baseline: no FMA contraction), results are bit-identical to
 * the reference's own ops.c.  The pin is checked by tests/test_oracle.py
 * against the reference's known-answer tests and golden vectors produced by
 * the reference's compiled ops.c (oracle/_ref).
 */
#ifndef TE_ORACLE_H
#define TE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status values are the reference's te_status codes (c/include/tinyengine.h:28-35). */
enum {
    OR_OK = 0,
    OR_INVALID_ARGUMENT = 1,
    OR_UNSUPPORTED = 3,
    OR_OUT_OF_MEMORY = 4
};

int or_rope_f32(float *values, size_t heads, size_t head_dim, size_t position, float theta);
int or_rope_table(float *cos_table, float *sin_table, size_t positions, size_t head_dim, float theta);
int or_rope_cached(float *values, size_t heads, size_t head_dim,
                   const float *cos_table, const float *sin_table, size_t position);
int or_attention_decode_f32(const float *query, const float *key_cache, const float *value_cache,
                            size_t position, size_t heads, size_t kv_heads, size_t head_dim,
                            float *out);

uint16_t or_f32_to_f16(float value);
float or_f16_to_f32(uint16_t bits);
void or_f32_to_f16_array(const float *in, uint16_t *out, size_t n);
void or_f16_to_f32_array(const uint16_t *in, float *out, size_t n);

int or_append_rope_f16(const float *k_raw, const float *v_raw, size_t n_tokens, size_t first_position,
                       size_t kv_heads, size_t head_dim, float theta,
                       uint16_t *k_cache, uint16_t *v_cache);
int or_causal_prefill_f32(const float *q_rot, const float *key_cache, const float *value_cache,
                          size_t seq_len, size_t heads, size_t kv_heads, size_t head_dim, float *out);
int or_decode_partial_f32(const float *query, const float *key_cache, const float *value_cache,
                          size_t token_begin, size_t token_end, size_t heads, size_t kv_heads,
                          size_t head_dim, float *partial);
int or_merge_partials_f32(const float *partials, size_t n_parts, size_t heads, size_t head_dim,
                          float *out);

int or_matvec_q4_0_f32(const uint8_t *w, size_t rows, size_t cols, const float *x, float *out);
int or_matvec_q8_0_f32(const uint8_t *w, size_t rows, size_t cols, const float *x, float *out);

#ifdef __cplusplus
}
#endif

#endif
