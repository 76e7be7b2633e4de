/*
 * CPU oracle for the attention stage (TEST INFRASTRUCTURE ONLY).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load
 * this file's shared object, and only as the checker or the timed CPU
 * baseline.  The product (libtinyengine.so) does not link or call it.
 *
 * Restated from TinyEngine (paths relative to the TinyEngine project root):
 *   or_rope_f32             c/src/ops.c:295-321          (te_rope_f32)
 *   or_rope_table           c/src/qwen.c:531-539         (host cos/sin table)
 *   or_rope_cached          c/src/qwen.c:2133-2160       (te_qwen_rope_cached)
 *   or_attention_decode_f32 c/src/ops.c:323-395          (te_attention_decode_f32)
 *   or_f16_to_f32           c/src/ops.c:435-462          (te_f16_to_f32)
 *   or_f32_to_f16           Metal half() cast used by the f16 KV mirror,
 *                           c/src/metal/metal_kernels.metal.inc:2414-2427
 *                           (IEEE-754 binary32 -> binary16, round to nearest even)
 *   or_append_rope_f16      c/src/metal/metal_kernels.metal.inc:2344-2429
 *                           (k/v part of te_qkv_bias_rope_cache_batch_h_f32)
 *   or_causal_prefill_f32   c/src/qwen.c:810-824         (decode call per prompt token)
 *   or_matvec_q4_0_f32      c/src/ops.c:584-602, 824-845  (te_q4_0_dot_row, scalar path,
 *                           per row as te_matvec_worker calls it)
 *   or_matvec_q8_0_f32      c/src/ops.c:604-620, 824-845  (te_q8_0_dot_row, scalar path)
 * Not in the reference (the multi-GPU KV split is new); restated from the
 * (m, l, acc) rescale of c/src/metal/metal_kernels.metal.inc:2650-2681:
 *   or_decode_partial_f32, or_merge_partials_f32
 */
#include "te_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#define OR_STACK_SCORES 1024u /* c/src/ops.c:22 */

int or_rope_f32(float *values, size_t heads, size_t head_dim, size_t position, float theta) {
    if (values == NULL || heads == 0u || head_dim == 0u || (head_dim % 2u) != 0u || theta <= 0.0f) {
        return OR_INVALID_ARGUMENT;
    }
    const size_t half = head_dim / 2u;
    for (size_t h = 0; h < heads; ++h) {
        float *row = values + h * head_dim;
        for (size_t i = 0; i < half; ++i) {
            const float freq = powf(theta, -(2.0f * (float)i) / (float)head_dim);
            const float angle = (float)position * freq;
            const float s = sinf(angle);
            const float c = cosf(angle);
            const float a = row[i];
            const float b = row[i + half];
            row[i] = a * c - b * s;
            row[i + half] = b * c + a * s;
        }
    }
    return OR_OK;
}

int or_rope_table(float *cos_table, float *sin_table, size_t positions, size_t head_dim, float theta) {
    if (cos_table == NULL || sin_table == NULL || head_dim == 0u || (head_dim % 2u) != 0u || theta <= 0.0f) {
        return OR_INVALID_ARGUMENT;
    }
    const size_t half = head_dim / 2u;
    for (size_t p = 0; p < positions; ++p) {
        for (size_t i = 0; i < half; ++i) {
            const float freq = powf(theta, -(2.0f * (float)i) / (float)head_dim);
            const float angle = (float)p * freq;
            cos_table[p * half + i] = cosf(angle);
            sin_table[p * half + i] = sinf(angle);
        }
    }
    return OR_OK;
}

int or_rope_cached(float *values, size_t heads, size_t head_dim,
                   const float *cos_table, const float *sin_table, size_t position) {
    if (values == NULL || cos_table == NULL || sin_table == NULL ||
        heads == 0u || head_dim == 0u || (head_dim % 2u) != 0u) {
        return OR_INVALID_ARGUMENT;
    }
    const size_t half = head_dim / 2u;
    const float *crow = cos_table + position * half;
    const float *srow = sin_table + position * half;
    for (size_t h = 0; h < heads; ++h) {
        float *row = values + h * head_dim;
        for (size_t i = 0; i < half; ++i) {
            const float a = row[i];
            const float b = row[i + half];
            row[i] = a * crow[i] - b * srow[i];
            row[i + half] = b * crow[i] + a * srow[i];
        }
    }
    return OR_OK;
}

int or_attention_decode_f32(const float *query, const float *key_cache, const float *value_cache,
                            size_t position, size_t heads, size_t kv_heads, size_t head_dim,
                            float *out) {
    if (query == NULL || key_cache == NULL || value_cache == NULL || out == NULL ||
        heads == 0u || kv_heads == 0u || head_dim == 0u || (heads % kv_heads) != 0u) {
        return OR_INVALID_ARGUMENT;
    }
    if (position == SIZE_MAX) {
        return OR_UNSUPPORTED;
    }
    const size_t group = heads / kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    const size_t n = position + 1u;
    float stack_scores[OR_STACK_SCORES];
    float *scores = n <= OR_STACK_SCORES ? stack_scores : (float *)malloc(n * sizeof(float));
    if (scores == NULL) {
        return OR_OUT_OF_MEMORY;
    }
    for (size_t h = 0; h < heads; ++h) {
        const size_t kvh = h / group;
        const float *q = query + h * head_dim;
        for (size_t t = 0; t < n; ++t) {
            const float *k = key_cache + (t * kv_heads + kvh) * head_dim;
            float dot = 0.0f;
            for (size_t d = 0; d < head_dim; ++d) {
                dot += q[d] * k[d];
            }
            scores[t] = dot * scale;
        }
        float mx = -FLT_MAX;
        for (size_t t = 0; t < n; ++t) {
            if (scores[t] > mx) {
                mx = scores[t];
            }
        }
        float sum = 0.0f;
        for (size_t t = 0; t < n; ++t) {
            scores[t] = expf(scores[t] - mx);
            sum += scores[t];
        }
        if (sum > 0.0f) {
            for (size_t t = 0; t < n; ++t) {
                scores[t] /= sum;
            }
        }
        for (size_t d = 0; d < head_dim; ++d) {
            float acc = 0.0f;
            for (size_t t = 0; t < n; ++t) {
                acc += scores[t] * value_cache[(t * kv_heads + kvh) * head_dim + d];
            }
            out[h * head_dim + d] = acc;
        }
    }
    if (scores != stack_scores) {
        free(scores);
    }
    return OR_OK;
}

/* binary32 -> binary16, round to nearest, ties to even; NaN stays NaN, overflow -> inf. */
uint16_t or_f32_to_f16(float value) {
    uint32_t x;
    memcpy(&x, &value, sizeof(x));
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t exp32 = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp32 == 0xffu) {
        return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0u));
    }
    const int32_t e = (int32_t)exp32 - 127 + 15;
    if (e >= 31) {
        return (uint16_t)(sign | 0x7c00u);
    }
    if (e <= 0) {
        /* subnormal half (or zero): value = man_with_hidden * 2^(e-1-10-13) */
        if (e < -10) {
            return sign;
        }
        man |= 0x800000u;
        const uint32_t shift = (uint32_t)(14 - e);
        uint32_t q = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1u);
        if (rem > halfway || (rem == halfway && (q & 1u))) {
            q += 1u;
        }
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) {
        q += 1u; /* may carry into the exponent, reaching inf correctly */
    }
    return (uint16_t)(sign | q);
}

float or_f16_to_f32(uint16_t bits) {
    const uint32_t sign = ((uint32_t)bits & 0x8000u) << 16;
    uint32_t e = ((uint32_t)bits >> 10) & 0x1fu;
    uint32_t m = (uint32_t)bits & 0x3ffu;
    uint32_t x;
    if (e == 0u) {
        if (m == 0u) {
            x = sign;
        } else {
            int32_t ue = -14;
            while ((m & 0x400u) == 0u) {
                m <<= 1;
                --ue;
            }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(ue + 127) << 23) | (m << 13);
        }
    } else if (e == 31u) {
        x = sign | 0x7f800000u | (m << 13);
    } else {
        x = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, sizeof(f));
    return f;
}

void or_f32_to_f16_array(const float *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        out[i] = or_f32_to_f16(in[i]);
    }
}

void or_f16_to_f32_array(const uint16_t *in, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        out[i] = or_f16_to_f32(in[i]);
    }
}

/*
 * k_raw, v_raw: [n_tokens][kv_heads][head_dim] fp32 (post-bias, pre-RoPE).
 * k_cache, v_cache: [n_tokens][kv_heads][head_dim] f16 bits, written at
 * positions first_position + t.  RoPE uses the host table recipe
 * (qwen.c:531-539), identical in value to te_rope_f32's per-call trig.
 */
int or_append_rope_f16(const float *k_raw, const float *v_raw, size_t n_tokens, size_t first_position,
                       size_t kv_heads, size_t head_dim, float theta,
                       uint16_t *k_cache, uint16_t *v_cache) {
    if (k_raw == NULL || v_raw == NULL || k_cache == NULL || v_cache == NULL ||
        kv_heads == 0u || head_dim == 0u || (head_dim % 2u) != 0u || theta <= 0.0f) {
        return OR_INVALID_ARGUMENT;
    }
    const size_t kv = kv_heads * head_dim;
    float *row = (float *)malloc(kv * sizeof(float));
    if (row == NULL) {
        return OR_OUT_OF_MEMORY;
    }
    for (size_t t = 0; t < n_tokens; ++t) {
        memcpy(row, k_raw + t * kv, kv * sizeof(float));
        or_rope_f32(row, kv_heads, head_dim, first_position + t, theta);
        or_f32_to_f16_array(row, k_cache + t * kv, kv);
        or_f32_to_f16_array(v_raw + t * kv, v_cache + t * kv, kv);
    }
    free(row);
    return OR_OK;
}

/* q_rot: [seq_len][heads][head_dim]; caches [seq_len][kv_heads][head_dim]; out like q. */
int or_causal_prefill_f32(const float *q_rot, const float *key_cache, const float *value_cache,
                          size_t seq_len, size_t heads, size_t kv_heads, size_t head_dim, float *out) {
    const size_t hidden = heads * head_dim;
    for (size_t t = 0; t < seq_len; ++t) {
        const int st = or_attention_decode_f32(q_rot + t * hidden, key_cache, value_cache, t,
                                               heads, kv_heads, head_dim, out + t * hidden);
        if (st != OR_OK) {
            return st;
        }
    }
    return OR_OK;
}

/*
 * Partial softmax state over tokens [token_begin, token_end) for every head:
 * partial[h] = { acc[0..head_dim), m, l } with m the running max of
 * score*log2(e) (score = q.k/sqrt(head_dim)), l = sum 2^(score*log2e - m),
 * acc = sum 2^(score*log2e - m) * v.  This is the record the engine exchanges
 * between GPUs for the KV-sequence split.
 */
int or_decode_partial_f32(const float *query, const float *key_cache, const float *value_cache,
                          size_t token_begin, size_t token_end, size_t heads, size_t kv_heads,
                          size_t head_dim, float *partial) {
    if (query == NULL || key_cache == NULL || value_cache == NULL || partial == NULL ||
        heads == 0u || kv_heads == 0u || head_dim == 0u || (heads % kv_heads) != 0u ||
        token_end <= token_begin) {
        return OR_INVALID_ARGUMENT;
    }
    const size_t group = heads / kv_heads;
    const float scale = 1.0f / sqrtf((float)head_dim);
    const float log2e = 1.4426950408889634f;
    for (size_t h = 0; h < heads; ++h) {
        const size_t kvh = h / group;
        const float *q = query + h * head_dim;
        float *rec = partial + h * (head_dim + 2u);
        float m = -INFINITY;
        float l = 0.0f;
        for (size_t d = 0; d < head_dim; ++d) {
            rec[d] = 0.0f;
        }
        for (size_t t = token_begin; t < token_end; ++t) {
            const float *k = key_cache + (t * kv_heads + kvh) * head_dim;
            float dot = 0.0f;
            for (size_t d = 0; d < head_dim; ++d) {
                dot += q[d] * k[d];
            }
            const float s = dot * scale * log2e;
            const float mn = s > m ? s : m;
            const float alpha = exp2f(m - mn);
            const float p = exp2f(s - mn);
            l = l * alpha + p;
            const float *v = value_cache + (t * kv_heads + kvh) * head_dim;
            for (size_t d = 0; d < head_dim; ++d) {
                rec[d] = rec[d] * alpha + p * v[d];
            }
            m = mn;
        }
        rec[head_dim] = m;
        rec[head_dim + 1u] = l;
    }
    return OR_OK;
}

/* partials: [n_parts][heads][head_dim + 2]; out: [heads][head_dim] normalised. */
int or_merge_partials_f32(const float *partials, size_t n_parts, size_t heads, size_t head_dim,
                          float *out) {
    if (partials == NULL || out == NULL || n_parts == 0u || heads == 0u || head_dim == 0u) {
        return OR_INVALID_ARGUMENT;
    }
    const size_t rec = head_dim + 2u;
    for (size_t h = 0; h < heads; ++h) {
        float mx = -INFINITY;
        for (size_t p = 0; p < n_parts; ++p) {
            const float m = partials[(p * heads + h) * rec + head_dim];
            if (m > mx) {
                mx = m;
            }
        }
        float total = 0.0f;
        for (size_t d = 0; d < head_dim; ++d) {
            out[h * head_dim + d] = 0.0f;
        }
        for (size_t p = 0; p < n_parts; ++p) {
            const float *r = partials + (p * heads + h) * rec;
            if (r[head_dim + 1u] <= 0.0f) {
                continue;
            }
            const float w = exp2f(r[head_dim] - mx);
            total += r[head_dim + 1u] * w;
            for (size_t d = 0; d < head_dim; ++d) {
                out[h * head_dim + d] += r[d] * w;
            }
        }
        for (size_t d = 0; d < head_dim; ++d) {
            out[h * head_dim + d] = total > 0.0f ? out[h * head_dim + d] / total : 0.0f;
        }
    }
    return OR_OK;
}

/* GGUF Q4_0 / Q8_0 row-major matrices [rows][cols], 32-weight blocks:
 * Q4_0 block = f16 scale (little-endian) + 16 bytes, byte j holding weight j
 * in its low nibble and weight j + 16 in its high nibble, both offset by 8;
 * Q8_0 block = f16 scale + 32 int8.  One sequential fp32 sum per row, in the
 * reference's element order (c/src/ops.c:584-620). */
int or_matvec_q4_0_f32(const uint8_t *w, size_t rows, size_t cols, const float *x, float *out) {
    if (w == NULL || x == NULL || out == NULL || rows == 0u || cols == 0u || (cols % 32u) != 0u) {
        return OR_INVALID_ARGUMENT;
    }
    const size_t blocks = cols / 32u;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t *row = w + r * blocks * 18u;
        float sum = 0.0f;
        for (size_t b = 0; b < blocks; ++b) {
            const uint8_t *src = row + b * 18u;
            const float scale = or_f16_to_f32((uint16_t)(src[0] | ((uint16_t)src[1] << 8)));
            const uint8_t *qs = src + 2u;
            const float *xb = x + b * 32u;
            for (size_t j = 0; j < 16u; ++j) {
                sum += (((float)(qs[j] & 0x0fu) - 8.0f) * scale) * xb[j];
                sum += (((float)(qs[j] >> 4u) - 8.0f) * scale) * xb[j + 16u];
            }
        }
        out[r] = sum;
    }
    return OR_OK;
}

int or_matvec_q8_0_f32(const uint8_t *w, size_t rows, size_t cols, const float *x, float *out) {
    if (w == NULL || x == NULL || out == NULL || rows == 0u || cols == 0u || (cols % 32u) != 0u) {
        return OR_INVALID_ARGUMENT;
    }
    const size_t blocks = cols / 32u;
    for (size_t r = 0; r < rows; ++r) {
        const uint8_t *row = w + r * blocks * 34u;
        float sum = 0.0f;
        for (size_t b = 0; b < blocks; ++b) {
            const uint8_t *src = row + b * 34u;
            const float scale = or_f16_to_f32((uint16_t)(src[0] | ((uint16_t)src[1] << 8)));
            const int8_t *qs = (const int8_t *)(src + 2u);
            const float *xb = x + b * 32u;
            for (size_t j = 0; j < 32u; ++j) {
                sum += ((float)qs[j] * scale) * xb[j];
            }
        }
        out[r] = sum;
    }
    return OR_OK;
}
