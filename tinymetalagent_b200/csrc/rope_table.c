/*
 * Host RoPE tables, computed exactly as TinyEngine does on the CPU:
 *   freq  = powf(theta, -(2.0f * (float)i) / (float)head_dim)
 *   angle = (float)position * freq
 *   cos = cosf(angle), sin = sinf(angle)
 * (c/src/qwen.c:531-539; te_rope_f32 recomputes the same expressions per call,
 * c/src/ops.c:308-312).  Built as C with -O2 -ffp-contract=off so the values
 * equal the reference's bit for bit on the same C library; the GPU only
 * multiplies and adds with them.
 */
#include <math.h>
#include <stddef.h>

void te_host_rope_table(float *cos_table, float *sin_table, size_t first_position, size_t positions,
                        size_t head_dim, float theta) {
    const size_t half = head_dim / 2u;
    for (size_t p = 0; p < positions; ++p) {
        const size_t position = first_position + p;
        for (size_t i = 0; i < half; ++i) {
            const float freq = powf(theta, -(2.0f * (float)i) / (float)head_dim);
            const float angle = (float)position * freq;
            cos_table[p * half + i] = cosf(angle);
            sin_table[p * half + i] = sinf(angle);
        }
    }
}
