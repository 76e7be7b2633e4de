/*
 * Link stubs for building the reference's c/src/ops.c on Linux as a checker
 * (TEST INFRASTRUCTURE ONLY).  ops.c's matvec path references three symbols
 * from the Metal backend and the GGUF loader; the attention and RoPE functions
 * used as the oracle never call them.  Every stub reports "unsupported".
 *
 * Signatures follow c/src/metal_backend.h:13-22 and
 * c/src/tinyengine_internal.h:92-98 of the TinyEngine project.
 */
#include "tinyengine_internal.h"
#include "metal_backend.h"

te_status te_metal_matvec_f32(const void *mapping, size_t mapping_len, uint64_t tensor_offset,
                              uint32_t ggml_type, const float *input, size_t cols, size_t rows,
                              float *out) {
    (void)mapping; (void)mapping_len; (void)tensor_offset; (void)ggml_type;
    (void)input; (void)cols; (void)rows; (void)out;
    return TE_STATUS_UNSUPPORTED;
}

const te_gguf_tensor *te_model_find_tensor(const te_model *model, const char *name) {
    (void)model; (void)name;
    return NULL;
}

te_status te_model_tensor_data(const te_model *model, const te_gguf_tensor *tensor,
                               const uint8_t **out_data, size_t *out_len) {
    (void)model; (void)tensor; (void)out_data; (void)out_len;
    return TE_STATUS_UNSUPPORTED;
}
