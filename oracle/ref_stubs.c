/*
 * Link stubs for building the reference's c/src/ops.c on Linux as a checker
 * (TEST INFRASTRUCTURE ONLY).  ops.c's matvec path references three symbols
 * from the Metal backend and the GGUF loader.  The Metal stub reports
 * "unsupported", so te_model_matvec_f32 takes its own CPU row loop; the two
 * loader stubs describe one rank-2 tensor that a test registers with
 * ref_stub_register_tensor (its bytes stay owned by the caller), so that the
 * reference's quantized dot products run on test data.
 *
 * Signatures follow c/src/metal_backend.h:13-22 and
 * c/src/tinyengine_internal.h:92-98 of the TinyEngine project.
 */
#include "tinyengine_internal.h"
#include "metal_backend.h"

#include <string.h>

te_status te_metal_matvec_f32(const void *mapping, size_t mapping_len, uint64_t tensor_offset,
                              uint32_t ggml_type, const float *input, size_t cols, size_t rows,
                              float *out) {
    (void)mapping; (void)mapping_len; (void)tensor_offset; (void)ggml_type;
    (void)input; (void)cols; (void)rows; (void)out;
    return TE_STATUS_UNSUPPORTED;
}

static te_gguf_tensor stub_tensor;
static const uint8_t *stub_data;
static size_t stub_len;
static struct te_model stub_model;

/* Registers the tensor that te_model_find_tensor returns for any name:
 * ggml type (0 F32, 2 Q4_0, 8 Q8_0), dims {cols, rows}, raw bytes. */
void ref_stub_register_tensor(uint32_t ggml_type, uint64_t cols, uint64_t rows, const uint8_t *data, size_t len) {
    memset(&stub_tensor, 0, sizeof(stub_tensor));
    stub_tensor.n_dims = 2u;
    stub_tensor.dims[0] = cols;
    stub_tensor.dims[1] = rows;
    stub_tensor.ggml_type = ggml_type;
    stub_tensor.bytes = len;
    stub_data = data;
    stub_len = len;
}

/* A zeroed model to pass to te_model_matvec_f32 (only its mapping fields are read, for the Metal stub). */
const te_model *ref_stub_model(void) {
    return &stub_model;
}

const te_gguf_tensor *te_model_find_tensor(const te_model *model, const char *name) {
    (void)model; (void)name;
    return stub_data != NULL ? &stub_tensor : NULL;
}

te_status te_model_tensor_data(const te_model *model, const te_gguf_tensor *tensor,
                               const uint8_t **out_data, size_t *out_len) {
    (void)model;
    if (tensor != &stub_tensor || stub_data == NULL) return TE_STATUS_UNSUPPORTED;
    *out_data = stub_data;
    *out_len = stub_len;
    return TE_STATUS_OK;
}
