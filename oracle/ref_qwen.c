/* TEST INFRASTRUCTURE ONLY -- the checker for the layer-step integration.
 *
 * Builds the reference's own CPU forward pass from its sources where they
 * lie: c/src/qwen.c is compiled as part of this file (the #include below), so
 * its file-local te_qwen_state_init (:424-629), te_qwen_forward_token
 * (:907-1112: embedding row, per layer RMSNorm, q/k/v projections + biases,
 * RoPE from the cached table, fp32 KV cache, te_attention_decode_f32, output
 * projection + residual, RMSNorm, SwiGLU MLP + residual) and
 * te_qwen_project_next (:1303-1377: output norm, lm_head, argmax) are
 * reachable.  gguf.c, ops.c and tokenizer.c are linked as they are; the Metal
 * entry points answer "unsupported" (ref_metal_off.c), and the environment
 * switches the reference reads turn its fused Metal paths off, so every step
 * runs the reference's CPU branch.  Greedy projection (temperature 0).
 *
 * Exported: rq_open(path, context_tokens) -> 0 on success; rq_forward(token,
 * position, hidden_out[hidden]); rq_project(logits_out[vocab], &token);
 * rq_dims(out[8]) = hidden, ffn, layers, heads, kv_heads, head_dim, vocab,
 * context_tokens; rq_close(). */
#define _GNU_SOURCE
#include "qwen.c"

static te_model *rq_model;
static te_context rq_ctx;
static te_qwen_state rq_state;
static int rq_ready;

/* tinyengine.c (model load, options) is Apple-only; these are the few
 * helpers of it that gguf.c and tokenizer.c call, restated. */
char *te_strdup(const char *value) {
    if (value == NULL) return NULL;
    const size_t n = strlen(value) + 1u;
    char *out = (char *)malloc(n);
    if (out != NULL) memcpy(out, value, n);
    return out;
}

void rq_close(void) {
    if (rq_ready) {
        te_qwen_state_release(&rq_state);
        rq_ready = 0;
    }
    if (rq_model != NULL) {
        te_tokenizer_release(rq_model);
        te_model_release_gguf(rq_model);
        free(rq_model->path);
        free(rq_model);
        rq_model = NULL;
    }
}

int rq_open(const char *path, uint32_t context_tokens) {
    rq_close();
    setenv("TINYENGINE_DECODE_ALL_LAYERS", "0", 1);
    setenv("TINYENGINE_FUSED_DECODE_LAYER", "0", 1);
    setenv("TINYENGINE_METAL_QKV", "0", 1);
    setenv("TINYENGINE_METAL_ARGMAX", "0", 1);
    setenv("TINYENGINE_TEMPERATURE", "0", 1);
    rq_model = (te_model *)calloc(1, sizeof(*rq_model));
    if (rq_model == NULL) return TE_STATUS_OUT_OF_MEMORY;
    rq_model->path = te_strdup(path);
    rq_model->options.abi_version = TE_ABI_VERSION;
    rq_model->options.context_tokens = context_tokens;
    rq_model->options.batch_tokens = 128;
    te_status st = te_model_parse_gguf(rq_model, path);
    if (st != TE_STATUS_OK) {
        free(rq_model->path);
        free(rq_model);
        rq_model = NULL;
        return st;
    }
    rq_ctx.model = rq_model;
    rq_ctx.options = rq_model->options;
    st = te_qwen_state_init(&rq_state, &rq_ctx, 0);
    if (st != TE_STATUS_OK) {
        rq_close();
        return st;
    }
    rq_state.temperature = 0.0f;
    rq_ready = 1;
    return TE_STATUS_OK;
}

int rq_dims(uint64_t *out) {
    if (!rq_ready || out == NULL) return TE_STATUS_INVALID_ARGUMENT;
    out[0] = rq_state.hidden;
    out[1] = rq_state.ffn;
    out[2] = rq_state.layers;
    out[3] = rq_state.heads;
    out[4] = rq_state.kv_heads;
    out[5] = rq_state.head_dim;
    out[6] = rq_state.vocab;
    out[7] = rq_state.context_tokens;
    return TE_STATUS_OK;
}

int rq_forward(uint32_t token, size_t position, float *hidden_out) {
    if (!rq_ready) return TE_STATUS_INVALID_ARGUMENT;
    const te_status st = te_qwen_forward_token(&rq_ctx, &rq_state, token, position);
    if (st == TE_STATUS_OK && hidden_out != NULL) {
        memcpy(hidden_out, rq_state.hidden_buf, rq_state.hidden * sizeof(float));
    }
    return st;
}

int rq_project(float *logits_out, uint32_t *token_out) {
    if (!rq_ready || token_out == NULL) return TE_STATUS_INVALID_ARGUMENT;
    const te_status st = te_qwen_project_next(&rq_ctx, &rq_state, token_out);
    if (st == TE_STATUS_OK && logits_out != NULL) {
        memcpy(logits_out, rq_state.logits, rq_state.vocab * sizeof(float));
    }
    return st;
}
