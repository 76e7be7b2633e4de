/* TEST INFRASTRUCTURE ONLY.  Stand-ins for the reference's Metal entry
 * points (declared in c/src/metal_backend.h) when its CPU forward pass is
 * built as a checker on a machine without Metal: every one answers
 * TE_STATUS_UNSUPPORTED, which sends the reference's callers down their own
 * CPU branches (qwen.c:936-1110, ops.c te_model_matvec_f32).  The
 * prototypes are the header's; the parameter names are placeholders. */
#include "metal_backend.h"

te_status te_metal_matvec_f32(const void * a0, size_t a1, uint64_t a2, uint32_t a3, const float * a4, size_t a5, size_t a6, float * a7) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_matvec_argmax_f32(const void * a0, size_t a1, uint64_t a2, uint32_t a3, const float * a4, size_t a5, size_t a6, uint32_t * a7) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_project_argmax_f32(const void * a0, size_t a1, uint64_t a2, uint32_t a3, const float * a4, const float * a5, size_t a6, size_t a7, float a8, uint32_t * a9) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_matvec2_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint32_t a4, const float * a5, size_t a6, size_t a7, float * a8, float * a9) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_matvec_batch_f32(const void * a0, size_t a1, uint64_t a2, uint32_t a3, const float * a4, size_t a5, size_t a6, size_t a7, float * a8) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_qkv_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint64_t a4, uint32_t a5, const float * a6, size_t a7, size_t a8, float * a9, float * a10, float * a11) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10; (void)a11;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_qkv_batch_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint64_t a4, uint32_t a5, const float * a6, size_t a7, size_t a8, size_t a9, float * a10, float * a11, float * a12) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10; (void)a11; (void)a12;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_attention_qk_mma_f32(const float * a0, const float * a1, size_t a2, size_t a3, size_t a4, float * a5) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_attention_tile_mma_f32(const float * a0, const float * a1, const float * a2, size_t a3, size_t a4, size_t a5, float * a6) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_attention_stream_mma_f32(const float * a0, const float * a1, const float * a2, size_t a3, size_t a4, size_t a5, float * a6) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_attention_causal_mma_f32(const float * a0, const float * a1, const float * a2, size_t a3, size_t a4, size_t a5, size_t a6, float * a7) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_mlp_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint64_t a4, uint32_t a5, const float * a6, size_t a7, size_t a8, float * a9) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_post_attn_mlp_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint64_t a4, uint64_t a5, uint32_t a6, const float * a7, const float * a8, const float * a9, size_t a10, size_t a11, float a12, float * a13) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10; (void)a11; (void)a12; (void)a13;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_mlp_batch_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint64_t a4, uint32_t a5, const float * a6, size_t a7, size_t a8, size_t a9, float * a10) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_post_attn_mlp_batch_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint64_t a4, uint64_t a5, uint32_t a6, const float * a7, const float * a8, const float * a9, size_t a10, size_t a11, size_t a12, float a13, float * a14) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10; (void)a11; (void)a12; (void)a13; (void)a14;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_decode_layer_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint64_t a4, uint64_t a5, uint64_t a6, uint64_t a7, uint64_t a8, uint32_t a9, const float * a10, const float * a11, const float * a12, const float * a13, const float * a14, const float * a15, const float * a16, const float * a17, float * a18, float * a19, size_t a20, size_t a21, size_t a22, size_t a23, size_t a24, size_t a25, size_t a26, size_t a27, float a28, float * a29) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10; (void)a11; (void)a12; (void)a13; (void)a14; (void)a15; (void)a16; (void)a17; (void)a18; (void)a19; (void)a20; (void)a21; (void)a22; (void)a23; (void)a24; (void)a25; (void)a26; (void)a27; (void)a28; (void)a29;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_decode_all_layers_f32(const void * a0, size_t a1, const uint64_t * a2, const uint64_t * a3, const uint64_t * a4, const uint64_t * a5, const uint64_t * a6, const uint64_t * a7, const uint64_t * a8, size_t a9, uint32_t a10, const float * a11, const float * a12, const float * a13, const float * a14, const float * a15, const float * a16, const float * a17, const float * a18, float * a19, float * a20, size_t a21, size_t a22, size_t a23, size_t a24, size_t a25, size_t a26, size_t a27, size_t a28, float a29, float * a30, uint64_t a31, uint32_t a32, const float * a33, size_t a34, uint32_t * a35) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10; (void)a11; (void)a12; (void)a13; (void)a14; (void)a15; (void)a16; (void)a17; (void)a18; (void)a19; (void)a20; (void)a21; (void)a22; (void)a23; (void)a24; (void)a25; (void)a26; (void)a27; (void)a28; (void)a29; (void)a30; (void)a31; (void)a32; (void)a33; (void)a34; (void)a35;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_prefill_layer_f32(const void * a0, size_t a1, uint64_t a2, uint64_t a3, uint64_t a4, uint64_t a5, uint64_t a6, uint64_t a7, uint64_t a8, uint32_t a9, const float * a10, const float * a11, const float * a12, const float * a13, const float * a14, const float * a15, const float * a16, const float * a17, float * a18, float * a19, size_t a20, size_t a21, size_t a22, size_t a23, size_t a24, size_t a25, size_t a26, size_t a27, float a28, float * a29) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10; (void)a11; (void)a12; (void)a13; (void)a14; (void)a15; (void)a16; (void)a17; (void)a18; (void)a19; (void)a20; (void)a21; (void)a22; (void)a23; (void)a24; (void)a25; (void)a26; (void)a27; (void)a28; (void)a29;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_prefill_all_layers_f32(const void * a0, size_t a1, const uint64_t * a2, const uint64_t * a3, const uint64_t * a4, const uint64_t * a5, const uint64_t * a6, const uint64_t * a7, const uint64_t * a8, size_t a9, uint32_t a10, const float * a11, const float * a12, const float * a13, const float * a14, const float * a15, const float * a16, const float * a17, const float * a18, float * a19, float * a20, size_t a21, size_t a22, size_t a23, size_t a24, size_t a25, size_t a26, size_t a27, size_t a28, float a29, float * a30) {
  (void)a0; (void)a1; (void)a2; (void)a3; (void)a4; (void)a5; (void)a6; (void)a7; (void)a8; (void)a9; (void)a10; (void)a11; (void)a12; (void)a13; (void)a14; (void)a15; (void)a16; (void)a17; (void)a18; (void)a19; (void)a20; (void)a21; (void)a22; (void)a23; (void)a24; (void)a25; (void)a26; (void)a27; (void)a28; (void)a29; (void)a30;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_warm_model(const void * a0, size_t a1) {
  (void)a0; (void)a1;
  return TE_STATUS_UNSUPPORTED;
}

te_status te_metal_release_model(const void * a0, size_t a1) {
  (void)a0; (void)a1;
  return TE_STATUS_UNSUPPORTED;
}
