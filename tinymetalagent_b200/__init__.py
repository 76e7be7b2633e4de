"""B200-native attention stage for TinyEngine (Qwen2-style GQA).

The product is ``libtinyengine.so`` (built from ``csrc/``) behind the C ABI in
``include/tinyengine.h`` and ``include/tinyengine_attn.h``; this package holds
its ctypes binding, the multi-GPU host orchestration, and the qwen2 decode
step built on them (``qwen.QwenDecoder``, with the GGUF reader ``gguf``).
"""
from .runtime import (  # noqa: F401
    TE_ATTN_ACCUMULATE,
    TE_ATTN_ADVANCE,
    TE_ATTN_HOST_BUFFERS,
    TE_ATTN_INPUT_F16,
    TE_ATTN_NO_ROPE,
    TE_ATTN_PARTIAL,
    TE_ATTN_QKV_BIAS,
    TE_ATTN_RMSNORM_INPUT,
    TE_ATTN_SWIGLU_INPUT,
    TE_ATTN_EXACT_Q,
    TE_ATTN_STEP_HEAD,
    AttnEngine,
    KVCache,
    QwenStep,
    TinyEngineError,
    attention_decode_f32,
    load_library,
    rope_f32,
)
