"""Writes a small synthetic Qwen2 GGUF file (TEST INFRASTRUCTURE).

No model file is available offline, so the layer-step parity tests run the
reference's CPU forward pass and this repository's GPU layer step on the same
seeded random model: GGUF v3 (little-endian: magic, version, tensor and
key-value counts, the key-values, the tensor infos, then the tensor data at
32-byte aligned offsets), the qwen2 metadata keys the reference's parser
reads (c/src/gguf.c:370-500), and the tensor names its forward pass uses
(c/src/qwen.c:936-952 and the state set-up at :424-629).  No tokenizer arrays:
the vocabulary size comes from token_embd.weight, as the parser allows
(gguf.c:500-508).

Weights are seeded N(0, sigma^2)-scale values stored as GGUF Q4_0 / Q8_0
blocks (random codes, per-block f16 scales drawn around sigma / code std), so
that activations stay O(1) through the layers; norms and biases are fp32.
"""
from __future__ import annotations

import struct
from pathlib import Path

import numpy as np

GGML_F32, GGML_Q4_0, GGML_Q8_0 = 0, 2, 8
_T_U32, _T_I32, _T_F32, _T_STRING, _T_ARRAY = 4, 5, 6, 8, 9
_ALIGN = 32


def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def quant_blocks(rng, ggml_type: int, rows: int, cols: int, sigma: float) -> np.ndarray:
    """rows x cols weights as raw GGUF blocks (row-major), weight std about sigma."""
    blocks = cols // 32
    if ggml_type == GGML_Q4_0:
        width, code_std = 18, 4.6   # codes 0..15, offset 8
    else:
        width, code_std = 34, 74.0  # int8 codes
    w = np.zeros((rows, blocks, width), np.uint8)
    scales = (sigma / code_std * (1.0 + 0.25 * rng.standard_normal((rows, blocks)))).astype(np.float16)
    w[:, :, 0:2] = scales.view(np.uint8).reshape(rows, blocks, 2)
    w[:, :, 2:] = np.frombuffer(rng.bytes(rows * blocks * (width - 2)), np.uint8).reshape(rows, blocks, width - 2)
    return w.reshape(-1)


def write_qwen2(path: Path, *, layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=512, context=128,
                quant_attn=GGML_Q8_0, quant_ffn=GGML_Q4_0, seed=1, rope_base=1e6, eps=1e-6, tied=False,
                tokenizer=False, alignment=None, version=3) -> dict:
    """Write the model; returns its dimensions.  tied: no output.weight, so the lm_head is
    token_embd.weight (as in Qwen2.5-0.5B; the reference falls back to it, qwen.c:1305).
    tokenizer: also write tokenizer.ggml.* arrays (vocab strings, int32 token types, merges) -- the
    vocabulary size then comes from them; alignment: write general.alignment (u32) and lay the data out
    on it; version: 2 or 3 (same layout for these types)."""
    rng = np.random.default_rng(seed)
    hd = hidden // heads
    kv = kv_heads * hd
    tensors: list[tuple[str, int, tuple[int, ...], bytes]] = []

    def mat(name, qt, rows, cols, sigma):
        tensors.append((name, qt, (cols, rows), quant_blocks(rng, qt, rows, cols, sigma).tobytes()))

    def vec(name, values):
        tensors.append((name, GGML_F32, (values.size,), values.astype(np.float32).tobytes()))

    mat("token_embd.weight", GGML_Q8_0, vocab, hidden, 1.0)
    for layer in range(layers):
        p = f"blk.{layer}."
        vec(p + "attn_norm.weight", 1.0 + 0.1 * rng.standard_normal(hidden))
        mat(p + "attn_q.weight", quant_attn, hidden, hidden, 1.0 / np.sqrt(hidden))
        vec(p + "attn_q.bias", 0.3 * rng.standard_normal(hidden))
        mat(p + "attn_k.weight", quant_attn, kv, hidden, 1.0 / np.sqrt(hidden))
        vec(p + "attn_k.bias", 0.3 * rng.standard_normal(kv))
        mat(p + "attn_v.weight", quant_attn, kv, hidden, 1.0 / np.sqrt(hidden))
        vec(p + "attn_v.bias", 0.3 * rng.standard_normal(kv))
        mat(p + "attn_output.weight", quant_attn, hidden, hidden, 0.5 / np.sqrt(hidden))
        vec(p + "ffn_norm.weight", 1.0 + 0.1 * rng.standard_normal(hidden))
        mat(p + "ffn_gate.weight", quant_ffn, ffn, hidden, 1.0 / np.sqrt(hidden))
        mat(p + "ffn_up.weight", quant_ffn, ffn, hidden, 1.0 / np.sqrt(hidden))
        mat(p + "ffn_down.weight", quant_ffn, hidden, ffn, 0.5 / np.sqrt(ffn))
    vec("output_norm.weight", 1.0 + 0.1 * rng.standard_normal(hidden))
    if not tied:
        mat("output.weight", GGML_Q8_0, vocab, hidden, 4.0 / np.sqrt(hidden))  # logits O(4): clear greedy margins

    align = alignment or _ALIGN
    kvs = [
        ("general.architecture", _T_STRING, "qwen2"),
        ("general.name", _T_STRING, "synthetic-qwen2"),
        ("qwen2.context_length", _T_U32, context),
        ("qwen2.embedding_length", _T_U32, hidden),
        ("qwen2.block_count", _T_U32, layers),
        ("qwen2.feed_forward_length", _T_U32, ffn),
        ("qwen2.attention.head_count", _T_U32, heads),
        ("qwen2.attention.head_count_kv", _T_U32, kv_heads),
        ("qwen2.rope.freq_base", _T_F32, rope_base),
        ("qwen2.attention.layer_norm_rms_epsilon", _T_F32, eps),
    ]
    if alignment is not None:
        kvs.append(("general.alignment", _T_U32, alignment))
    if tokenizer:
        kvs += [
            ("tokenizer.ggml.model", _T_STRING, "gpt2"),
            ("tokenizer.ggml.tokens", _T_ARRAY, (_T_STRING, [f"tok{i}" for i in range(vocab)])),
            ("tokenizer.ggml.token_type", _T_ARRAY, (_T_I32, [1] * vocab)),
            ("tokenizer.ggml.merges", _T_ARRAY, (_T_STRING, ["t o", "to k"])),
            ("tokenizer.ggml.eos_token_id", _T_U32, vocab - 1),
        ]
    out = bytearray(b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(kvs)))

    def value_bytes(t, value):
        if t == _T_STRING:
            return _gguf_str(value)
        if t == _T_U32:
            return struct.pack("<I", value)
        if t == _T_I32:
            return struct.pack("<i", value)
        if t == _T_F32:
            return struct.pack("<f", value)
        etype, items = value  # array
        return struct.pack("<IQ", etype, len(items)) + b"".join(value_bytes(etype, v) for v in items)

    for key, t, value in kvs:
        out += _gguf_str(key) + struct.pack("<I", t) + value_bytes(t, value)
    offset = 0
    offsets = []
    for name, qt, dims, data in tensors:
        offsets.append(offset)
        out += _gguf_str(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        out += struct.pack("<IQ", qt, offset)
        offset += (len(data) + align - 1) // align * align
    out += b"\0" * (-len(out) % align)
    base = len(out)
    for (name, qt, dims, data), off in zip(tensors, offsets):
        out += b"\0" * (base + off - len(out))
        out += data
    Path(path).write_bytes(bytes(out))
    return {"layers": layers, "hidden": hidden, "heads": heads, "kv_heads": kv_heads, "head_dim": hd, "ffn": ffn,
            "vocab": vocab, "context": context, "rope_base": rope_base, "eps": eps}
