"""Generates tests/golden/golden.npz from the reference's own CPU code.

Runs TinyEngine's c/src/ops.c, compiled from the reference sources by
oracle/Makefile into oracle/_ref/libteref.so, on seeded inputs.  The fixture
pins the oracle restatement (oracle/te_oracle.c) and the CUDA path without
needing the reference at test time.  Regenerate with
    make -C oracle && python tests/golden/make_golden.py
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from oracle import oracle as O  # noqa: E402

THETA = 1e6


def quant_matrix(rng, ggml_type: int, rows: int, cols: int) -> np.ndarray:
    """Random GGUF Q4_0 (type 2: f16 scale + 16 nibble bytes) or Q8_0 (type 8: f16 scale + 32 int8)
    blocks of 32 weights, row-major [rows][cols / 32 blocks] as raw bytes."""
    blocks = cols // 32
    width = 18 if ggml_type == 2 else 34
    w = np.zeros((rows, blocks, width), np.uint8)
    scales = (rng.standard_normal((rows, blocks)) * 0.02).astype(np.float16)
    w[:, :, 0:2] = scales.view(np.uint8).reshape(rows, blocks, 2)
    w[:, :, 2:] = rng.integers(0, 256, (rows, blocks, width - 2), dtype=np.uint8)
    return w.reshape(-1)


def make_matvec(ref, dst: Path) -> None:
    """te_model_matvec_f32 of the reference (its CPU row loop) on seeded GGUF matrices."""
    rng = np.random.default_rng(20261202)
    g: dict[str, np.ndarray] = {}
    for i, (ggml_type, rows, cols) in enumerate([(2, 32, 896), (2, 48, 1024), (8, 32, 896), (8, 48, 1024)]):
        w = quant_matrix(rng, ggml_type, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        g[f"mv{i}_meta"] = np.array([ggml_type, rows, cols], np.int64)
        g[f"mv{i}_w"] = w
        g[f"mv{i}_x"] = x
        g[f"mv{i}_out"] = ref.model_matvec_f32(ggml_type, w, rows, cols, x)
    np.savez_compressed(dst, **g)
    print("wrote", dst)


def main() -> None:
    ref = O.ref()
    rng = np.random.default_rng(20261201)
    g: dict[str, np.ndarray] = {}

    # Known-answer inputs of c/tests/kernel_ops.c:330-356, outputs from the reference.
    v = np.array([1, 2, 3, 4], np.float32)
    ref.rope_f32(v, 1, 4, 1, 10000.0)
    g["kat_rope_out"] = v
    g["kat_attn_out"] = ref.attention_decode_f32(np.array([1, 0, 0, 1], np.float32), np.array([1, 0, 0, 1], np.float32),
                                                 np.array([10, 20, 30, 40], np.float32), 1, 2, 1, 2)

    # RoPE cases: (heads, head_dim, position, theta)
    rope_cases = [(14, 64, 512, THETA), (2, 128, 4096, THETA), (4, 128, 32768, THETA), (1, 2, 0, 1e4), (3, 6, 7, 10.0)]
    for i, (h, hd, pos, th) in enumerate(rope_cases):
        x = rng.standard_normal(h * hd).astype(np.float32)
        y = x.copy()
        ref.rope_f32(y, h, hd, pos, th)
        g[f"rope{i}_in"], g[f"rope{i}_out"] = x, y
        g[f"rope{i}_shape"] = np.array([h, hd, pos], np.int64)
        g[f"rope{i}_theta"] = np.array([th], np.float32)

    # Attention cases with f16-representable K/V (the engine's cache type):
    # (heads, kv_heads, head_dim, n_tokens)
    attn_cases = [(14, 2, 64, 513), (16, 2, 128, 300), (28, 4, 128, 65), (4, 4, 64, 1), (8, 1, 128, 1030),
                  (4, 2, 64, 129)]
    for i, (h, hkv, hd, n) in enumerate(attn_cases):
        k = rng.standard_normal((n, hkv, hd)).astype(np.float16)
        vv = rng.standard_normal((n, hkv, hd)).astype(np.float16)
        q = rng.standard_normal((h, hd)).astype(np.float32)
        out = ref.attention_decode_f32(q.ravel(), k.astype(np.float32).ravel(), vv.astype(np.float32).ravel(),
                                       n - 1, h, hkv, hd)
        g[f"attn{i}_q"], g[f"attn{i}_k"], g[f"attn{i}_v"] = q, k, vv
        g[f"attn{i}_out"] = out.reshape(h, hd)
        g[f"attn{i}_shape"] = np.array([h, hkv, hd, n], np.int64)

    # Append: raw fp32 K rows rotated by the reference at positions p0.., then f16 RNE.
    n, hkv, hd, p0 = 70, 2, 64, 3
    kraw = rng.standard_normal((n, hkv, hd)).astype(np.float32)
    kro = kraw.copy()
    for t in range(n):
        row = np.ascontiguousarray(kro[t]).ravel()
        ref.rope_f32(row, hkv, hd, p0 + t, THETA)
        kro[t] = row.reshape(hkv, hd)
    g["append_kraw"] = kraw
    g["append_kbits"] = kro.astype(np.float16).view(np.uint16)
    g["append_shape"] = np.array([n, hkv, hd, p0], np.int64)

    # Causal prefill (c/src/qwen.c:810-824): decode per position over the growing cache.
    s, h, hkv, hd = 37, 4, 2, 64
    q = rng.standard_normal((s, h, hd)).astype(np.float32)
    k = rng.standard_normal((s, hkv, hd)).astype(np.float16).astype(np.float32)
    vv = rng.standard_normal((s, hkv, hd)).astype(np.float16).astype(np.float32)
    out = np.zeros((s, h, hd), np.float32)
    for t in range(s):
        out[t] = ref.attention_decode_f32(q[t].ravel(), k.ravel(), vv.ravel(), t, h, hkv, hd).reshape(h, hd)
    g["prefill_q"], g["prefill_k"], g["prefill_v"], g["prefill_out"] = q, k.astype(np.float16), vv.astype(np.float16), out
    g["prefill_shape"] = np.array([s, h, hkv, hd], np.int64)

    dst = Path(__file__).resolve().parent / "golden.npz"
    np.savez_compressed(dst, **g)
    print(f"wrote {dst} ({dst.stat().st_size} bytes, {len(g)} arrays)")
    make_matvec(ref, Path(__file__).resolve().parent / "golden_matvec.npz")


if __name__ == "__main__":
    main()
