"""C-ABI surface without a GPU: every declared symbol is exported, argument
guards return the reference's status codes, and compute entry points refuse
to run (no CPU fallback) when no CUDA device is present.  Mirrors the
reference's generated guard tests (c/tests/generate_metal_guard_tests.py:19-81)."""
import ctypes
import re

import numpy as np
import pytest

from tinymetalagent_b200 import runtime as R

ROOT = __import__("pathlib").Path(__file__).resolve().parents[1]


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = h.read_text()
        names.update(re.findall(r"TE_API\s+[\w\s\*]+?\b(te_\w+)\s*\(", text))
    return names


def test_every_declared_symbol_is_exported(lib):
    names = declared_symbols()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert declared_symbols() == set(R.SIGNATURES)


def test_strerror_strings(lib):
    # c/src/tinyengine.c:17-34
    exp = ["ok", "invalid argument", "I/O error", "unsupported", "out of memory", "runtime error"]
    assert [lib.te_strerror(i).decode() for i in range(6)] == exp
    assert lib.te_strerror(99).decode() == "unknown error"


def test_rope_guards(lib):
    v = np.zeros(8, np.float32)
    p = v.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    assert lib.te_rope_f32(None, 1, 4, 0, 1e4) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_rope_f32(p, 0, 4, 0, 1e4) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_rope_f32(p, 1, 0, 0, 1e4) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_rope_f32(p, 1, 3, 0, 1e4) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_rope_f32(p, 1, 4, 0, 0.0) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_rope_f32(p, 1, 4, 0, -1.0) == R.TE_STATUS_INVALID_ARGUMENT


def test_attention_guards(lib):
    a = np.zeros(64, np.float32)
    p = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    f = lib.te_attention_decode_f32
    assert f(None, p, p, 0, 2, 1, 2, p) == R.TE_STATUS_INVALID_ARGUMENT
    assert f(p, None, p, 0, 2, 1, 2, p) == R.TE_STATUS_INVALID_ARGUMENT
    assert f(p, p, None, 0, 2, 1, 2, p) == R.TE_STATUS_INVALID_ARGUMENT
    assert f(p, p, p, 0, 2, 1, 2, None) == R.TE_STATUS_INVALID_ARGUMENT
    assert f(p, p, p, 0, 0, 1, 2, p) == R.TE_STATUS_INVALID_ARGUMENT
    assert f(p, p, p, 0, 2, 0, 2, p) == R.TE_STATUS_INVALID_ARGUMENT
    assert f(p, p, p, 0, 2, 1, 0, p) == R.TE_STATUS_INVALID_ARGUMENT
    assert f(p, p, p, 0, 3, 2, 2, p) == R.TE_STATUS_INVALID_ARGUMENT
    assert f(p, p, p, 2**64 - 1, 2, 1, 2, p) == R.TE_STATUS_UNSUPPORTED  # position == SIZE_MAX


def test_engine_api_null_guards(lib):
    assert lib.te_attn_engine_create(None, None) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_kv_cache_create(None, None, None) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_attn_engine_synchronize(None) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_kv_append_rope(None, 0, 1, 0, None, None, 1, 0) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_attention_decode(None, 0, 1, None, 1, None, None, None, None, 8, None, 0) == \
        R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_attention_prefill(None, 0, 1, 0, None, None, None, 1, 8, None, 0) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_attention_merge_partials(None, None, 1, 1, 64, None, 0) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_kv_cache_seq_reset(None, 0, 0) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_kv_cache_set_qkv_bias(None, 0, 1, 8, None, None, None) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_attn_exchange_create(None, 2, 0, 8, 128, None, None) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_attn_exchange_connect(None, None) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_attn_exchange_merge(None, None, None) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_matvec_gguf(None, 4, None, 1, 32, None, 1, None, 0) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_matvec_gguf_fused(None, 4, None, 1, 32, None, 1, None, 1e-6, None, R.TE_ATTN_RMSNORM_INPUT) == \
        R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_qwen_step_create(None, None, None) == R.TE_STATUS_INVALID_ARGUMENT
    assert lib.te_qwen_step_run(None, 0, None, None, None, None, 0) == R.TE_STATUS_INVALID_ARGUMENT
    lib.te_qwen_step_free(None)
    lib.te_attn_exchange_free(None)
    lib.te_attn_engine_free(None)
    lib.te_kv_cache_free(None)
    assert lib.te_attn_engine_launch_count(None) == 0


def test_qwen_step_desc_layout():
    # te_qwen_step_desc (include/tinyengine_attn.h): six uint32, a float, five
    # uint32 quant kinds, then nine pointers
    d = R.QwenStepDesc
    assert ctypes.sizeof(d) == 120
    assert d.eps.offset == 24 and d.quant_qkv.offset == 28 and d.quant_head.offset == 44
    assert d.w_qkv.offset == 48 and d.embedding.offset == 112


def test_qwen_step_checks_layer_lists_before_the_library():
    # one matrix per layer for each projection, checked by the binding before any C call
    class Fake:
        engine = None
        lib = None
    with pytest.raises(ValueError):
        R.QwenStep(Fake(), layers=2, hidden=64, heads=1, ffn=64, vocab=8, eps=1e-6,
                   quants={"qkv": 4, "o": 4, "gu": 4, "down": 4, "head": 8}, w_qkv=[0], w_o=[0, 0],
                   w_gu=[0, 0], w_down=[0, 0], w_head=0, attn_norm=0, ffn_norm=0, out_norm=0, embedding=0)


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback_without_gpu(lib):
    # Valid arguments, no device: the library must refuse, not compute on the CPU.
    v = np.array([1, 2, 3, 4], np.float32)
    p = v.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    assert lib.te_rope_f32(p, 1, 4, 1, 1e4) == R.TE_STATUS_UNSUPPORTED
    assert np.array_equal(v, [1, 2, 3, 4])
    q = np.array([1, 0, 0, 1], np.float32)
    out = np.full(4, -7.0, np.float32)
    fp = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))  # noqa: E731
    assert lib.te_attention_decode_f32(fp(q), fp(q), fp(q), 1, 2, 1, 2, fp(out)) == R.TE_STATUS_UNSUPPORTED
    assert np.all(out == -7.0)
    with pytest.raises(R.TinyEngineError) as ei:
        R.AttnEngine(0)
    assert ei.value.status == R.TE_STATUS_UNSUPPORTED


def test_set_qkv_bias_checks_shapes_before_the_library():
    # The binding validates the bias widths (heads * head_dim, kv_heads * head_dim)
    # and row counts before calling the C function.
    cache = object.__new__(R.KVCache)
    cache.head_dim, cache.kv_heads = 128, 2
    with pytest.raises(ValueError):
        cache.set_qkv_bias(0, 16, np.zeros((2, 16 * 128 + 1), np.float32))
    with pytest.raises(ValueError):
        cache.set_qkv_bias(0, 16, np.zeros((2, 16 * 128), np.float32), np.zeros((3, 2 * 128), np.float32))
    with pytest.raises(ValueError):
        cache.set_qkv_bias(0, 16)
