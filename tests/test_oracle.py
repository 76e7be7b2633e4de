"""The CPU oracle restatement against the reference: KATs, golden vectors and,
where the reference build exists, the reference's compiled ops.c directly."""
import math
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O


def test_rope_kat(port):
    # c/tests/kernel_ops.c:330-339
    v = np.array([1, 2, 3, 4], np.float32)
    assert port.rope_f32(v, 1, 4, 1, 10000.0) == 0
    s0, c0, s1, c1 = math.sin(1.0), math.cos(1.0), math.sin(0.01), math.cos(0.01)
    exp = [1 * c0 - 3 * s0, 2 * c1 - 4 * s1, 3 * c0 + 1 * s0, 4 * c1 + 2 * s1]
    np.testing.assert_allclose(v, exp, atol=1e-6)


def test_attention_kat(port):
    # c/tests/kernel_ops.c:341-356
    out = port.attention_decode_f32(np.array([1, 0, 0, 1], np.float32), np.array([1, 0, 0, 1], np.float32),
                                    np.array([10, 20, 30, 40], np.float32), 1, 2, 1, 2)
    s = 1 / math.sqrt(2)
    hi, lo = math.exp(s) / (math.exp(s) + 1), 1 / (math.exp(s) + 1)
    np.testing.assert_allclose(out, [hi * 10 + lo * 30, hi * 20 + lo * 40, lo * 10 + hi * 30, lo * 20 + hi * 40],
                               atol=1e-5)


def test_golden_kats_bit_exact(port, golden):
    v = np.array([1, 2, 3, 4], np.float32)
    port.rope_f32(v, 1, 4, 1, 10000.0)
    assert np.array_equal(v, golden["kat_rope_out"])
    out = port.attention_decode_f32(np.array([1, 0, 0, 1], np.float32), np.array([1, 0, 0, 1], np.float32),
                                    np.array([10, 20, 30, 40], np.float32), 1, 2, 1, 2)
    assert np.array_equal(out, golden["kat_attn_out"])


def test_golden_rope_bit_exact(port, golden):
    i = 0
    while f"rope{i}_in" in golden:
        h, hd, pos = (int(x) for x in golden[f"rope{i}_shape"])
        x = golden[f"rope{i}_in"].copy()
        port.rope_f32(x, h, hd, pos, float(golden[f"rope{i}_theta"][0]))
        assert np.array_equal(x, golden[f"rope{i}_out"]), i
        i += 1
    assert i >= 5


def test_golden_attention_bit_exact(port, golden):
    i = 0
    while f"attn{i}_q" in golden:
        h, hkv, hd, n = (int(x) for x in golden[f"attn{i}_shape"])
        out = port.attention_decode_f32(golden[f"attn{i}_q"].ravel(), golden[f"attn{i}_k"].astype(np.float32).ravel(),
                                        golden[f"attn{i}_v"].astype(np.float32).ravel(), n - 1, h, hkv, hd)
        assert np.array_equal(out.reshape(h, hd), golden[f"attn{i}_out"]), i
        i += 1
    assert i >= 6


def test_golden_append_bit_exact(port, golden):
    n, hkv, hd, p0 = (int(x) for x in golden["append_shape"])
    kraw = golden["append_kraw"]
    kb, vb = port.append_rope_f16(kraw, kraw, p0, hkv, hd, 1e6)
    assert np.array_equal(kb, golden["append_kbits"])
    assert np.array_equal(vb, kraw.astype(np.float16).view(np.uint16))


def test_golden_prefill_bit_exact(port, golden):
    s, h, hkv, hd = (int(x) for x in golden["prefill_shape"])
    out = port.causal_prefill_f32(golden["prefill_q"], golden["prefill_k"].astype(np.float32),
                                  golden["prefill_v"].astype(np.float32), s, h, hkv, hd)
    assert np.array_equal(out, golden["prefill_out"])


def test_rope_table_matches_per_call_rope(port):
    # qwen.c:531-539 table == te_rope_f32 per-call trig (ops.c:308-312), bit for bit.
    cos, sin = port.rope_table(600, 64, 1e6)
    rng = np.random.default_rng(1)
    for pos in (0, 1, 511, 599):
        x = rng.standard_normal(2 * 64).astype(np.float32)
        a = x.copy()
        port.rope_f32(a, 2, 64, pos, 1e6)
        b = x.copy()
        port.lib.or_rope_cached.argtypes = [O._f32p, O._sz, O._sz, O._f32p, O._f32p, O._sz]
        port.lib.or_rope_cached(b.ctypes.data_as(O._f32p), 2, 64, cos.ctypes.data_as(O._f32p),
                                sin.ctypes.data_as(O._f32p), pos)
        assert np.array_equal(a, b)


def test_f16_conversion_matches_ieee_rne(port):
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.standard_normal(50000).astype(np.float32) * np.float32(1000),
                        rng.standard_normal(50000).astype(np.float32) * np.float32(1e-5),
                        np.array([65504, 65519.99, 65520, 2.9802322e-08, 5.96e-8, -0.0, np.inf, -np.inf], np.float32)])
    with np.errstate(over="ignore"):
        expect = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(port.f32_to_f16_bits(x), expect)
    assert np.array_equal(port.f16_bits_to_f32(expect), expect.view(np.float16).astype(np.float32))


def test_partials_merge_equals_full(port):
    rng = np.random.default_rng(3)
    h, hkv, hd, n = 8, 2, 64, 300
    q = rng.standard_normal(h * hd).astype(np.float32)
    k = rng.standard_normal(n * hkv * hd).astype(np.float32)
    v = rng.standard_normal(n * hkv * hd).astype(np.float32)
    full = port.attention_decode_f32(q, k, v, n - 1, h, hkv, hd).reshape(h, hd)
    cuts = [0, 1, 77, 200, 300]
    parts = np.stack([port.decode_partial_f32(q, k, v, a, b, h, hkv, hd) for a, b in zip(cuts[:-1], cuts[1:])])
    merged = port.merge_partials_f32(parts, h, hd)
    np.testing.assert_allclose(merged, full, atol=1e-5, rtol=1e-4)


@pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) absent")
def test_port_equals_reference_random(port):
    ref = O.ref()
    rng = np.random.default_rng(4)
    for (h, hkv, hd, n) in [(14, 2, 64, 513), (16, 2, 128, 1100), (3, 1, 10, 5), (28, 4, 128, 2)]:
        q = rng.standard_normal(h * hd).astype(np.float32)
        k = rng.standard_normal(n * hkv * hd).astype(np.float32)
        v = rng.standard_normal(n * hkv * hd).astype(np.float32)
        assert np.array_equal(port.attention_decode_f32(q, k, v, n - 1, h, hkv, hd),
                              ref.attention_decode_f32(q, k, v, n - 1, h, hkv, hd))
        x = rng.standard_normal(h * hd).astype(np.float32)
        y = x.copy()
        port.rope_f32(x, h, hd, n, 1e6)
        ref.rope_f32(y, h, hd, n, 1e6)
        assert np.array_equal(x, y)


def test_oracle_rejects_like_reference(port):
    z = np.zeros(8, np.float32)
    assert port.rope_f32(z, 1, 3, 0, 1e4) == 1      # odd head_dim
    assert port.rope_f32(z, 1, 4, 0, 0.0) == 1      # theta <= 0
    with pytest.raises(RuntimeError):
        port.attention_decode_f32(z, z, z, 0, 3, 2, 1)  # heads % kv_heads != 0


def test_golden_matvec_bit_exact(port):
    """The restated Q4_0 / Q8_0 row dot products equal the reference's te_model_matvec_f32
    (its CPU row loop, c/src/ops.c:216-262 and :584-620) on the committed fixture."""
    g = dict(np.load(Path(__file__).resolve().parent / "golden" / "golden_matvec.npz"))
    for i in range(4):
        ggml_type, rows, cols = (int(v) for v in g[f"mv{i}_meta"])
        fn = port.matvec_q4_0_f32 if ggml_type == 2 else port.matvec_q8_0_f32
        assert np.array_equal(fn(g[f"mv{i}_w"], rows, cols, g[f"mv{i}_x"]), g[f"mv{i}_out"])


@pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) absent")
def test_matvec_port_equals_reference_random(port):
    import sys
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    from make_golden import quant_matrix
    ref = O.ref()
    rng = np.random.default_rng(77)
    for ggml_type, rows, cols in [(2, 1, 32), (2, 600, 2048), (8, 5, 3584), (8, 520, 512)]:
        w = quant_matrix(rng, ggml_type, rows, cols)
        x = rng.standard_normal(cols).astype(np.float32)
        fn = port.matvec_q4_0_f32 if ggml_type == 2 else port.matvec_q8_0_f32
        assert np.array_equal(fn(w, rows, cols, x), ref.model_matvec_f32(ggml_type, w, rows, cols, x))
