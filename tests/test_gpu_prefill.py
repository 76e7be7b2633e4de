"""GPU parity of the tcgen05 causal prefill against the CPU oracle.

The reference's causal prefill is te_attention_decode_f32 called once per
prompt token over the cache filled so far (c/src/qwen.c:810-824).  Bars: the
f16 cache is bit-exact after the fused RoPE + append; outputs within
1e-3 + 2e-3 |ref|.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 2e-3
THETA = 1e6


def close(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    err = np.abs(a - b) - (ATOL + RTOL * np.abs(b))
    assert err.max() <= 0, f"max excess {err.max():.3e}, max abs diff {np.abs(a - b).max():.3e}"


def dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def oracle_prefill(port, q_raw, k_raw, v_raw, h, hkv, hd, positions=None, q_offset=0):
    """q_raw [S][h][hd], k_raw/v_raw [T][hkv][hd] with T = q_offset + S (pre-RoPE).
    Returns (out [S][h][hd] or rows at `positions`, k_bits, v_bits)."""
    kb, vb = port.append_rope_f16(k_raw, v_raw, 0, hkv, hd, THETA)
    k = port.f16_bits_to_f32(kb).ravel()
    v = port.f16_bits_to_f32(vb).ravel()
    s = q_raw.shape[0]
    rows = range(s) if positions is None else positions
    out = {}
    for t in rows:
        q = q_raw[t].astype(np.float32).copy().ravel()
        pos = q_offset + t
        port.rope_f32(q, h, hd, pos, THETA)
        out[t] = port.attention_decode_f32(q, k, v, pos, h, hkv, hd).reshape(h, hd)
    return out, kb, vb


@pytest.mark.parametrize("shape", [(16, 2, 1), (16, 2, 37), (16, 2, 128), (16, 2, 129), (28, 4, 300),
                                   (8, 8, 200), (16, 1, 257)])
def test_prefill_small(port, shape):
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, AttnEngine
    h, hkv, s = shape
    hd = 128
    rng = np.random.default_rng(s * 31 + h)
    q = rng.standard_normal((s, h, hd)).astype(np.float32)
    k = rng.standard_normal((s, hkv, hd)).astype(np.float32)
    v = rng.standard_normal((s, hkv, hd)).astype(np.float32)
    exp, kb, vb = oracle_prefill(port, q, k, v, h, hkv, hd)
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=2, max_seqs=2, max_tokens_per_seq=s + 5, kv_heads=hkv, head_dim=hd)
    out = torch.zeros((1, s, h, hd), dtype=torch.float32, device="cuda")
    cache.prefill(1, 1, 1, dev(q[None]), dev(k[None]), dev(v[None]), s, h, out, TE_ATTN_ADVANCE)
    eng.synchronize()
    assert cache.length(1) == s
    got = out.cpu().numpy()[0]
    for t in range(s):
        close(got[t], exp[t])
    kg, vg = cache.read_f16(1, 1, 0, s)
    assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    cache.close()
    eng.close()


def test_prefill_f16_inputs_multi_layer(port):
    """Config-3 style: f16 Q/K/V inputs, several layers in one call."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, AttnEngine
    h, hkv, hd, s, L = 16, 2, 128, 200, 3
    rng = np.random.default_rng(3)
    q16 = rng.standard_normal((L, s, h, hd)).astype(np.float16)
    k16 = rng.standard_normal((L, s, hkv, hd)).astype(np.float16)
    v16 = rng.standard_normal((L, s, hkv, hd)).astype(np.float16)
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
    out = torch.zeros((L, s, h, hd), dtype=torch.float32, device="cuda")
    cache.prefill(0, L, 0, dev(q16.view(np.uint16)).view(torch.float16), dev(k16.view(np.uint16)).view(torch.float16),
                  dev(v16.view(np.uint16)).view(torch.float16), s, h, out, TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16)
    eng.synchronize()
    got = out.cpu().numpy()
    for layer in range(L):
        exp, kb, vb = oracle_prefill(port, q16[layer].astype(np.float32), k16[layer].astype(np.float32),
                                     v16[layer].astype(np.float32), h, hkv, hd, positions=[0, 1, 63, 127, 128, 199])
        for t, e in exp.items():
            close(got[layer, t], e)
        kg, vg = cache.read_f16(layer, 0, 0, s)
        assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    cache.close()
    eng.close()


def test_prefill_f16_no_rope(port):
    """f16 inputs with RoPE off: the kernel reads the queries as they are (no rotation)."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, TE_ATTN_NO_ROPE, AttnEngine
    h, hkv, hd, s = 16, 2, 128, 300
    rng = np.random.default_rng(21)
    q16 = rng.standard_normal((1, s, h, hd)).astype(np.float16)
    k16 = rng.standard_normal((1, s, hkv, hd)).astype(np.float16)
    v16 = rng.standard_normal((1, s, hkv, hd)).astype(np.float16)
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
    out = torch.zeros((1, s, h, hd), dtype=torch.float32, device="cuda")
    t16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
    cache.prefill(0, 1, 0, t16(q16), t16(k16), t16(v16), s, h, out,
                  TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16 | TE_ATTN_NO_ROPE)
    eng.synchronize()
    got = out.cpu().numpy()[0]
    k = k16[0].astype(np.float32).ravel()
    v = v16[0].astype(np.float32).ravel()
    for t in (0, 1, 127, 128, 299):
        exp = port.attention_decode_f32(q16[0, t].astype(np.float32).ravel(), k, v, t, h, hkv, hd)
        close(got[t], exp.reshape(h, hd))
    kg, vg = cache.read_f16(0, 0, 0, s)
    assert np.array_equal(kg, k16[0].view(np.uint16)) and np.array_equal(vg, v16[0].view(np.uint16))
    cache.close()
    eng.close()


@pytest.mark.parametrize("split", [(100, 60), (128, 128), (70, 200)])
def test_chunked_prefill_then_decode(port, split):
    """Prefill in two calls (the second attends to the cached first part), then one decode step."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, AttnEngine
    h, hkv, hd = 16, 2, 128
    s1, s2 = split
    s = s1 + s2
    rng = np.random.default_rng(s1)
    q = rng.standard_normal((s + 1, h, hd)).astype(np.float32)
    k = rng.standard_normal((s + 1, hkv, hd)).astype(np.float32)
    v = rng.standard_normal((s + 1, hkv, hd)).astype(np.float32)
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=s + 1, kv_heads=hkv, head_dim=hd)
    out1 = torch.zeros((1, s1, h, hd), dtype=torch.float32, device="cuda")
    out2 = torch.zeros((1, s2, h, hd), dtype=torch.float32, device="cuda")
    cache.prefill(0, 1, 0, dev(q[None, :s1]), dev(k[None, :s1]), dev(v[None, :s1]), s1, h, out1, TE_ATTN_ADVANCE)
    cache.prefill(0, 1, 0, dev(q[None, s1:s]), dev(k[None, s1:s]), dev(v[None, s1:s]), s2, h, out2, TE_ATTN_ADVANCE)
    dout = torch.zeros((1, 1, h, hd), dtype=torch.float32, device="cuda")
    cache.decode(0, 1, [0], dev(q[None, s:s + 1]), dout, h, k_new=dev(k[None, s:s + 1]), v_new=dev(v[None, s:s + 1]),
                 flags=TE_ATTN_ADVANCE)
    eng.synchronize()
    exp, kb, vb = oracle_prefill(port, q, k, v, h, hkv, hd, positions=[0, s1 - 1, s1, s - 1, s])
    close(out1.cpu().numpy()[0, 0], exp[0])
    close(out1.cpu().numpy()[0, s1 - 1], exp[s1 - 1])
    close(out2.cpu().numpy()[0, 0], exp[s1])
    close(out2.cpu().numpy()[0, s2 - 1], exp[s - 1])
    close(dout.cpu().numpy()[0, 0], exp[s])
    kg, vg = cache.read_f16(0, 0, 0, s + 1)
    assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    cache.close()
    eng.close()


def test_prefill_config3_rows(port):
    """BASELINE config 3 shape for one layer (S=2048, H16/Hkv2/hd128, f16 inputs); rows across tiles checked."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, AttnEngine
    h, hkv, hd, s = 16, 2, 128, 2048
    rng = np.random.default_rng(2048)
    q16 = rng.standard_normal((s, h, hd)).astype(np.float16)
    k16 = rng.standard_normal((s, hkv, hd)).astype(np.float16)
    v16 = rng.standard_normal((s, hkv, hd)).astype(np.float16)
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
    out = torch.zeros((1, s, h, hd), dtype=torch.float32, device="cuda")
    t16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
    cache.prefill(0, 1, 0, t16(q16[None]), t16(k16[None]), t16(v16[None]), s, h, out,
                  TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16)
    eng.synchronize()
    rows = [0, 1, 127, 128, 255, 640, 1023, 1024, 1500, 1919, 2046, 2047]
    exp, kb, vb = oracle_prefill(port, q16.astype(np.float32), k16.astype(np.float32), v16.astype(np.float32),
                                 h, hkv, hd, positions=rows)
    got = out.cpu().numpy()[0]
    for t in rows:
        close(got[t], exp[t])
    assert np.isfinite(got).all()
    kg, vg = cache.read_f16(0, 0, 0, s)
    assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    cache.close()
    eng.close()


def test_prefill_host_buffers(port):
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_HOST_BUFFERS, AttnEngine
    h, hkv, hd, s = 16, 2, 128, 150
    rng = np.random.default_rng(12)
    q = rng.standard_normal((1, s, h, hd)).astype(np.float32)
    k = rng.standard_normal((1, s, hkv, hd)).astype(np.float32)
    v = rng.standard_normal((1, s, hkv, hd)).astype(np.float32)
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
    out = np.zeros((1, s, h, hd), np.float32)
    cache.prefill(0, 1, 0, q, k, v, s, h, out, TE_ATTN_ADVANCE | TE_ATTN_HOST_BUFFERS)
    exp, _, _ = oracle_prefill(port, q[0], k[0], v[0], h, hkv, hd, positions=[0, 77, 149])
    for t, e in exp.items():
        close(out[0, t], e)
    cache.close()
    eng.close()


@pytest.mark.parametrize("shape", [(16, 2), (28, 4)])
def test_prefill_growing_scores(port, shape):
    """Keys grow with position (16x over 600 tokens), so a row's running max
    rises by far more than 2^8 between key tiles and the accumulated O is
    rescaled many times (paired and single-head items).  f16 inputs with RoPE
    off: the kernel multiplies exactly the oracle's query values, which keeps
    this check on the online softmax.  (With a rotated fp32 query, its f16
    rounding alone moves attention weights at these score magnitudes by a few
    tenths of a percent, beyond the output tolerance.)"""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, TE_ATTN_NO_ROPE, AttnEngine
    h, hkv = shape
    hd, s = 128, 600
    rng = np.random.default_rng(77 + h)
    q16 = rng.standard_normal((s, h, hd)).astype(np.float16)
    k16 = (rng.standard_normal((s, hkv, hd)) * (1.0 + np.arange(s) / 40.0)[:, None, None]).astype(np.float16)
    v16 = rng.standard_normal((s, hkv, hd)).astype(np.float16)
    eng = AttnEngine(0)
    try:
        cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
        out = torch.zeros((1, s, h, hd), dtype=torch.float32, device="cuda")
        t16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
        cache.prefill(0, 1, 0, t16(q16[None]), t16(k16[None]), t16(v16[None]), s, h, out,
                      TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16 | TE_ATTN_NO_ROPE)
        eng.synchronize()
        got = out.cpu().numpy()[0]
        k = k16.astype(np.float32).ravel()
        v = v16.astype(np.float32).ravel()
        for t in (0, 1, 63, 64, 127, 128, 129, 255, 256, 383, 384, 511, 512, 599):
            exp = port.attention_decode_f32(q16[t].astype(np.float32).ravel(), k, v, t, h, hkv, hd)
            close(got[t], exp.reshape(h, hd))
        kg, vg = cache.read_f16(0, 0, 0, s)
        assert np.array_equal(kg, k16.view(np.uint16)) and np.array_equal(vg, v16.view(np.uint16))
    finally:
        eng.close()


@pytest.mark.parametrize("s", [1, 37, 128, 513])
@pytest.mark.parametrize("f16_inputs", [False, True])
def test_prefill_head_dim_64(port, s, f16_inputs):
    """head_dim 64 at the Qwen2.5-0.5B shape (H14/Hkv2, the model of BASELINE
    config 1 and of the reference's only MMA prefill,
    c/src/metal/metal_kernels.metal.inc:2693-2836): fp32 inputs (query as hi +
    lo f16 parts, one head per item) and f16 inputs (single rounding, head
    pairs); cache bit-exact, every row against the oracle."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, AttnEngine
    h, hkv, hd = 14, 2, 64
    rng = np.random.default_rng(640 + s)
    q = rng.standard_normal((s, h, hd)).astype(np.float32)
    k = rng.standard_normal((s, hkv, hd)).astype(np.float32)
    v = rng.standard_normal((s, hkv, hd)).astype(np.float32)
    flags = TE_ATTN_ADVANCE
    if f16_inputs:
        q, k, v = (a.astype(np.float16) for a in (q, k, v))
        flags |= TE_ATTN_INPUT_F16
    exp, kb, vb = oracle_prefill(port, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), h, hkv, hd)
    eng = AttnEngine(0)
    try:
        cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
        out = torch.zeros((1, s, h, hd), dtype=torch.float32, device="cuda")
        if f16_inputs:
            t16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
            cache.prefill(0, 1, 0, t16(q[None]), t16(k[None]), t16(v[None]), s, h, out, flags)
        else:
            cache.prefill(0, 1, 0, dev(q[None]), dev(k[None]), dev(v[None]), s, h, out, flags)
        eng.synchronize()
        got = out.cpu().numpy()[0]
        for t in range(s):
            close(got[t], exp[t])
        kg, vg = cache.read_f16(0, 0, 0, s)
        assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    finally:
        eng.close()


@pytest.mark.parametrize("shape", [(16, 2, 128), (28, 4, 128), (14, 2, 64)])
@pytest.mark.parametrize("mode", ["fp32", "f16_exact_q"])
def test_prefill_growing_scores_rotated_query(port, shape, mode):
    """Rotated queries against keys that grow 16x over 600 tokens (|q.k| /
    sqrt(hd) of tens): a query rounded once to f16 moves the weights beyond
    the bar here.  fp32 inputs, and f16 inputs with TE_ATTN_EXACT_Q, feed the
    rotated query as f16 hi + lo parts into the same accumulator and must meet
    1e-3 + 2e-3 |ref| on every checked row, with many O rescales per row."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_EXACT_Q, TE_ATTN_INPUT_F16, AttnEngine
    h, hkv, hd = shape
    s = 600
    rng = np.random.default_rng(177 + h + hd)
    q = rng.standard_normal((s, h, hd)).astype(np.float32)
    k = (rng.standard_normal((s, hkv, hd)) * (1.0 + np.arange(s) / 40.0)[:, None, None]).astype(np.float32)
    v = rng.standard_normal((s, hkv, hd)).astype(np.float32)
    flags = TE_ATTN_ADVANCE
    if mode == "f16_exact_q":
        q, k, v = (a.astype(np.float16) for a in (q, k, v))
        flags |= TE_ATTN_INPUT_F16 | TE_ATTN_EXACT_Q
    rows = (0, 1, 63, 64, 127, 128, 129, 255, 256, 383, 384, 511, 512, 599)
    exp, kb, vb = oracle_prefill(port, q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), h, hkv, hd,
                                 positions=rows)
    eng = AttnEngine(0)
    try:
        cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
        out = torch.zeros((1, s, h, hd), dtype=torch.float32, device="cuda")
        if mode == "f16_exact_q":
            t16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
            cache.prefill(0, 1, 0, t16(q[None]), t16(k[None]), t16(v[None]), s, h, out, flags)
        else:
            cache.prefill(0, 1, 0, dev(q[None]), dev(k[None]), dev(v[None]), s, h, out, flags)
        eng.synchronize()
        got = out.cpu().numpy()[0]
        for t in rows:
            close(got[t], exp[t])
        kg, vg = cache.read_f16(0, 0, 0, s)
        assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    finally:
        eng.close()
