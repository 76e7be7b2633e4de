"""GPU parity of the fused projection-bias prologue (TE_ATTN_QKV_BIAS).

The reference adds the q/k/v biases with te_add_f32 (c/src/ops.c:408-416:
one fp32 addition per element) before RoPE and the cache append
(c/src/qwen.c:998-1011 decode, :771-783 prefill); the oracle here is that
fp32 addition (numpy float32, round to nearest) followed by the oracle's RoPE,
f16 append and attention.  Bars as elsewhere: cache bit-exact, outputs within
1e-3 + 2e-3 |ref|.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

THETA = 1e6


def close(a, b, atol=1e-3, rtol=2e-3):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    err = np.abs(a - b) - (atol + rtol * np.abs(b))
    assert err.max() <= 0, f"max excess {err.max():.3e}, max abs diff {np.abs(a - b).max():.3e}"


def dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def biases(rng, layers, h, hkv, hd):
    qb = (rng.standard_normal((layers, h * hd)) * 0.5).astype(np.float32)
    kb = (rng.standard_normal((layers, hkv * hd)) * 0.5).astype(np.float32)
    vb = (rng.standard_normal((layers, hkv * hd)) * 0.5).astype(np.float32)
    return qb, kb, vb


@pytest.mark.parametrize("f16", [False, True])
def test_append_with_bias_bit_exact(port, f16):
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, TE_ATTN_QKV_BIAS, AttnEngine
    rng = np.random.default_rng(31 + f16)
    L, h, hkv, hd, n = 3, 16, 2, 128, 200
    qb, kb, vb = biases(rng, L, h, hkv, hd)
    k = rng.standard_normal((2, n, hkv, hd)).astype(np.float16 if f16 else np.float32)
    v = rng.standard_normal((2, n, hkv, hd)).astype(np.float16 if f16 else np.float32)
    eng = AttnEngine(0)
    try:
        cache = eng.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=256, kv_heads=hkv, head_dim=hd)
        cache.set_qkv_bias(0, h, qb, kb, vb)
        flags = TE_ATTN_ADVANCE | TE_ATTN_QKV_BIAS | (TE_ATTN_INPUT_F16 if f16 else 0)
        to_dev = (lambda a: dev(a.view(np.uint16)).view(torch.float16)) if f16 else dev
        cache.append_rope(1, 2, 0, to_dev(k), to_dev(v), n, flags)  # cache layers 1 and 2
        eng.synchronize()
        for ll in range(2):
            layer = 1 + ll
            kf = k[ll].astype(np.float32) + kb[layer].reshape(hkv, hd)
            vf = v[ll].astype(np.float32) + vb[layer].reshape(hkv, hd)
            ek, ev = port.append_rope_f16(kf, vf, 0, hkv, hd, THETA)
            kg, vg = cache.read_f16(layer, 0, 0, n)
            assert np.array_equal(kg, ek) and np.array_equal(vg, ev)
    finally:
        eng.close()


@pytest.mark.parametrize("shape", [(16, 2, 128, 3000), (28, 4, 128, 700), (14, 2, 64, 513)])
@pytest.mark.parametrize("chunk", [0, 64])
def test_decode_step_with_bias(port, shape, chunk):
    """Two layers, one decode step that appends the new token: q, k_new and v_new
    get their layer's biases inside the decode launch (helper and appender warps)."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_QKV_BIAS, AttnEngine
    h, hkv, hd, n = shape
    L = 2
    rng = np.random.default_rng(h * 7 + n)
    qb, kb, vb = biases(rng, L, h, hkv, hd)
    kraw = rng.standard_normal((L, n, hkv, hd)).astype(np.float32)
    vraw = rng.standard_normal((L, n, hkv, hd)).astype(np.float32)
    qraw = rng.standard_normal((L, 1, h, hd)).astype(np.float32)
    eng = AttnEngine(0, decode_chunk_tokens=chunk)
    try:
        cache = eng.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=n + 8, kv_heads=hkv, head_dim=hd)
        cache.set_qkv_bias(0, h, qb, kb, vb)
        cache.append_rope(0, L, 0, dev(kraw[:, :-1]), dev(vraw[:, :-1]), n - 1, TE_ATTN_ADVANCE | TE_ATTN_QKV_BIAS)
        out = torch.zeros((L, 1, h, hd), dtype=torch.float32, device="cuda")
        cache.decode(0, L, [0], dev(qraw), out, h, k_new=dev(kraw[:, -1:]), v_new=dev(vraw[:, -1:]),
                     flags=TE_ATTN_ADVANCE | TE_ATTN_QKV_BIAS)
        eng.synchronize()
        got = out.cpu().numpy()
        for layer in range(L):
            kf = kraw[layer] + kb[layer].reshape(hkv, hd)
            vf = vraw[layer] + vb[layer].reshape(hkv, hd)
            ek, ev = port.append_rope_f16(kf, vf, 0, hkv, hd, THETA)
            q = (qraw[layer, 0] + qb[layer].reshape(h, hd)).astype(np.float32).ravel()
            port.rope_f32(q, h, hd, n - 1, THETA)
            exp = port.attention_decode_f32(q, port.f16_bits_to_f32(ek).ravel(), port.f16_bits_to_f32(ev).ravel(),
                                            n - 1, h, hkv, hd)
            close(got[layer, 0], exp.reshape(h, hd))
            kg, vg = cache.read_f16(layer, 0, 0, n)
            assert np.array_equal(kg, ek) and np.array_equal(vg, ev)
    finally:
        eng.close()


@pytest.mark.parametrize("mode", ["fp32_rope", "f16_no_rope"])
def test_prefill_with_bias(port, mode):
    """Prefill with biases: fp32 inputs with RoPE, and f16 inputs without RoPE
    (the queries then still take a preparation pass, for the bias)."""
    import torch
    from tinymetalagent_b200 import (TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, TE_ATTN_NO_ROPE, TE_ATTN_QKV_BIAS,
                                     AttnEngine)
    h, hkv, hd, s, L = 28, 4, 128, 300, 2
    rng = np.random.default_rng(57 + len(mode))
    qb, kb, vb = biases(rng, L, h, hkv, hd)
    f16 = mode == "f16_no_rope"
    dt = np.float16 if f16 else np.float32
    q = rng.standard_normal((L, s, h, hd)).astype(dt)
    k = rng.standard_normal((L, s, hkv, hd)).astype(dt)
    v = rng.standard_normal((L, s, hkv, hd)).astype(dt)
    eng = AttnEngine(0)
    try:
        cache = eng.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
        cache.set_qkv_bias(0, h, qb, kb, vb)
        out = torch.zeros((L, s, h, hd), dtype=torch.float32, device="cuda")
        flags = TE_ATTN_ADVANCE | TE_ATTN_QKV_BIAS
        if f16:
            flags |= TE_ATTN_INPUT_F16 | TE_ATTN_NO_ROPE
            t16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
            cache.prefill(0, L, 0, t16(q), t16(k), t16(v), s, h, out, flags)
        else:
            cache.prefill(0, L, 0, dev(q), dev(k), dev(v), s, h, out, flags)
        eng.synchronize()
        got = out.cpu().numpy()
        for layer in range(L):
            kf = k[layer].astype(np.float32) + kb[layer].reshape(hkv, hd)
            vf = v[layer].astype(np.float32) + vb[layer].reshape(hkv, hd)
            if f16:
                ek, ev = kf.astype(np.float16).view(np.uint16), vf.astype(np.float16).view(np.uint16)
            else:
                ek, ev = port.append_rope_f16(kf, vf, 0, hkv, hd, THETA)
            kk, vv = port.f16_bits_to_f32(ek).ravel(), port.f16_bits_to_f32(ev).ravel()
            for t in (0, 1, 127, 128, 299):
                qt = (q[layer, t].astype(np.float32) + qb[layer].reshape(h, hd)).astype(np.float32).ravel()
                if not f16:
                    port.rope_f32(qt, h, hd, t, THETA)
                exp = port.attention_decode_f32(qt, kk, vv, t, h, hkv, hd)
                close(got[layer, t], exp.reshape(h, hd))
            kg, vg = cache.read_f16(layer, 0, 0, s)
            assert np.array_equal(kg, ek) and np.array_equal(vg, ev)
    finally:
        eng.close()


def test_bias_flag_needs_biases(engine):
    import torch
    from tinymetalagent_b200 import TE_ATTN_QKV_BIAS, TinyEngineError
    cache = engine.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=64, kv_heads=2, head_dim=128)
    try:
        k = torch.zeros((1, 2, 128), dtype=torch.float32, device="cuda")
        with pytest.raises(TinyEngineError):
            cache.append_rope(0, 1, 0, k, k, 1, TE_ATTN_QKV_BIAS)
        cache.set_qkv_bias(0, 16, np.zeros((1, 16 * 128), np.float32), None, None)
        with pytest.raises(TinyEngineError):
            cache.set_qkv_bias(0, 8, np.zeros((1, 8 * 128), np.float32), None, None)  # heads fixed at 16
        q = torch.zeros((1, 1, 8, 128), dtype=torch.float32, device="cuda")
        out = torch.zeros_like(q)
        with pytest.raises(TinyEngineError):
            cache.decode(0, 1, [0], q, out, 8, k_new=k, v_new=k, flags=TE_ATTN_QKV_BIAS)  # heads differ
    finally:
        cache.close()
