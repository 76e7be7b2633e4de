"""GPU parity at BASELINE.json's own workload shapes, against the CPU oracle
(the reference's te_rope_f32 / te_attention_decode_f32 semantics,
c/src/ops.c:295-395, and its causal prefill loop, c/src/qwen.c:810-824).

Bars as everywhere: the f16 cache bit-exact after RoPE + append; attention
outputs within 1e-3 + 2e-3 |ref|.
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


def oracle_decode(port, kraw, vraw, qraw, pos0, hkv, hd, h):
    """RoPE + f16 append of every token at positions pos0.., then RoPE(q) at the
    last position and the reference attention over all of them."""
    n = kraw.shape[0]
    kb, vb = port.append_rope_f16(kraw, vraw, pos0, hkv, hd, THETA)
    k = port.f16_bits_to_f32(kb)
    v = port.f16_bits_to_f32(vb)
    q = qraw.astype(np.float32).copy().ravel()
    port.rope_f32(q, h, hd, pos0 + n - 1, THETA)
    return port.attention_decode_f32(q, k.ravel(), v.ravel(), n - 1, h, hkv, hd).reshape(h, hd), kb, vb


def test_config4_ragged_64_sequences(port):
    """Config 4: Qwen2.5-7B shape (H28/Hkv4/hd128), 64 sequences with the
    bench's lengths (default_rng(7).integers(256, 8193)), fp32 N(0,1) inputs,
    RoPE on; one launch appends each sequence's newest token and attends all
    64 sequences."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, AttnEngine
    h, hkv, hd = 28, 4, 128
    lens = np.random.default_rng(7).integers(256, 8193, size=64)

    def raw(i):
        rng = np.random.default_rng(1000 + i)
        n = int(lens[i])
        return (rng.standard_normal((n, hkv, hd), dtype=np.float32), rng.standard_normal((n, hkv, hd), dtype=np.float32),
                rng.standard_normal((h, hd), dtype=np.float32))

    eng = AttnEngine(0)
    try:
        cache = eng.kv_cache(layers=1, max_seqs=64, max_tokens_per_seq=int(lens.max()), kv_heads=hkv, head_dim=hd)
        q = np.zeros((1, 64, h, hd), np.float32)
        kn = np.zeros((1, 64, hkv, hd), np.float32)
        vn = np.zeros((1, 64, hkv, hd), np.float32)
        for i in range(64):
            k, v, qi = raw(i)
            cache.append_rope(0, 1, i, dev(k[:-1]), dev(v[:-1]), int(lens[i]) - 1, TE_ATTN_ADVANCE)
            eng.synchronize()
            q[0, i], kn[0, i], vn[0, i] = qi, k[-1], v[-1]
        out = torch.zeros((1, 64, h, hd), dtype=torch.float32, device="cuda")
        cache.decode(0, 1, list(range(64)), dev(q), out, h, k_new=dev(kn), v_new=dev(vn), flags=TE_ATTN_ADVANCE)
        eng.synchronize()
        got = out.cpu().numpy()[0]
        for i in range(64):
            k, v, qi = raw(i)
            exp, kb, vb = oracle_decode(port, k, v, qi, 0, hkv, hd, h)
            close(got[i], exp)
            assert cache.length(i) == int(lens[i])
            kg, vg = cache.read_f16(0, i, 0, int(lens[i]))
            assert np.array_equal(kg, kb) and np.array_equal(vg, vb), i
        cache.close()
    finally:
        eng.close()


def test_config5_long_context_whole_and_four_way_split(port):
    """Config 5: one 32 769-token sequence (32 768 cached + the appended one),
    H28/Hkv4/hd128, RoPE theta 1e6, on one GPU -- as a whole, and as four
    KV-split shards (TE_ATTN_PARTIAL records, each shard's cache at its global
    position offset, the tail shard appending) merged by
    te_attention_merge_partials."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_PARTIAL, AttnEngine
    h, hkv, hd = 28, 4, 128
    n = 32769
    rng = np.random.default_rng(55)
    kraw = rng.standard_normal((n, hkv, hd), dtype=np.float32)
    vraw = rng.standard_normal((n, hkv, hd), dtype=np.float32)
    qraw = rng.standard_normal((h, hd), dtype=np.float32)
    expect, kb, vb = oracle_decode(port, kraw, vraw, qraw, 0, hkv, hd, h)
    eng = AttnEngine(0)
    try:
        # whole
        cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=n, kv_heads=hkv, head_dim=hd)
        cache.append_rope(0, 1, 0, dev(kraw[:-1]), dev(vraw[:-1]), n - 1, TE_ATTN_ADVANCE)
        out = torch.zeros((h, hd), dtype=torch.float32, device="cuda")
        cache.decode(0, 1, [0], dev(qraw), out, h, k_new=dev(kraw[-1:]), v_new=dev(vraw[-1:]), flags=TE_ATTN_ADVANCE)
        eng.synchronize()
        close(out.cpu().numpy(), expect)
        kg, vg = cache.read_f16(0, 0, 0, n)
        assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
        cache.close()
        # four KV-split shards on one GPU
        cuts = [0, 8192, 16384, 24576, n]
        parts = torch.zeros((4, h, hd + 2), dtype=torch.float32, device="cuda")
        shards = []
        for gi, (a, b) in enumerate(zip(cuts[:-1], cuts[1:])):
            c = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=b - a, kv_heads=hkv, head_dim=hd,
                             max_position=n)
            c.reset(0, position_offset=a)
            tail = b == n
            m = b - a - (1 if tail else 0)
            c.append_rope(0, 1, 0, dev(kraw[a:a + m]), dev(vraw[a:a + m]), m, TE_ATTN_ADVANCE)
            if tail:
                c.decode(0, 1, [0], dev(qraw), parts[gi], h, k_new=dev(kraw[-1:]), v_new=dev(vraw[-1:]),
                         flags=TE_ATTN_PARTIAL | TE_ATTN_ADVANCE)
            else:
                c.decode(0, 1, [0], dev(qraw), parts[gi], h, q_positions=[n - 1], flags=TE_ATTN_PARTIAL)
            eng.synchronize()
            kg, vg = c.read_f16(0, 0, 0, b - a)
            assert np.array_equal(kg, kb[a:b]) and np.array_equal(vg, vb[a:b]), gi
            shards.append(c)
        merged = torch.zeros((h, hd), dtype=torch.float32, device="cuda")
        eng.merge_partials(parts, 4, h, hd, merged)
        eng.synchronize()
        close(merged.cpu().numpy(), expect)
        for c in shards:
            c.close()
    finally:
        eng.close()


def test_config3_prefill_three_full_layers(port):
    """Config 3: the 2048-token causal prefill (H16/Hkv2/hd128, f16 Q/K/V
    N(0,1), RoPE theta 1e6 at positions 0..2047) on three whole layers in one
    call; every 16th row and the last 16 rows of every layer against the
    oracle's per-token loop, and every layer's cache bit-exact."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16, AttnEngine
    h, hkv, hd, s, L = 16, 2, 128, 2048, 3
    rng = np.random.default_rng(33)
    q16 = rng.standard_normal((L, s, h, hd), dtype=np.float32).astype(np.float16)
    k16 = rng.standard_normal((L, s, hkv, hd), dtype=np.float32).astype(np.float16)
    v16 = rng.standard_normal((L, s, hkv, hd), dtype=np.float32).astype(np.float16)
    eng = AttnEngine(0)
    try:
        cache = eng.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=s, kv_heads=hkv, head_dim=hd)
        t16 = lambda a: dev(a.view(np.uint16)).view(torch.float16)  # noqa: E731
        out = torch.zeros((L, s, h, hd), dtype=torch.float32, device="cuda")
        cache.prefill(0, L, 0, t16(q16), t16(k16), t16(v16), s, h, out, TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16)
        eng.synchronize()
        got = out.cpu().numpy()
        rows = sorted(set(range(0, s, 16)) | set(range(s - 16, s)))
        for layer in range(L):
            kb, vb = port.append_rope_f16(k16[layer].astype(np.float32), v16[layer].astype(np.float32), 0, hkv, hd,
                                          THETA)
            k = port.f16_bits_to_f32(kb).ravel()
            v = port.f16_bits_to_f32(vb).ravel()
            for t in rows:
                q = q16[layer, t].astype(np.float32).ravel().copy()
                port.rope_f32(q, h, hd, t, THETA)
                close(got[layer, t], port.attention_decode_f32(q, k, v, t, h, hkv, hd).reshape(h, hd))
            kg, vg = cache.read_f16(layer, 0, 0, s)
            assert np.array_equal(kg, kb) and np.array_equal(vg, vb), layer
        cache.close()
    finally:
        eng.close()
