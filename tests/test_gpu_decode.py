"""GPU parity of the decode path against the CPU oracle (reference ops.c semantics).

Bars: f16 cache contents bit-exact after RoPE + append; attention outputs
within |x - ref| <= 1e-3 + 2e-3 |ref| (f16 KV, fp32 accumulation), the
tolerance the engine is specified to.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 2e-3


def close(a, b, atol=ATOL, rtol=RTOL):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    err = np.abs(a - b) - (atol + rtol * np.abs(b))
    assert err.max() <= 0, f"max excess {err.max():.3e}, max abs diff {np.abs(a - b).max():.3e}"


def torch_dev(x, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


# ---------------------------------------------------------------- drop-ins

def test_rope_f32_dropin_bit_exact(golden, engine):
    from tinymetalagent_b200 import rope_f32
    i = 0
    while f"rope{i}_in" in golden:
        h, hd, pos = (int(x) for x in golden[f"rope{i}_shape"])
        x = golden[f"rope{i}_in"].copy()
        rope_f32(x, h, hd, pos, float(golden[f"rope{i}_theta"][0]))
        assert np.array_equal(x, golden[f"rope{i}_out"]), i
        i += 1


def test_rope_f32_dropin_kat(engine):
    from tinymetalagent_b200 import rope_f32
    import math
    v = np.array([1, 2, 3, 4], np.float32)
    rope_f32(v, 1, 4, 1, 10000.0)
    s0, c0, s1, c1 = math.sin(1.0), math.cos(1.0), math.sin(0.01), math.cos(0.01)
    np.testing.assert_allclose(v, [1 * c0 - 3 * s0, 2 * c1 - 4 * s1, 3 * c0 + 1 * s0, 4 * c1 + 2 * s1], atol=1e-6)


def test_attention_decode_f32_dropin(golden, engine):
    from tinymetalagent_b200 import attention_decode_f32
    i = 0
    while f"attn{i}_q" in golden:
        h, hkv, hd, n = (int(x) for x in golden[f"attn{i}_shape"])
        out = np.zeros(h * hd, np.float32)
        attention_decode_f32(golden[f"attn{i}_q"].ravel(), golden[f"attn{i}_k"].astype(np.float32).ravel(),
                             golden[f"attn{i}_v"].astype(np.float32).ravel(), n - 1, h, hkv, hd, out)
        close(out.reshape(h, hd), golden[f"attn{i}_out"], atol=1e-5, rtol=1e-4)
        i += 1
    # KAT of c/tests/kernel_ops.c:341-356
    out = np.zeros(4, np.float32)
    attention_decode_f32(np.array([1, 0, 0, 1], np.float32), np.array([1, 0, 0, 1], np.float32),
                         np.array([10, 20, 30, 40], np.float32), 1, 2, 1, 2, out)
    close(out, golden["kat_attn_out"], atol=1e-5, rtol=1e-5)


def test_attention_decode_f32_dropin_odd_shapes(port, engine):
    from tinymetalagent_b200 import attention_decode_f32
    rng = np.random.default_rng(11)
    for (h, hkv, hd, n) in [(3, 1, 5, 1), (6, 3, 10, 17), (2, 2, 300, 40), (8, 2, 64, 2100)]:
        q = rng.standard_normal(h * hd).astype(np.float32)
        k = rng.standard_normal(n * hkv * hd).astype(np.float32)
        v = rng.standard_normal(n * hkv * hd).astype(np.float32)
        out = np.zeros(h * hd, np.float32)
        attention_decode_f32(q, k, v, n - 1, h, hkv, hd, out)
        close(out, port.attention_decode_f32(q, k, v, n - 1, h, hkv, hd), atol=1e-5, rtol=1e-4)


# ---------------------------------------------------------------- append

@pytest.mark.parametrize("hd", [64, 128])
def test_append_rope_bit_exact(port, engine, golden, hd):
    rng = np.random.default_rng(hd)
    if hd == 64:
        n, hkv, _, p0 = (int(x) for x in golden["append_shape"])
        kraw = golden["append_kraw"]
        expect_k = golden["append_kbits"]
    else:
        n, hkv, p0 = 300, 2, 4000
        kraw = rng.standard_normal((n, hkv, hd)).astype(np.float32)
        expect_k, _ = port.append_rope_f16(kraw, kraw, p0, hkv, hd, 1e6)
    vraw = (rng.standard_normal((n, hkv, hd)) * 3).astype(np.float32)
    cache = engine.kv_cache(layers=2, max_seqs=3, max_tokens_per_seq=512, kv_heads=hkv, head_dim=hd,
                            max_position=p0 + 512)
    cache.reset(1, position_offset=p0)
    kd, vd = torch_dev(np.stack([kraw, kraw])), torch_dev(np.stack([vraw, vraw]))
    # two calls: 1 token then the rest, exercising the length bookkeeping
    from tinymetalagent_b200 import TE_ATTN_ADVANCE
    cache.append_rope(0, 2, 1, kd[:, :1].contiguous(), vd[:, :1].contiguous(), 1, TE_ATTN_ADVANCE)
    cache.append_rope(0, 2, 1, kd[:, 1:].contiguous(), vd[:, 1:].contiguous(), n - 1, TE_ATTN_ADVANCE)
    engine.synchronize()
    assert cache.length(1) == n
    for layer in (0, 1):
        kb, vb = cache.read_f16(layer, 1, 0, n)
        assert np.array_equal(kb, expect_k)
        assert np.array_equal(vb, vraw.astype(np.float16).view(np.uint16))
    cache.close()


def test_append_f16_input(port, engine):
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_INPUT_F16
    rng = np.random.default_rng(5)
    n, hkv, hd = 130, 2, 128
    k16 = rng.standard_normal((n, hkv, hd)).astype(np.float16)
    v16 = rng.standard_normal((n, hkv, hd)).astype(np.float16)
    cache = engine.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=256, kv_heads=hkv, head_dim=hd)
    import torch
    cache.append_rope(0, 1, 0, torch_dev(k16.view(np.uint16)).view(torch.float16),
                      torch_dev(v16.view(np.uint16)).view(torch.float16), n, TE_ATTN_ADVANCE | TE_ATTN_INPUT_F16)
    engine.synchronize()
    kb, vb = cache.read_f16(0, 0, 0, n)
    ek, _ = port.append_rope_f16(k16.astype(np.float32), k16.astype(np.float32), 0, hkv, hd, 1e6)
    assert np.array_equal(kb, ek)
    assert np.array_equal(vb, v16.view(np.uint16))
    cache.close()


# ---------------------------------------------------------------- decode

@pytest.mark.parametrize("chunk", [0, 64])
def test_decode_golden_vectors(golden, chunk):
    """Golden reference outputs with the cache filled from the same f16 values."""
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_NO_ROPE
    eng = AttnEngine(0, decode_chunk_tokens=chunk)
    i = 0
    while f"attn{i}_q" in golden:
        h, hkv, hd, n = (int(x) for x in golden[f"attn{i}_shape"])
        cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=n, kv_heads=hkv, head_dim=hd)
        cache.write_f16(0, 0, 0, golden[f"attn{i}_k"].view(np.uint16), golden[f"attn{i}_v"].view(np.uint16))
        q = torch_dev(golden[f"attn{i}_q"])
        import torch
        out = torch.zeros((h, hd), dtype=torch.float32, device="cuda")
        cache.decode(0, 1, [0], q, out, h, flags=TE_ATTN_NO_ROPE)
        eng.synchronize()
        close(out.cpu().numpy(), golden[f"attn{i}_out"])
        cache.close()
        i += 1
    eng.close()


def _oracle_decode(port, kraw_all, vraw_all, qraw, pos0, hkv, hd, h):
    """Oracle: RoPE+f16 append of every token, then RoPE(q) at the last position and attention."""
    n = kraw_all.shape[0]
    kb, vb = port.append_rope_f16(kraw_all, vraw_all, pos0, hkv, hd, 1e6)
    k = port.f16_bits_to_f32(kb)
    v = port.f16_bits_to_f32(vb)
    q = qraw.astype(np.float32).copy().ravel()
    port.rope_f32(q, h, hd, pos0 + n - 1, 1e6)
    return port.attention_decode_f32(q, k.ravel(), v.ravel(), n - 1, h, hkv, hd).reshape(h, hd), kb, vb


@pytest.mark.parametrize("shape", [(14, 2, 64, 513), (16, 2, 128, 4097), (28, 4, 128, 300), (8, 1, 128, 1),
                                   (16, 1, 128, 129), (4, 2, 64, 64)])
@pytest.mark.parametrize("chunk", [0, 64, 192])
def test_decode_append_rope_step(port, shape, chunk):
    """One decode step: RoPE+append of the new token fused into the attention launch."""
    import torch
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_ADVANCE
    h, hkv, hd, n = shape
    rng = np.random.default_rng(h * 1000 + n)
    kraw = rng.standard_normal((n, hkv, hd)).astype(np.float32)
    vraw = rng.standard_normal((n, hkv, hd)).astype(np.float32)
    qraw = rng.standard_normal((h, hd)).astype(np.float32)
    expect, kb, vb = _oracle_decode(port, kraw, vraw, qraw, 0, hkv, hd, h)
    eng = AttnEngine(0, decode_chunk_tokens=chunk)
    cache = eng.kv_cache(layers=1, max_seqs=2, max_tokens_per_seq=n + 64, kv_heads=hkv, head_dim=hd)
    if n > 1:
        cache.append_rope(0, 1, 1, torch_dev(kraw[:-1]), torch_dev(vraw[:-1]), n - 1, TE_ATTN_ADVANCE)
    out = torch.zeros((h, hd), dtype=torch.float32, device="cuda")
    cache.decode(0, 1, [1], torch_dev(qraw), out, h, k_new=torch_dev(kraw[-1:]), v_new=torch_dev(vraw[-1:]),
                 flags=TE_ATTN_ADVANCE)
    eng.synchronize()
    assert cache.length(1) == n
    close(out.cpu().numpy(), expect)
    kg, vg = cache.read_f16(0, 1, 0, n)
    assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    cache.close()
    eng.close()


@pytest.mark.parametrize("page_tokens", [64, 128])
def test_decode_interleaved_pages(port, page_tokens):
    """Sequences filled in alternating chunks own interleaved (non-consecutive)
    pages, so the kernel reads the page table; a third sequence filled in one
    go owns consecutive pages (page ids computed).  One fused append+decode step."""
    import torch
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_ADVANCE
    h, hkv, hd = 16, 2, 128
    lens = {0: 5 * page_tokens + 17, 1: 3 * page_tokens + 1, 2: 4 * page_tokens - 3}
    rng = np.random.default_rng(page_tokens)
    raw = {s: (rng.standard_normal((n, hkv, hd)).astype(np.float32),
               rng.standard_normal((n, hkv, hd)).astype(np.float32)) for s, n in lens.items()}
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=1, max_seqs=3, max_tokens_per_seq=8 * page_tokens, kv_heads=hkv, head_dim=hd,
                         page_tokens=page_tokens)
    filled = {0: 0, 1: 0}
    while any(filled[s] < lens[s] - 1 for s in (0, 1)):
        for s in (0, 1):  # one page at a time, alternating: interleaved page ids
            n = min(page_tokens, lens[s] - 1 - filled[s])
            if n > 0:
                k, v = raw[s]
                cache.append_rope(0, 1, s, torch_dev(k[filled[s]:filled[s] + n]), torch_dev(v[filled[s]:filled[s] + n]),
                                  n, TE_ATTN_ADVANCE)
                filled[s] += n
    k, v = raw[2]
    cache.append_rope(0, 1, 2, torch_dev(k[:-1]), torch_dev(v[:-1]), lens[2] - 1, TE_ATTN_ADVANCE)
    q = rng.standard_normal((1, 3, h, hd)).astype(np.float32)
    kn = np.stack([raw[s][0][-1] for s in (0, 1, 2)])[None]
    vn = np.stack([raw[s][1][-1] for s in (0, 1, 2)])[None]
    out = torch.zeros((1, 3, h, hd), dtype=torch.float32, device="cuda")
    cache.decode(0, 1, [0, 1, 2], torch_dev(q), out, h, k_new=torch_dev(kn), v_new=torch_dev(vn),
                 flags=TE_ATTN_ADVANCE)
    eng.synchronize()
    got = out.cpu().numpy()
    for i, s in enumerate((0, 1, 2)):
        expect, kb, vb = _oracle_decode(port, raw[s][0], raw[s][1], q[0, i], 0, hkv, hd, h)
        close(got[0, i], expect)
        kg, vg = cache.read_f16(0, s, 0, lens[s])
        assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    cache.close()
    eng.close()


def test_decode_ragged_multi_layer_multi_seq(port):
    """Ragged batch (several sequences, several layers) in one launch, small chunks."""
    import torch
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_ADVANCE, TE_ATTN_NO_ROPE
    h, hkv, hd, L = 28, 4, 128, 3
    lens = [1, 63, 64, 65, 127, 128, 129, 700, 1500]
    rng = np.random.default_rng(7)
    eng = AttnEngine(0, decode_chunk_tokens=128)
    cache = eng.kv_cache(layers=L, max_seqs=12, max_tokens_per_seq=2048, kv_heads=hkv, head_dim=hd)
    seq_ids = [3, 0, 11, 5, 1, 2, 7, 9, 4]
    ks, vs = {}, {}
    for sid, n in zip(seq_ids, lens):
        for layer in range(L):
            k = rng.standard_normal((n, hkv, hd)).astype(np.float16)
            v = rng.standard_normal((n, hkv, hd)).astype(np.float16)
            cache.write_f16(layer, sid, 0, k.view(np.uint16), v.view(np.uint16))
            ks[sid, layer], vs[sid, layer] = k, v
    q = rng.standard_normal((L, len(seq_ids), h, hd)).astype(np.float32)
    out = torch.zeros((L, len(seq_ids), h, hd), dtype=torch.float32, device="cuda")
    cache.decode(0, L, seq_ids, torch_dev(q), out, h, flags=TE_ATTN_NO_ROPE)
    eng.synchronize()
    got = out.cpu().numpy()
    for li in range(L):
        for si, (sid, n) in enumerate(zip(seq_ids, lens)):
            exp = port.attention_decode_f32(q[li, si].ravel(), ks[sid, li].astype(np.float32).ravel(),
                                            vs[sid, li].astype(np.float32).ravel(), n - 1, h, hkv, hd)
            close(got[li, si], exp.reshape(h, hd))
    # repeat: the split-K counters must have reset themselves
    out2 = torch.zeros_like(out)
    cache.decode(0, L, seq_ids, torch_dev(q), out2, h, flags=TE_ATTN_NO_ROPE)
    eng.synchronize()
    assert torch.equal(out, out2)
    cache.close()
    eng.close()


def test_decode_layer_subrange_and_many_seqs(port):
    """More sequences than one launch holds (64) and a layer sub-range."""
    import torch
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_NO_ROPE
    h, hkv, hd, L, S = 8, 2, 64, 4, 70
    rng = np.random.default_rng(8)
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=L, max_seqs=S, max_tokens_per_seq=200, kv_heads=hkv, head_dim=hd)
    lens = rng.integers(1, 200, size=S)
    data = {}
    for s in range(S):
        k = rng.standard_normal((lens[s], hkv, hd)).astype(np.float16)
        v = rng.standard_normal((lens[s], hkv, hd)).astype(np.float16)
        cache.write_f16(2, s, 0, k.view(np.uint16), v.view(np.uint16))
        data[s] = (k, v)
    q = rng.standard_normal((1, S, h, hd)).astype(np.float32)
    out = torch.zeros((1, S, h, hd), dtype=torch.float32, device="cuda")
    cache.decode(2, 1, list(range(S)), torch_dev(q), out, h, flags=TE_ATTN_NO_ROPE)
    eng.synchronize()
    got = out.cpu().numpy()
    for s in range(S):
        k, v = data[s]
        exp = port.attention_decode_f32(q[0, s].ravel(), k.astype(np.float32).ravel(), v.astype(np.float32).ravel(),
                                        int(lens[s]) - 1, h, hkv, hd)
        close(got[0, s], exp.reshape(h, hd))
    cache.close()
    eng.close()


def test_kv_split_partials_and_merge(port):
    """KV-sequence split: shards produce partial records; the LSE merge equals full attention."""
    import torch
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_ADVANCE, TE_ATTN_PARTIAL
    h, hkv, hd = 28, 4, 128
    n = 3000
    cuts = [0, 1000, 2100, n]
    rng = np.random.default_rng(9)
    kraw = rng.standard_normal((n, hkv, hd)).astype(np.float32)
    vraw = rng.standard_normal((n, hkv, hd)).astype(np.float32)
    qraw = rng.standard_normal((h, hd)).astype(np.float32)
    expect, _, _ = _oracle_decode(port, kraw, vraw, qraw, 0, hkv, hd, h)
    eng = AttnEngine(0)
    parts = torch.zeros((len(cuts) - 1, h, hd + 2), dtype=torch.float32, device="cuda")
    caches = []
    for gi, (a, b) in enumerate(zip(cuts[:-1], cuts[1:])):
        c = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=b - a, kv_heads=hkv, head_dim=hd,
                         max_position=n)
        c.reset(0, position_offset=a)
        last = b == n
        m = b - a - (1 if last else 0)
        c.append_rope(0, 1, 0, torch_dev(kraw[a:a + m]), torch_dev(vraw[a:a + m]), m, TE_ATTN_ADVANCE)
        if last:
            c.decode(0, 1, [0], torch_dev(qraw), parts[gi], h, k_new=torch_dev(kraw[-1:]),
                     v_new=torch_dev(vraw[-1:]), flags=TE_ATTN_PARTIAL | TE_ATTN_ADVANCE)
        else:
            c.decode(0, 1, [0], torch_dev(qraw), parts[gi], h, q_positions=[n - 1], flags=TE_ATTN_PARTIAL)
        caches.append(c)
    out = torch.zeros((h, hd), dtype=torch.float32, device="cuda")
    eng.merge_partials(parts, len(cuts) - 1, h, hd, out)
    eng.synchronize()
    close(out.cpu().numpy(), expect)
    # the partial records match the oracle's (m, l) bookkeeping after merging on the CPU too
    merged_cpu = port.merge_partials_f32(parts.cpu().numpy(), h, hd)
    close(merged_cpu, expect)
    for c in caches:
        c.close()
    eng.close()


@pytest.mark.parametrize("L", [2, 12])
@pytest.mark.parametrize("pinned", [False, True])
def test_decode_host_buffers(port, L, pinned):
    """The same step through host buffers (the e2e path): copies in, compute,
    output back, synchronous.  A pinned `out` is written by the kernel
    directly (no copy back), a pageable one through a copy; both must equal
    the device-pointer call's results bit for bit."""
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_ADVANCE, TE_ATTN_HOST_BUFFERS
    import torch
    h, hkv, hd, n = 16, 2, 128, 700
    rng = np.random.default_rng(10)
    kraw = rng.standard_normal((L, n, hkv, hd)).astype(np.float32)
    vraw = rng.standard_normal((L, n, hkv, hd)).astype(np.float32)
    qraw = rng.standard_normal((L, 1, h, hd)).astype(np.float32)
    eng = AttnEngine(0)
    cache = eng.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=n, kv_heads=hkv, head_dim=hd)
    cache.append_rope(0, L, 0, torch_dev(kraw[:, :-1]), torch_dev(vraw[:, :-1]), n - 1, TE_ATTN_ADVANCE)
    out = np.zeros((L, 1, h, hd), np.float32)
    kn = np.ascontiguousarray(kraw[:, -1:])
    vn = np.ascontiguousarray(vraw[:, -1:])
    if pinned:
        ins = [torch.from_numpy(a).pin_memory() for a in (qraw, kn, vn)]
        out_p = torch.zeros((L, 1, h, hd), dtype=torch.float32).pin_memory()
        cache.decode(0, L, [0], ins[0], out_p, h, k_new=ins[1], v_new=ins[2],
                     flags=TE_ATTN_ADVANCE | TE_ATTN_HOST_BUFFERS)
        out = out_p.numpy()
    else:
        cache.decode(0, L, [0], qraw, out, h, k_new=kn, v_new=vn, flags=TE_ATTN_ADVANCE | TE_ATTN_HOST_BUFFERS)
    assert cache.length(0) == n
    for layer in range(L):
        exp, kb, vb = _oracle_decode(port, kraw[layer], vraw[layer], qraw[layer, 0], 0, hkv, hd, h)
        close(out[layer, 0], exp)
        kg, vg = cache.read_f16(layer, 0, 0, n)
        assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    # the device-pointer call on the same state gives the same bits
    cache.truncate(0, n - 1)
    dout = torch.zeros((L, 1, h, hd), dtype=torch.float32, device="cuda")
    cache.decode(0, L, [0], torch_dev(qraw), dout, h, k_new=torch_dev(kn), v_new=torch_dev(vn), flags=TE_ATTN_ADVANCE)
    eng.synchronize()
    assert np.array_equal(dout.cpu().numpy(), out)
    cache.close()
    eng.close()


def test_decode_rejects_bad_arguments(engine):
    import torch
    from tinymetalagent_b200 import TinyEngineError
    cache = engine.kv_cache(layers=1, max_seqs=2, max_tokens_per_seq=64, kv_heads=2, head_dim=64)
    q = torch.zeros((1, 8, 64), device="cuda")
    out = torch.zeros_like(q)
    with pytest.raises(TinyEngineError):
        cache.decode(0, 1, [0], q, out, 8)          # empty sequence
    with pytest.raises(TinyEngineError):
        cache.decode(0, 1, [5], q, out, 8)          # bad sequence id
    with pytest.raises(TinyEngineError):
        cache.decode(0, 1, [0], q, out, 7)          # heads % kv_heads
    with pytest.raises(TinyEngineError):
        cache.decode(0, 2, [0], q, out, 8)          # layer range
    cache.close()


def test_decode_steps_in_cuda_graph_match_eager():
    """Decode steps captured in a CUDA graph (pages reserved first) give the eager results."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, AttnEngine
    h, hkv, hd, L, n0, steps = 16, 2, 128, 3, 1000, 4
    g = torch.Generator(device="cuda").manual_seed(3)
    k0 = [(torch.randn((n0, hkv, hd), generator=g, device="cuda") * 0.5).half() for _ in range(L)]
    v0 = [(torch.randn((n0, hkv, hd), generator=g, device="cuda") * 0.5).half() for _ in range(L)]
    qs = [torch.randn((L, 1, h, hd), generator=g, device="cuda") for _ in range(steps)]
    ks = [torch.randn((L, 1, hkv, hd), generator=g, device="cuda") for _ in range(steps)]
    vs = [torch.randn((L, 1, hkv, hd), generator=g, device="cuda") for _ in range(steps)]
    outs = {}
    for mode in ("eager", "graph"):
        eng = AttnEngine(0)
        st = torch.cuda.ExternalStream(eng.stream)
        cache = eng.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=n0 + steps, kv_heads=hkv, head_dim=hd)
        torch.cuda.synchronize()
        for layer in range(L):
            cache.write_f16(layer, 0, 0, k0[layer], v0[layer])
        cache.reserve(0, n0 + steps)
        out = [torch.zeros((L, 1, h, hd), device="cuda") for _ in range(steps)]

        def run():
            for i in range(steps):
                cache.decode(0, L, [0], qs[i], out[i], h, k_new=ks[i], v_new=vs[i], flags=TE_ATTN_ADVANCE)

        if mode == "eager":
            run()
        else:
            # warm the engine's scratch at the same shapes, then capture from the same start
            run()
            eng.synchronize()
            cache.truncate(0, n0)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=st):
                run()
            for o in out:
                o.zero_()
            torch.cuda.synchronize()
            with torch.cuda.stream(st):
                graph.replay()
            st.synchronize()
            del graph
        eng.synchronize()
        outs[mode] = [o.clone() for o in out]
        cache.close()
        eng.close()
    for a, b in zip(outs["eager"], outs["graph"]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("chunk", [0, 128])
def test_decode_growing_scores(port, chunk):
    """Cached keys grow with position (16x over 3000 tokens), so every split's
    running max rises by far more than 2^8 between stages and the accumulators
    are rescaled many times before the split-K combine (cluster and stream-K
    splits).  The queries are f16 values given as fp32 without RoPE, so the
    kernel multiplies exactly the oracle's query."""
    import torch
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_NO_ROPE
    h, hkv, hd, n = 16, 2, 128, 3000
    rng = np.random.default_rng(91)
    k = (rng.standard_normal((n, hkv, hd)) * (1.0 + np.arange(n) / 200.0)[:, None, None]).astype(np.float16)
    v = rng.standard_normal((n, hkv, hd)).astype(np.float16)
    q = rng.standard_normal((1, 1, h, hd)).astype(np.float16).astype(np.float32)
    eng = AttnEngine(0, decode_chunk_tokens=chunk)
    try:
        cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=n, kv_heads=hkv, head_dim=hd)
        cache.write_f16(0, 0, 0, k.view(np.uint16), v.view(np.uint16))
        out = torch.zeros((1, 1, h, hd), dtype=torch.float32, device="cuda")
        cache.decode(0, 1, [0], torch_dev(q), out, h, flags=TE_ATTN_NO_ROPE)
        eng.synchronize()
        exp = port.attention_decode_f32(q.ravel(), k.astype(np.float32).ravel(), v.astype(np.float32).ravel(),
                                        n - 1, h, hkv, hd)
        close(out.cpu().numpy()[0, 0], exp.reshape(h, hd))
    finally:
        eng.close()


@pytest.mark.parametrize("shape", [(16, 2, 128), (28, 4, 128), (16, 1, 128), (14, 2, 64), (16, 1, 64)])
@pytest.mark.parametrize("chunk", [0, 128])
def test_decode_growing_scores_fp32_rope(port, shape, chunk):
    """Rotated fp32 queries against keys that grow 16x over 3000 tokens, so
    |q.k| / sqrt(hd) reaches tens: a query rounded once to f16 moves the
    attention weights beyond the bar here.  The kernel feeds the tensor cores
    q = f16(q) + f16(q - f16(q)) (the low part in the padding rows of the
    group's fragments for groups <= 8, a second fragment set for groups of
    9-16), so the products keep the fp32 query.  RoPE on, the new token
    appended by the same launch, cluster and stream-K splits."""
    import torch
    from tinymetalagent_b200 import AttnEngine, TE_ATTN_ADVANCE
    h, hkv, hd = shape
    n = 3000
    rng = np.random.default_rng(93 + h + hd)
    ramp = (1.0 + np.arange(n) / 200.0)[:, None, None]
    kraw = (rng.standard_normal((n, hkv, hd)) * ramp).astype(np.float32)
    vraw = rng.standard_normal((n, hkv, hd)).astype(np.float32)
    qraw = rng.standard_normal((h, hd)).astype(np.float32)
    expect, kb, vb = _oracle_decode(port, kraw, vraw, qraw, 0, hkv, hd, h)
    eng = AttnEngine(0, decode_chunk_tokens=chunk)
    try:
        cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=n, kv_heads=hkv, head_dim=hd)
        cache.append_rope(0, 1, 0, torch_dev(kraw[:-1]), torch_dev(vraw[:-1]), n - 1, TE_ATTN_ADVANCE)
        out = torch.zeros((h, hd), dtype=torch.float32, device="cuda")
        cache.decode(0, 1, [0], torch_dev(qraw), out, h, k_new=torch_dev(kraw[-1:]), v_new=torch_dev(vraw[-1:]),
                     flags=TE_ATTN_ADVANCE)
        eng.synchronize()
        close(out.cpu().numpy(), expect)
        kg, vg = cache.read_f16(0, 0, 0, n)
        assert np.array_equal(kg, kb) and np.array_equal(vg, vb)
    finally:
        eng.close()
