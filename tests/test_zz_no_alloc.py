"""The allocation-free decode entry point against the engine's decode.

te_attention_decode_paged_noalloc serves callers that cannot allocate device
memory (a host framework that owns every allocation, a fixed-budget runtime):
it keeps its split-K scratch in a fixed file-scope device array instead of
engine memory.  Here it is called through the C ABI on a caller-built paged
cache and must agree with te_attention_decode on the same tokens, on two
consecutive calls (the second reuses the shared scratch left by the first).

The file name sorts last so that a run stopping at the first failure has
already run every other test.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-3, 2e-3


def _engine_decode(k, v, q, heads, kv_heads, head_dim):
    """Reference result from the existing entry point (engine-owned cache and scratch)."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_NO_ROPE, AttnEngine
    eng = AttnEngine(0)
    n = k.shape[0]
    cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=n, kv_heads=kv_heads, head_dim=head_dim)
    cache.write_f16(0, 0, 0, k, v)
    out = torch.zeros((heads, head_dim), dtype=torch.float32, device="cuda")
    cache.decode(0, 1, [0], q, out, heads, flags=TE_ATTN_NO_ROPE)
    eng.synchronize()
    res = out.cpu().numpy()
    cache.close()
    eng.close()
    return res


def test_noalloc_decode_matches_engine_decode_twice():
    import torch
    from tinymetalagent_b200 import runtime as R
    lib = R.load_library()
    heads, kv_heads, head_dim, page_tokens, num_pages = 16, 2, 128, 128, 48
    g = torch.Generator(device="cuda").manual_seed(77)
    # Caller-owned paged cache: pages in a shuffled order, as a real allocator would hand out.
    k_pool = torch.zeros((num_pages, kv_heads, page_tokens, head_dim), dtype=torch.float16, device="cuda")
    v_pool = torch.zeros_like(k_pool)
    order = torch.randperm(num_pages, generator=torch.Generator().manual_seed(5)).to(torch.int32)
    page_table = order.cuda()
    n_max = 40 * page_tokens
    k = torch.randn((n_max, kv_heads, head_dim), generator=g, device="cuda").half()
    v = torch.randn((n_max, kv_heads, head_dim), generator=g, device="cuda").half()
    for t0 in range(0, n_max, page_tokens):
        pg = int(order[t0 // page_tokens])
        k_pool[pg] = k[t0:t0 + page_tokens].transpose(0, 1)
        v_pool[pg] = v[t0:t0 + page_tokens].transpose(0, 1)
    stream = torch.cuda.current_stream()

    for call, n_tokens in enumerate([n_max - 77, 1000]):  # two calls in a row on the shared scratch
        q = torch.randn((heads, head_dim), generator=g, device="cuda")
        out = torch.full((heads, head_dim), float("nan"), dtype=torch.float32, device="cuda")
        st = lib.te_attention_decode_paged_noalloc(
            k_pool.data_ptr(), v_pool.data_ptr(), page_table.data_ptr(), num_pages, page_tokens, n_tokens,
            q.data_ptr(), heads, kv_heads, head_dim, out.data_ptr(), stream.cuda_stream)
        assert st == R.TE_STATUS_OK, lib.te_strerror(st)
        stream.synchronize()
        got = out.cpu().numpy()
        expect = _engine_decode(k[:n_tokens].contiguous(), v[:n_tokens].contiguous(), q, heads, kv_heads,
                                head_dim)
        assert np.isfinite(got).all(), call
        excess = np.abs(got - expect) - (ATOL + RTOL * np.abs(expect))
        assert excess.max() <= 0, (call, float(np.abs(got - expect).max()))


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("group", [7, 16])
@pytest.mark.parametrize("n_tokens", [1, 63, 65, 3001])
def test_noalloc_decode_matches_oracle(port, head_dim, group, n_tokens):
    """The allocation-free path against the CPU oracle (the reference's
    te_attention_decode_f32 over the same f16 K/V widened to fp32), so a fault
    shared with the engine's decode would show: head_dim 64/128, groups of 7
    (the padded-fragment layout) and 16 (two fragment sets), one partial stage
    up to a long multi-CTA split; the page table maps two of its entries to one
    page (tokens that repeat), as a caller may."""
    import torch
    from tinymetalagent_b200 import runtime as R
    lib = R.load_library()
    kv_heads, page_tokens = 2, 64
    heads = group * kv_heads
    n_pages_seq = (n_tokens + page_tokens - 1) // page_tokens
    num_pages = n_pages_seq + 3
    rng = np.random.default_rng(head_dim * 1000 + group * 10 + n_tokens)
    pool_k = rng.standard_normal((num_pages, kv_heads, page_tokens, head_dim), dtype=np.float32).astype(np.float16)
    pool_v = rng.standard_normal((num_pages, kv_heads, page_tokens, head_dim), dtype=np.float32).astype(np.float16)
    table = rng.permutation(num_pages)[:n_pages_seq].astype(np.int32)
    if n_pages_seq >= 3:
        table[-1] = table[0]  # a repeated page: its tokens appear twice in the sequence
    # the sequence as the oracle reads it: [n_tokens][kv_heads][head_dim]
    k_seq = pool_k[table].transpose(0, 2, 1, 3).reshape(-1, kv_heads, head_dim)[:n_tokens]
    v_seq = pool_v[table].transpose(0, 2, 1, 3).reshape(-1, kv_heads, head_dim)[:n_tokens]
    q = rng.standard_normal((heads, head_dim), dtype=np.float32)
    expect = port.attention_decode_f32(q.ravel(), k_seq.astype(np.float32).ravel(), v_seq.astype(np.float32).ravel(),
                                       n_tokens - 1, heads, kv_heads, head_dim).reshape(heads, head_dim)
    dk = torch.from_numpy(pool_k.view(np.uint16)).cuda()
    dv = torch.from_numpy(pool_v.view(np.uint16)).cuda()
    dt = torch.from_numpy(table).cuda()
    dq = torch.from_numpy(q).cuda()
    stream = torch.cuda.current_stream()
    for call in range(2):  # twice in a row on the shared scratch
        out = torch.full((heads, head_dim), float("nan"), dtype=torch.float32, device="cuda")
        st = lib.te_attention_decode_paged_noalloc(dk.data_ptr(), dv.data_ptr(), dt.data_ptr(), num_pages,
                                                   page_tokens, n_tokens, dq.data_ptr(), heads, kv_heads, head_dim,
                                                   out.data_ptr(), stream.cuda_stream)
        assert st == R.TE_STATUS_OK, lib.te_strerror(st)
        code = ctypes.c_int(-1)
        assert lib.te_attention_decode_paged_noalloc_status(stream.cuda_stream, ctypes.byref(code)) == R.TE_STATUS_OK
        assert code.value == 0
        got = out.cpu().numpy()
        excess = np.abs(got - expect) - (ATOL + RTOL * np.abs(expect))
        assert excess.max() <= 0, (call, float(np.abs(got - expect).max()))


def test_noalloc_rejects_out_of_range_shapes():
    from tinymetalagent_b200 import runtime as R
    lib = R.load_library()
    p = ctypes.c_void_p(16)  # never dereferenced: every case fails validation first
    f = lib.te_attention_decode_paged_noalloc
    assert f(p, p, p, 4, 128, 100, p, 16, 2, 96, p, None) == R.TE_STATUS_UNSUPPORTED      # head_dim
    assert f(p, p, p, 4, 128, 100, p, 34, 2, 128, p, None) == R.TE_STATUS_UNSUPPORTED     # group > 16
    assert f(p, p, p, 4, 128, 600, p, 16, 2, 128, p, None) == R.TE_STATUS_INVALID_ARGUMENT  # more tokens than pages
    assert f(p, p, p, 4, 100, 100, p, 16, 2, 128, p, None) == R.TE_STATUS_INVALID_ARGUMENT  # page size
    assert f(None, p, p, 4, 128, 100, p, 16, 2, 128, p, None) == R.TE_STATUS_INVALID_ARGUMENT
