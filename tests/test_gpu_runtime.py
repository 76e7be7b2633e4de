"""Runtime behaviour on the GPU: a cross-GPU wait that runs out becomes a
status, not a hang; the per-kernel device-time profile.

The reference reports a failed GPU step as TE_STATUS_RUNTIME_ERROR (the status
check of each Metal command buffer, c/src/metal/metal_backend_layers.mm.inc:
2318,2581) and profiles with TINYENGINE_PROFILE (c/src/qwen.c:47-73,
2216-2304).
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROWS, HD = 56, 128


def _silent_peer(handles, done):
    """Rank 1 of a two-rank exchange that exports its area and never pushes."""
    import torch
    from tinymetalagent_b200 import AttnEngine
    from tinymetalagent_b200.runtime import Exchange
    torch.cuda.set_device(0)
    eng = AttnEngine(0)
    ex = Exchange(eng, 2, 1, ROWS, HD)
    handles.put(ex.ipc_handle)
    done.wait(timeout=120)
    ex.close()
    eng.close()


def test_exchange_wait_runs_out_and_the_context_survives():
    """The NVLink exchange kernel waits (bounded) for the peers' pushes.  Here
    the peer -- another process, which never launches the exchange -- never
    pushes, so the kernel's wait on its arrival counter runs out after the
    engine's 300 ms limit: the kernel records the error and leaves, the next
    synchronisation raises TinyEngineError(TE_STATUS_RUNTIME_ERROR), and the
    same engine then runs a decode correctly.  Only one kernel waits, on a
    counter that nothing increments; nothing waits on it."""
    import torch
    import torch.multiprocessing as mp
    from tinymetalagent_b200 import TE_ATTN_NO_ROPE, AttnEngine, TinyEngineError
    from tinymetalagent_b200.runtime import TE_STATUS_RUNTIME_ERROR, Exchange
    ctx = mp.get_context("spawn")
    handles, done = ctx.Queue(), ctx.Event()
    peer = ctx.Process(target=_silent_peer, args=(handles, done))
    peer.start()
    eng = AttnEngine(0)
    try:
        eng.set_wait_limit(300)
        ex = Exchange(eng, 2, 0, ROWS, HD)
        ex.connect([ex.ipc_handle, handles.get(timeout=120)])
        partial = torch.zeros((ROWS, HD + 2), device="cuda")
        partial[:, HD + 1] = 1.0
        out = torch.zeros((ROWS, HD), device="cuda")
        t0 = time.monotonic()
        ex.merge(partial, out)
        with pytest.raises(TinyEngineError) as err:
            eng.synchronize()
        waited = time.monotonic() - t0
        assert err.value.status == TE_STATUS_RUNTIME_ERROR
        assert 0.25 <= waited < 10.0, waited
        ex.close()
        # the error was reported once and cleared; the context is usable
        eng.synchronize()
        rng = np.random.default_rng(4)
        k = rng.standard_normal((200, 2, HD)).astype(np.float16)
        v = rng.standard_normal((200, 2, HD)).astype(np.float16)
        q = torch.from_numpy(rng.standard_normal((16, HD)).astype(np.float32)).cuda()
        cache = eng.kv_cache(layers=1, max_seqs=1, max_tokens_per_seq=200, kv_heads=2, head_dim=HD)
        cache.write_f16(0, 0, 0, k.view(np.uint16), v.view(np.uint16))
        o = torch.zeros((16, HD), device="cuda")
        cache.decode(0, 1, [0], q, o, 16, flags=TE_ATTN_NO_ROPE)
        eng.synchronize()
        s = (q.cpu().numpy().reshape(2, 8, HD) @ k.astype(np.float32).transpose(1, 2, 0)) / np.sqrt(HD)
        p = np.exp(s - s.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        ref = (p @ v.astype(np.float32).transpose(1, 0, 2)).reshape(16, HD)
        assert np.abs(o.cpu().numpy() - ref).max() < 1e-3
        cache.close()
    finally:
        done.set()
        eng.close()
        peer.join(timeout=120)
        if peer.is_alive():
            peer.kill()
    assert peer.exitcode == 0


def test_profile_counts_and_times_each_launch():
    """te_attn_engine_profile brackets every launch with CUDA events; the
    report line has the reference's 'name=ms/calls' shape and counts the
    launches made (graph-captured launches are not timed)."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, TE_ATTN_NO_ROPE, AttnEngine
    eng = AttnEngine(0)
    try:
        eng.profile(True)
        cache = eng.kv_cache(layers=2, max_seqs=1, max_tokens_per_seq=600, kv_heads=2, head_dim=HD)
        kv = torch.randn((2, 500, 2, HD), device="cuda")
        cache.append_rope(0, 2, 0, kv, kv, 500, TE_ATTN_ADVANCE)
        q = torch.randn((2, 1, 16, HD), device="cuda")
        o = torch.zeros_like(q)
        for _ in range(3):
            cache.decode(0, 2, [0], q, o, 16, flags=TE_ATTN_NO_ROPE)
        line = eng.profile_report()
        fields = dict(f.split("=") for f in line.split(": ", 1)[1].split())
        assert line.startswith("tinyengine_profile: ")
        assert fields["decode"].endswith("/3") and fields["append"].endswith("/1"), line
        assert fields["merge"] == "0.000/0"
        ms_decode = float(fields["decode"].split("/")[0])
        assert 0.0 < ms_decode < 100.0
        assert abs(float(fields["device_ms"]) - sum(float(v.split("/")[0]) for k, v in fields.items()
                                                    if k != "device_ms")) < 0.01
        cache.close()
    finally:
        eng.close()


def test_second_device_after_the_first(port):
    """The kernels' dynamic shared-memory limits are raised once per device:
    a decode and a prefill on device 1 after device 0 in the same process both
    run and match the oracle (a once-per-process flag left device 1 at the
    default 48 KiB and every launch there failed)."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ADVANCE, AttnEngine
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    h, hkv, hd, n = 16, 2, 128, 300
    rng = np.random.default_rng(12)
    k = rng.standard_normal((n, hkv, hd)).astype(np.float32)
    v = rng.standard_normal((n, hkv, hd)).astype(np.float32)
    q = rng.standard_normal((n, h, hd)).astype(np.float32)
    kb, vb = port.append_rope_f16(k, v, 0, hkv, hd, 1e6)
    kf = port.f16_bits_to_f32(kb).ravel()
    vf = port.f16_bits_to_f32(vb).ravel()
    for dev in (0, 1):
        eng = AttnEngine(dev)
        try:
            cache = eng.kv_cache(layers=1, max_seqs=2, max_tokens_per_seq=n, kv_heads=hkv, head_dim=hd)
            td = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(f"cuda:{dev}")  # noqa: E731
            out = torch.zeros((1, n, h, hd), device=f"cuda:{dev}")
            cache.prefill(0, 1, 0, td(q[None]), td(k[None]), td(v[None]), n, h, out, TE_ATTN_ADVANCE)
            cache.append_rope(0, 1, 1, td(k[:-1]), td(v[:-1]), n - 1, TE_ATTN_ADVANCE)
            dout = torch.zeros((h, hd), device=f"cuda:{dev}")
            cache.decode(0, 1, [1], td(q[-1]), dout, h, k_new=td(k[-1:]), v_new=td(v[-1:]), flags=TE_ATTN_ADVANCE)
            eng.synchronize()
            qr = q[-1].copy().ravel()
            port.rope_f32(qr, h, hd, n - 1, 1e6)
            exp = port.attention_decode_f32(qr, kf, vf, n - 1, h, hkv, hd).reshape(h, hd)
            for got in (out.cpu().numpy()[0, -1], dout.cpu().numpy()):
                err = np.abs(got - exp) - (1e-3 + 2e-3 * np.abs(exp))
                assert err.max() <= 0, (dev, float(np.abs(got - exp).max()))
            cache.close()
        finally:
            eng.close()
