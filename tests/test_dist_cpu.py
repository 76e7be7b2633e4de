"""Multi-GPU host logic on CPU: the sequence-sharding planner, the KV-split
ranges, and the KV-split decode protocol (partial records, all-gather, LSE
merge) run as world-size-2 gloo ranks with the CPU oracle standing in for the
per-rank GPU compute."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tinymetalagent_b200.dist import KVSplitDecoder, ShardSpec, kv_split_ranges, merge_partials_numpy, shard_sequences


def test_shard_sequences_balanced_and_complete():
    rng = np.random.default_rng(0)
    lengths = rng.integers(256, 8193, size=64)
    for world in (1, 2, 4, 8):
        shards = shard_sequences(lengths, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(64))
        loads = [int(sum(lengths[i] for i in s)) for s in shards]
        assert max(loads) - min(loads) <= int(lengths.max())
        assert shards == shard_sequences(lengths, world)


def test_kv_split_ranges_cover_contiguously():
    for n, w in [(32768, 1), (32768, 2), (32768, 8), (10, 3), (7, 7)]:
        r = kv_split_ranges(n, w)
        assert r[0][0] == 0 and r[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        assert max(e - b for b, e in r) - min(e - b for b, e in r) <= 1
        assert (r[-1][1] - r[-1][0]) == min(e - b for b, e in r)
    with pytest.raises(ValueError):
        kv_split_ranges(3, 4)


H, HKV, HD, N, STEPS, THETA = 8, 2, 64, 301, 3, 1e6


def _data():
    rng = np.random.default_rng(42)
    k = rng.standard_normal((N + STEPS, HKV, HD)).astype(np.float32)
    v = rng.standard_normal((N + STEPS, HKV, HD)).astype(np.float32)
    q = rng.standard_normal((STEPS, H, HD)).astype(np.float32)
    return k, v, q


def _worker(rank, world, port_no, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port_no)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as O
        port = O.port()
        kraw, vraw, qraw = _data()
        spec = ShardSpec.plan(rank, world, N)
        kb, vb = port.append_rope_f16(kraw[spec.begin:spec.end], vraw[spec.begin:spec.end], spec.begin, HKV, HD, THETA)
        local = {"k": port.f16_bits_to_f32(kb), "v": port.f16_bits_to_f32(vb)}

        def partial_fn(q, k_new, v_new, q_pos):
            if spec.is_tail:
                nk, nv = port.append_rope_f16(k_new.numpy()[0, 0][None], v_new.numpy()[0, 0][None], q_pos, HKV, HD, THETA)
                local["k"] = np.concatenate([local["k"], port.f16_bits_to_f32(nk)])
                local["v"] = np.concatenate([local["v"], port.f16_bits_to_f32(nv)])
            qr = q.numpy()[0, 0].copy().ravel()
            port.rope_f32(qr, H, HD, q_pos, THETA)
            n_local = local["k"].shape[0]
            return torch.from_numpy(port.decode_partial_f32(qr, local["k"].ravel(), local["v"].ravel(), 0, n_local,
                                                            H, HKV, HD))

        dec = KVSplitDecoder(spec, 1, H, HD, partial_fn=partial_fn,
                             merge_fn=lambda g: torch.from_numpy(merge_partials_numpy(g.numpy())), device="cpu")
        worst = 0.0
        for s in range(STEPS):
            out = dec.step(torch.from_numpy(qraw[s][None, None]), torch.from_numpy(kraw[N + s][None, None]),
                           torch.from_numpy(vraw[N + s][None, None])).numpy()
            # full-sequence oracle over positions 0..N+s
            kb_all, vb_all = port.append_rope_f16(kraw[:N + s + 1], vraw[:N + s + 1], 0, HKV, HD, THETA)
            qr = qraw[s].copy().ravel()
            port.rope_f32(qr, H, HD, N + s, THETA)
            exp = port.attention_decode_f32(qr, port.f16_bits_to_f32(kb_all).ravel(),
                                            port.f16_bits_to_f32(vb_all).ravel(), N + s, H, HKV, HD)
            worst = max(worst, float(np.max(np.abs(out.ravel() - exp) - (1e-5 + 1e-4 * np.abs(exp)))))
        results.put((rank, worst))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 3])
def test_kv_split_protocol_gloo(world):
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, _free_port() if False else 29611 + world, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    assert codes == [0] * world, codes
    got = sorted(results.get(timeout=5) for _ in range(world))
    assert [r for r, _ in got] == list(range(world))
    assert all(w <= 0 for _, w in got), got


def _fault_worker(rank, world, port_no, store_port, use_store, results):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port_no)
    os.environ["TE_FAULT_INJECT"] = "rank:1:step:1"
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
    outcome = (rank, "no error", -1, -1)
    try:
        from tinymetalagent_b200 import TinyEngineError
        store = dist.TCPStore("127.0.0.1", store_port, world, rank == 0, timeout=timedelta(seconds=20)) \
            if use_store else None
        spec = ShardSpec.plan(rank, world, N)
        rows = H

        def partial_fn(q, k_new, v_new, q_pos):  # a well-formed record: m = 0, l = 1, acc = rank
            rec = torch.zeros((rows, HD + 2))
            rec[:, :HD] = float(rank)
            rec[:, HD + 1] = 1.0
            return rec

        dec = KVSplitDecoder(spec, 1, H, HD, partial_fn=partial_fn,
                             merge_fn=lambda g: torch.from_numpy(merge_partials_numpy(g.numpy())), device="cpu",
                             store=store)
        q = torch.zeros((1, 1, H, HD))
        kv = torch.zeros((1, 1, HKV, HD))
        import time
        for s in range(3):
            t0 = time.monotonic()
            try:
                out = dec.step(q, kv, kv)
            except TinyEngineError as e:
                outcome = (rank, str(e), s, e.status, time.monotonic() - t0)
                break
            assert np.allclose(out.numpy(), (world - 1) / 2.0)  # the mean of the ranks' records
    finally:
        results.put(outcome)
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("use_store", [False, True])
def test_kv_split_rank_failure_ends_every_rank_with_an_error(use_store):
    """Host-side fault injection (TE_FAULT_INJECT=rank:1:step:1) on three gloo
    ranks: rank 1 fails its second step before any launch; the other ranks end
    that step with TinyEngineError / TE_STATUS_RUNTIME_ERROR -- from the shared
    store's fault record, or from the process group's 4 s timeout that ends
    their all-gather -- and no process hangs."""
    from tinymetalagent_b200.runtime import TE_STATUS_RUNTIME_ERROR
    world = 3
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    ports = (_free_port(), _free_port())
    procs = [ctx.Process(target=_fault_worker, args=(r, world, ports[0], ports[1], use_store, results))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=90)
    stuck = [p for p in procs if p.is_alive()]
    for p in stuck:  # our own children only
        p.kill()
    assert not stuck, "a rank hung"
    got = sorted(results.get(timeout=5) for _ in range(world))
    assert [g[0] for g in got] == list(range(world))
    for rank, msg, step, status, *_ in got:
        assert step == 1 and status == TE_STATUS_RUNTIME_ERROR, (rank, msg)
        if rank == 1:
            assert "injected fault" in msg
        else:
            assert "reported a failure" in msg or "all-gather" in msg, msg


def test_kv_split_polls_and_aborts_the_communicator():
    """With an NCCL group the decoder polls the communicator's asynchronous error
    before each step and aborts the communicator when a step fails.  A stand-in
    backend with ProcessGroupNCCL's get_error/abort interface checks the logic on
    the CPU: an error reported between steps ends the next step before any
    launch, with TE_STATUS_RUNTIME_ERROR, and the communicator is aborted."""
    from tinymetalagent_b200.runtime import TE_STATUS_RUNTIME_ERROR, TinyEngineError

    class FakeBackend:
        def __init__(self):
            self.error, self.aborted = "ErrorType.SUCCESS", False

        def get_error(self):
            return self.error

        def abort(self):
            self.aborted = True

    spec = ShardSpec.plan(0, 2, N)
    calls = []

    def partial_fn(q, k_new, v_new, q_pos):
        calls.append(q_pos)
        rec = torch.zeros((H, HD + 2))
        rec[:, HD + 1] = 1.0
        return rec

    dec = KVSplitDecoder(spec, 1, H, HD, partial_fn=partial_fn, merge_fn=lambda g: g[0, :, :HD], device="cpu")
    be = FakeBackend()
    dec._nccl_backend = lambda: be  # the stand-in for the group's NCCL backend
    dec.spec = ShardSpec(0, 1, spec.begin, spec.end, spec.global_len)  # one rank: no real collective
    q = torch.zeros((1, 1, H, HD))
    kv = torch.zeros((1, 1, HKV, HD))
    dec.step(q, kv, kv)
    assert calls == [N] and not be.aborted
    be.error = "ErrorType.REMOTE_ERROR"
    with pytest.raises(TinyEngineError) as err:
        dec.step(q, kv, kv)
    assert err.value.status == TE_STATUS_RUNTIME_ERROR and "REMOTE_ERROR" in str(err.value)
    assert be.aborted and calls == [N]  # no launch was made for the failed step
