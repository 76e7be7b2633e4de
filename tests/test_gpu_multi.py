"""KV-sequence split on two or four GPUs (BASELINE config 5's partitioning): each rank
holds a contiguous part of one sequence's cache, computes partial (acc, m, l) records, the
records are exchanged -- all-gathered over NCCL, or pushed into the peer's
memory over NVLink by the p2p exchange kernel -- and merged by log-sum-exp;
the tail rank appends the new token.  Checked against the CPU oracle over the whole
sequence (outputs within 1e-3 + 2e-3 |ref|; appended rows bit-exact).
Skipped on fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

L, H, HKV, HD, N, STEPS, THETA = 2, 16, 2, 128, 3000, 5, 1e6


def _data():
    rng = np.random.default_rng(2024)
    k = rng.standard_normal((L, N + STEPS, HKV, HD)).astype(np.float32)
    v = rng.standard_normal((L, N + STEPS, HKV, HD)).astype(np.float32)
    q = rng.standard_normal((STEPS, L, 1, H, HD)).astype(np.float32)
    return k, v, q


def _worker(rank, world, port_no, out_dir, exchange, graph=False):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port_no)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from tinymetalagent_b200 import TE_ATTN_ADVANCE, AttnEngine
        from tinymetalagent_b200.dist import KVSplitDecoder, ShardSpec
        kraw, vraw, qraw = _data()
        spec = ShardSpec.plan(rank, world, N)
        n_local = spec.end - spec.begin
        eng = AttnEngine(rank)
        cache = eng.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=n_local + STEPS + 4, kv_heads=HKV,
                             head_dim=HD, max_position=N + STEPS + 8, rope_theta=THETA)
        cache.reset(0, spec.begin)
        for layer in range(L):
            k = torch.from_numpy(np.ascontiguousarray(kraw[layer, spec.begin:spec.end])).cuda()
            v = torch.from_numpy(np.ascontiguousarray(vraw[layer, spec.begin:spec.end])).cuda()
            cache.append_rope(layer, 1, 0, k, v, n_local, TE_ATTN_ADVANCE if layer == L - 1 else 0)
        eng.synchronize()
        if spec.is_tail:
            cache.reserve(0, n_local + STEPS + 4)  # no page-table upload inside a graph capture
        dec = KVSplitDecoder(spec, L, H, HD, cache=cache, engine=eng, device="cuda", exchange=exchange)
        ins = [(torch.from_numpy(np.ascontiguousarray(qraw[s])).cuda(),
                torch.from_numpy(np.ascontiguousarray(kraw[:, N + s:N + s + 1])).cuda(),
                torch.from_numpy(np.ascontiguousarray(vraw[:, N + s:N + s + 1])).cuda()) for s in range(STEPS)]
        eager = 2 if graph else STEPS
        outs = []
        for s in range(eager):
            o = dec.step(*ins[s])
            eng.synchronize()
            outs.append(o.cpu().numpy().copy())
        if graph:
            # the remaining steps recorded as one CUDA graph on the engine's stream, then replayed once
            st = torch.cuda.ExternalStream(eng.stream)
            res = [torch.empty((L, 1, H, HD), device="cuda") for _ in range(STEPS - eager)]
            dist.barrier()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=st):
                for i in range(STEPS - eager):
                    res[i].copy_(dec.step(*ins[eager + i]))
            with torch.cuda.stream(st):
                g.replay()
            eng.synchronize()
            outs += [r.cpu().numpy() for r in res]
            del g
        np.save(os.path.join(out_dir, f"out{rank}.npy"), np.stack(outs))
        dist.barrier()  # every rank's last step is done before the exchange areas go away
        dec.close()
        if spec.is_tail:
            kg, vg = cache.read_f16(0, 0, n_local, STEPS)
            np.save(os.path.join(out_dir, "tail_k.npy"), kg)
            np.save(os.path.join(out_dir, "tail_v.npy"), vg)
        cache.close()
        eng.close()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("exchange", ["nccl", "p2p", "fused", "fused_graph"])
def test_kv_split_two_gpus_matches_oracle(port, tmp_path, exchange, world):
    """world ranks (2, or 4 where the box has them), each on its own GPU;
    exchange: NCCL all-gather + merge kernel, the NVLink push kernel, or the
    exchange fused into the decode launch (te_attention_decode_kv_split) --
    also with its last three steps recorded in a CUDA graph and replayed (the
    step count that picks the gather area's half lives on the device)."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    graph = exchange.endswith("_graph")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), exchange.replace("_graph", ""), graph),
                       nprocs=world, join=True, start_method="spawn")
    kraw, vraw, qraw = _data()
    outs = [np.load(tmp_path / f"out{r}.npy") for r in range(world)]
    for r in range(1, world):
        assert np.array_equal(outs[0], outs[r])  # every rank holds the same merged output
    for layer in range(L):
        kb, vb = port.append_rope_f16(kraw[layer], vraw[layer], 0, HKV, HD, THETA)
        kf = port.f16_bits_to_f32(kb)
        vf = port.f16_bits_to_f32(vb)
        for s in range(STEPS):
            n = N + s + 1
            q = qraw[s, layer, 0].copy().ravel()
            port.rope_f32(q, H, HD, n - 1, THETA)
            exp = port.attention_decode_f32(q, kf[:n].ravel(), vf[:n].ravel(), n - 1, H, HKV, HD).reshape(H, HD)
            got = outs[0][s, layer, 0]
            err = np.abs(got - exp) - (1e-3 + 2e-3 * np.abs(exp))
            assert err.max() <= 0, (layer, s, float(np.abs(got - exp).max()))
        if layer == 0:
            assert np.array_equal(np.load(tmp_path / "tail_k.npy"), kb[N:N + STEPS])
            assert np.array_equal(np.load(tmp_path / "tail_v.npy"), vb[N:N + STEPS])
