"""Multi-GPU orchestration of the attention stage: one process per GPU.

Two partitionings, chosen where the work shards naturally (the reference runs
on a single device; there is no counterpart):

* Sequence sharding (batched decode of independent sequences): each rank owns
  whole sequences and runs ``te_attention_decode`` on them; no collective on
  the data path.  ``shard_sequences`` balances total cached tokens per rank.
* KV-sequence split (one long context): rank r owns a contiguous token range of
  the sequence; the last rank owns the tail and appends new tokens.  Each rank
  computes partial softmax records (acc, m, l) over its range with the query
  rotated at the global position; the records are all-gathered over NCCL and
  merged by ``te_attention_merge_partials`` (log-sum-exp).

The per-rank compute of ``KVSplitDecoder`` is the engine; tests replace it with
a CPU stand-in to check the partition/gather/merge protocol on gloo ranks.

Failures surface as ``TinyEngineError`` with TE_STATUS_RUNTIME_ERROR, the
reference's status for a failed GPU step (a Metal command buffer that did not
complete, c/src/metal/metal_backend_layers.mm.inc:2318,2581).  A rank that
fails records it in an optional host store before raising; the other ranks
check the store before each step's launches, and a rank already inside the
exchange ends it through the process group's timeout (NCCL, gloo) or the
engine's bounded wait (the NVLink exchange, ``AttnEngine.set_wait_limit``).
With NCCL, each step first polls the communicator's asynchronous error
(``ProcessGroupNCCL.get_error``, i.e. ncclCommGetAsyncError) and a failure
aborts the communicator (``abort``, i.e. ncclCommAbort) before raising.
``TE_FAULT_INJECT="rank:k"`` (or ``"rank:k:step:s"``) makes rank k fail its
step s (default 0) on the host, before any launch of that step, to test this.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import numpy as np

FAULT_KEY = "te_kv_split_fault"


def injected_fault(rank: int, step: int, spec: Optional[str] = None) -> bool:
    """True when TE_FAULT_INJECT (or `spec`) names this rank and step:
    "rank:k" fails step 0 of rank k, "rank:k:step:s" its step s."""
    spec = os.environ.get("TE_FAULT_INJECT", "") if spec is None else spec
    if not spec:
        return False
    parts = spec.split(":")
    if len(parts) not in (2, 4) or parts[0] != "rank" or (len(parts) == 4 and parts[2] != "step"):
        raise ValueError(f"TE_FAULT_INJECT must be 'rank:k' or 'rank:k:step:s', not {spec!r}")
    return int(parts[1]) == rank and (int(parts[3]) if len(parts) == 4 else 0) == step


def shard_sequences(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Greedy longest-first assignment of sequences to ranks, balancing the sum
    of lengths (the decode work is proportional to cached tokens).  Returns, per
    rank, the sequence indices in ascending order; deterministic for equal input."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    loads = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        out[r].append(i)
        loads[r] += int(lengths[i])
    return [sorted(x) for x in out]


def kv_split_ranges(n_tokens: int, world: int) -> list[tuple[int, int]]:
    """Contiguous [begin, end) token ranges per rank; the remainder goes to the
    first ranks so the tail rank (which grows by appends) is never the largest."""
    if n_tokens < world:
        raise ValueError("fewer tokens than ranks")
    base, rem = divmod(n_tokens, world)
    out, b = [], 0
    for r in range(world):
        e = b + base + (1 if r < rem else 0)
        out.append((b, e))
        b = e
    return out


@dataclass
class ShardSpec:
    rank: int
    world: int
    begin: int          # global position of this rank's first cached token
    end: int            # one past its last cached token (before appends)
    global_len: int     # tokens cached over all ranks (before appends)

    @property
    def is_tail(self) -> bool:
        return self.rank == self.world - 1

    @staticmethod
    def plan(rank: int, world: int, n_tokens: int) -> "ShardSpec":
        b, e = kv_split_ranges(n_tokens, world)[rank]
        return ShardSpec(rank, world, b, e, n_tokens)


class KVSplitDecoder:
    """Decode steps of one long sequence split over `world` ranks.

    cache      this rank's KVCache (one sequence slot), holding tokens [begin, end)
    group      torch.distributed process group (NCCL for GPUs)
    partial_fn optional stand-in for the engine: (q, k_new, v_new, q_position) -> partial
               records [n_layers][heads][head_dim + 2] as a torch tensor
    merge_fn   optional stand-in for te_attention_merge_partials: (gathered [world][rows][hd+2]) -> out
    exchange   "nccl": all-gather the records over the process group, then
               te_attention_merge_partials; "p2p": one kernel pushes them into
               the peers' memory over NVLink and merges what arrived
               (te_attn_exchange_*; needs one GPU per rank, world <= 8);
               "fused": the decode launch itself exchanges and merges
               (te_attention_decode_kv_split: each finished group's record is
               stored into every rank's memory over NVLink and every rank merges
               its own output at the end of its launch; one launch per step, no
               collective; one GPU per rank, world <= 8)
    store      optional torch.distributed Store shared by the ranks: a rank that
               fails writes FAULT_KEY there, and every rank checks it before
               each step's launches (one host round trip per step)
    """

    def __init__(self, spec: ShardSpec, n_layers: int, heads: int, head_dim: int, cache=None, engine=None,
                 group=None, partial_fn: Optional[Callable] = None, merge_fn: Optional[Callable] = None,
                 device=None, exchange: str = "nccl", store=None):
        self.spec = spec
        self.store = store
        self.steps_done = 0
        self.n_layers, self.heads, self.head_dim = n_layers, heads, head_dim
        self.cache, self.engine, self.group = cache, engine, group
        self.partial_fn = partial_fn
        self.merge_fn = merge_fn
        self.device = device
        self.length = spec.global_len  # global length of the sequence (all ranks agree)
        import torch
        rows = n_layers * heads
        self._part = torch.empty((rows, head_dim + 2), dtype=torch.float32, device=device)
        # concatenated along dim 0 (the form every backend's all_gather_into_tensor accepts)
        self._gather_flat = torch.empty((spec.world * rows, head_dim + 2), dtype=torch.float32, device=device)
        self._gather = self._gather_flat.view(spec.world, rows, head_dim + 2)
        self._out = torch.empty((n_layers, 1, heads, head_dim), dtype=torch.float32, device=device)
        # the engine's kernels and the collective run on one stream (the engine's)
        self._stream = torch.cuda.ExternalStream(engine.stream) if engine is not None else None
        self._exchange = None
        if exchange not in ("nccl", "p2p", "fused"):
            raise ValueError("exchange is 'nccl', 'p2p' or 'fused'")
        self.fused = exchange == "fused" and spec.world > 1
        if exchange in ("p2p", "fused") and spec.world > 1:
            self._exchange = self._connect_p2p(engine, group, rows, head_dim)
        if self.fused:
            self._out = self._exchange.output((n_layers, 1, heads, head_dim))

    def _connect_p2p(self, engine, group, rows: int, head_dim: int):
        import torch
        import torch.distributed as dist
        from .runtime import Exchange
        if engine is None or self.partial_fn is not None or self.merge_fn is not None:
            raise ValueError("the p2p exchange runs the engine's kernels")
        if torch.cuda.device_count() < self.spec.world:
            # the exchange kernel waits for the other ranks: never two ranks on one GPU
            raise RuntimeError("the p2p exchange needs one GPU per rank")
        ex = Exchange(engine, self.spec.world, self.spec.rank, rows, head_dim)
        handles = [None] * self.spec.world
        dist.all_gather_object(handles, ex.ipc_handle, group=group)
        ex.connect(handles)
        dist.barrier(group=group)  # every rank mapped before any rank pushes
        return ex

    def close(self) -> None:
        """Frees the p2p exchange; call on every rank after a barrier that follows the last step."""
        if self._exchange is not None:
            self._exchange.close()
            self._exchange = None

    def _local_partial(self, q, k_new, v_new, q_pos: int):
        from .runtime import TE_ATTN_ADVANCE, TE_ATTN_PARTIAL
        if self.partial_fn is not None:
            self._part.copy_(self.partial_fn(q, k_new, v_new, q_pos).reshape(self._part.shape))
            return
        if self.spec.is_tail:
            self.cache.decode(0, self.n_layers, [0], q, self._part, self.heads, k_new=k_new, v_new=v_new,
                              flags=TE_ATTN_PARTIAL | TE_ATTN_ADVANCE)
        else:
            self.cache.decode(0, self.n_layers, [0], q, self._part, self.heads, q_positions=[q_pos],
                              flags=TE_ATTN_PARTIAL)

    def _nccl_backend(self):
        """The NCCL backend of the exchange's process group, or None (gloo, CPU stand-ins, one rank)."""
        if self.spec.world <= 1 or self.partial_fn is not None or self._exchange is not None:
            return None
        import torch.distributed as dist
        try:
            pg = self.group if self.group is not None else dist.distributed_c10d._get_default_group()
            import torch
            be = pg._get_backend(torch.device("cuda"))
        except Exception:
            return None
        return be if hasattr(be, "get_error") and hasattr(be, "abort") else None

    def _collective_error(self) -> Optional[str]:
        """The communicator's asynchronous error (NCCL's ncclCommGetAsyncError, as
        ProcessGroupNCCL.get_error reports it), or None when there is none."""
        be = self._nccl_backend()
        if be is None:
            return None
        err = be.get_error()
        return None if str(err).rsplit(".", 1)[-1] == "SUCCESS" else str(err)

    def _fail(self, why: str, cause: Optional[BaseException] = None):
        from .runtime import TE_STATUS_RUNTIME_ERROR, TinyEngineError
        be = self._nccl_backend()
        if be is not None:
            try:  # abort the communicator: no later collective of this group waits on a failed peer
                be.abort()
            except Exception:
                pass
        if self.store is not None:
            try:
                self.store.set(FAULT_KEY, str(self.spec.rank))
            except Exception:  # the store itself may be gone; the error below still stands
                pass
        raise TinyEngineError(f"KV-split rank {self.spec.rank}, step {self.steps_done}: {why}",
                              TE_STATUS_RUNTIME_ERROR) from cause

    def step(self, q, k_new, v_new):
        """One decode step: q [n_layers][1][heads][hd] raw fp32 (every rank gets the
        same q), k_new/v_new [n_layers][1][kv_heads][hd] (used by the tail rank).
        Returns the merged attention output [n_layers][1][heads][hd] on every rank
        (ready in stream order on the engine's stream).  Raises TinyEngineError
        (TE_STATUS_RUNTIME_ERROR) when this rank fails or learns that a peer has."""
        if self.store is not None and self.store.check([FAULT_KEY]):
            self._fail(f"rank {self.store.get(FAULT_KEY).decode()} reported a failure; no launch made")
        async_err = self._collective_error()
        if async_err is not None:
            self._fail(f"the communicator reported {async_err}; no launch made")
        if injected_fault(self.spec.rank, self.steps_done):
            self._fail("injected fault (TE_FAULT_INJECT)")
        if self._stream is None:
            out = self._step(q, k_new, v_new)
        else:
            import torch
            with torch.cuda.stream(self._stream):
                out = self._step(q, k_new, v_new)
        self.steps_done += 1
        return out

    def _step(self, q, k_new, v_new):
        import torch.distributed as dist
        q_pos = self.length  # global position of the new token
        if self.fused:
            from .runtime import TE_ATTN_ADVANCE
            if self.spec.is_tail:
                self._exchange.decode_kv_split(self.cache, 0, self.n_layers, 0, -1, q, k_new, v_new, self.heads,
                                               TE_ATTN_ADVANCE)
            else:
                self._exchange.decode_kv_split(self.cache, 0, self.n_layers, 0, q_pos, q, None, None, self.heads)
            self.length += 1
            return self._out
        self._local_partial(q, k_new, v_new, q_pos)
        if self._exchange is not None:
            self._exchange.merge(self._part, self._out)
            self.length += 1
            return self._out
        if self.spec.world > 1:
            try:
                dist.all_gather_into_tensor(self._gather_flat, self._part, group=self.group)
            except Exception as e:  # a peer failed or left: the group's timeout ended the collective
                self._fail(f"all-gather of the partial records failed ({type(e).__name__})", e)
        else:
            self._gather[0].copy_(self._part)
        if self.merge_fn is not None:
            self._out.copy_(self.merge_fn(self._gather).reshape(self._out.shape))
        else:
            self.engine.merge_partials(self._gather, self.spec.world, self.n_layers * self.heads, self.head_dim,
                                       self._out)
        self.length += 1
        return self._out


def merge_partials_numpy(parts: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge of partial records [parts][rows][hd+2] (m, l in log2 units);
    used by the host-side tests of the split protocol."""
    m = parts[..., -2]
    l = parts[..., -1]
    acc = parts[..., :-2]
    mx = np.max(np.where(l > 0, m, -np.inf), axis=0)
    w = np.where(l > 0, np.exp2(m - mx), 0.0)
    L = np.sum(l * w, axis=0)
    return np.sum(acc * w[..., None], axis=0) / L[..., None]
