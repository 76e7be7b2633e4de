"""ctypes binding of libtinyengine.so (include/tinyengine.h + include/tinyengine_attn.h).

Follows the shape of TinyEngine's own binding (python/tinyengine/runtime.py:
library discovery through ``TINYENGINE_LIBRARY`` (:244-268),
``_configure_library`` setting argtypes/restype (:271-378) and ``_check``
raising ``TinyEngineError`` with ``te_strerror`` text (:381-384)).

Compute entry points take device pointers; the helpers below accept torch CUDA
tensors (``data_ptr()``) or raw integer addresses.  Host-buffer calls
(``TE_ATTN_HOST_BUFFERS``) accept numpy arrays or pinned CPU tensors.
"""
from __future__ import annotations

import ctypes
import os
import weakref
from pathlib import Path
from typing import Optional, Sequence

TE_ABI_VERSION = 3
TE_ATTN_ABI_VERSION = 1

TE_STATUS_OK = 0
TE_STATUS_INVALID_ARGUMENT = 1
TE_STATUS_IO_ERROR = 2
TE_STATUS_UNSUPPORTED = 3
TE_STATUS_OUT_OF_MEMORY = 4
TE_STATUS_RUNTIME_ERROR = 5

TE_ATTN_ADVANCE = 1 << 0
TE_ATTN_PARTIAL = 1 << 1
TE_ATTN_NO_ROPE = 1 << 2
TE_ATTN_INPUT_F16 = 1 << 3
TE_ATTN_HOST_BUFFERS = 1 << 4
TE_ATTN_QKV_BIAS = 1 << 5
TE_ATTN_ACCUMULATE = 1 << 6
TE_ATTN_RMSNORM_INPUT = 1 << 7
TE_ATTN_SWIGLU_INPUT = 1 << 8
TE_ATTN_EXACT_Q = 1 << 9
TE_ATTN_STEP_HEAD = 1 << 10
TE_ATTN_QUANT_GGUF_Q4_0 = 4
TE_ATTN_QUANT_GGUF_Q8_0 = 8


class TinyEngineError(RuntimeError):
    def __init__(self, message: str, status: int = TE_STATUS_RUNTIME_ERROR):
        super().__init__(message)
        self.status = status


class AttnOptions(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32),
        ("device", ctypes.c_int32),
        ("stream", ctypes.c_void_p),
        ("decode_chunk_tokens", ctypes.c_uint32),
        ("flags", ctypes.c_uint32),
    ]


class KVCacheDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32),
        ("layers", ctypes.c_uint32),
        ("max_seqs", ctypes.c_uint32),
        ("max_tokens_per_seq", ctypes.c_uint32),
        ("kv_heads", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32),
        ("page_tokens", ctypes.c_uint32),
        ("total_pages", ctypes.c_uint32),
        ("max_position", ctypes.c_uint32),
        ("rope_theta", ctypes.c_float),
    ]


class QwenStepDesc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_uint32),
        ("layers", ctypes.c_uint32),
        ("hidden", ctypes.c_uint32),
        ("heads", ctypes.c_uint32),
        ("ffn", ctypes.c_uint32),
        ("vocab", ctypes.c_uint32),
        ("eps", ctypes.c_float),
        ("quant_qkv", ctypes.c_uint32),
        ("quant_o", ctypes.c_uint32),
        ("quant_gu", ctypes.c_uint32),
        ("quant_down", ctypes.c_uint32),
        ("quant_head", ctypes.c_uint32),
        ("w_qkv", ctypes.POINTER(ctypes.c_void_p)),
        ("w_o", ctypes.POINTER(ctypes.c_void_p)),
        ("w_gu", ctypes.POINTER(ctypes.c_void_p)),
        ("w_down", ctypes.POINTER(ctypes.c_void_p)),
        ("w_head", ctypes.c_void_p),
        ("attn_norm", ctypes.c_void_p),
        ("ffn_norm", ctypes.c_void_p),
        ("out_norm", ctypes.c_void_p),
        ("embedding", ctypes.c_void_p),
    ]


_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_int = ctypes.c_int


def _candidate_libraries() -> list[Path]:
    env = os.environ.get("TINYENGINE_LIBRARY")
    here = Path(__file__).resolve()
    out: list[Path] = []
    if env:
        out.append(Path(env))
    out.append(here.parent / "libtinyengine.so")
    return out


# Every entry point of include/*.h with its ctypes signature (restype, argtypes).
SIGNATURES: dict[str, tuple] = {
    "te_version": (ctypes.c_char_p, []),
    "te_strerror": (ctypes.c_char_p, [_int]),
    "te_rope_f32": (_int, [_f32p, _sz, _sz, _sz, ctypes.c_float]),
    "te_attention_decode_f32": (_int, [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _f32p]),
    "te_attn_default_options": (AttnOptions, []),
    "te_attn_engine_create": (_int, [ctypes.POINTER(AttnOptions), ctypes.POINTER(_vp)]),
    "te_attn_engine_free": (None, [_vp]),
    "te_attn_engine_set_stream": (_int, [_vp, _vp]),
    "te_attn_engine_stream": (_vp, [_vp]),
    "te_attn_engine_synchronize": (_int, [_vp]),
    "te_attn_engine_last_error": (ctypes.c_char_p, [_vp]),
    "te_attn_engine_launch_count": (ctypes.c_uint64, [_vp]),
    "te_attn_engine_time_kernels": (_int, [_vp, _int]),
    "te_attn_engine_set_wait_limit": (_int, [_vp, ctypes.c_uint32]),
    "te_attn_engine_profile": (_int, [_vp, _int]),
    "te_attn_engine_profile_report": (_int, [_vp, ctypes.c_char_p, _sz]),
    "te_attn_engine_last_kernel_ms": (_int, [_vp, ctypes.POINTER(ctypes.c_float)]),
    "te_kv_cache_default_desc": (KVCacheDesc, []),
    "te_kv_cache_create": (_int, [_vp, ctypes.POINTER(KVCacheDesc), ctypes.POINTER(_vp)]),
    "te_kv_cache_free": (None, [_vp]),
    "te_kv_cache_seq_reset": (_int, [_vp, _sz, _sz]),
    "te_kv_cache_seq_truncate": (_int, [_vp, _sz, _sz]),
    "te_kv_cache_seq_length": (_int, [_vp, _sz, ctypes.POINTER(_sz)]),
    "te_kv_cache_reserve": (_int, [_vp, _sz, _sz]),
    "te_kv_cache_write_f16": (_int, [_vp, _sz, _sz, _sz, _sz, _vp, _vp]),
    "te_kv_cache_read_f16": (_int, [_vp, _sz, _sz, _sz, _sz, _vp, _vp]),
    "te_kv_cache_set_qkv_bias": (_int, [_vp, _sz, _sz, _sz, _vp, _vp, _vp]),
    "te_kv_append_rope": (_int, [_vp, _sz, _sz, _sz, _vp, _vp, _sz, ctypes.c_uint32]),
    "te_attention_decode": (_int, [_vp, _sz, _sz, _u32p, _sz, _i64p, _vp, _vp, _vp, _sz, _vp, ctypes.c_uint32]),
    "te_attention_merge_partials": (_int, [_vp, _vp, _sz, _sz, _sz, _vp, ctypes.c_uint32]),
    "te_matvec_gguf": (_int, [_vp, ctypes.c_uint32, _vp, _sz, _sz, _vp, _sz, _vp, ctypes.c_uint32]),
    "te_matvec_gguf_fused": (_int, [_vp, ctypes.c_uint32, _vp, _sz, _sz, _vp, _sz, _vp, ctypes.c_float, _vp,
                                    ctypes.c_uint32]),
    "te_attn_exchange_create": (_int, [_vp, _sz, _sz, _sz, _sz, ctypes.POINTER(_vp), _vp]),
    "te_attn_exchange_connect": (_int, [_vp, _vp]),
    "te_attn_exchange_merge": (_int, [_vp, _vp, _vp]),
    "te_attn_exchange_free": (None, [_vp]),
    "te_attention_decode_kv_split": (_int, [_vp, _vp, _sz, _sz, _sz, ctypes.c_int64, _vp, _vp, _vp, _sz, ctypes.c_uint32]),
    "te_attn_exchange_output": (_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "te_attention_prefill": (_int, [_vp, _sz, _sz, _sz, _vp, _vp, _vp, _sz, _sz, _vp, ctypes.c_uint32]),
    "te_qwen_step_create": (_int, [_vp, ctypes.POINTER(QwenStepDesc), ctypes.POINTER(_vp)]),
    "te_qwen_step_run": (_int, [_vp, _sz, _vp, _vp, _vp, _vp, ctypes.c_uint32]),
    "te_qwen_step_free": (None, [_vp]),
    "te_attention_decode_paged_noalloc": (_int, [_vp, _vp, _vp, _sz, _sz, _sz, _vp, _sz, _sz, _sz, _vp, _vp]),
    "te_attention_decode_paged_noalloc_status": (_int, [_vp, ctypes.POINTER(ctypes.c_int)]),
}


def _configure_library(lib: ctypes.CDLL) -> None:
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes


_LIB: Optional[ctypes.CDLL] = None


def load_library() -> ctypes.CDLL:
    """Loads libtinyengine.so; raises TinyEngineError when it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    for cand in _candidate_libraries():
        if cand.is_file():
            lib = ctypes.CDLL(str(cand))
            _configure_library(lib)
            _LIB = lib
            return lib
    searched = "\n".join(str(p) for p in _candidate_libraries())
    raise TinyEngineError(
        "libtinyengine.so not found (build it with `python -m tinymetalagent_b200.build`). Searched:\n" + searched,
        TE_STATUS_UNSUPPORTED,
    )


def _check(lib: ctypes.CDLL, status: int, engine=None) -> None:
    if status != TE_STATUS_OK:
        message = lib.te_strerror(status).decode()
        if engine is not None:
            detail = lib.te_attn_engine_last_error(engine)
            if detail:
                message = f"{message}: {detail.decode()}"
        raise TinyEngineError(message, status)


def _addr(x) -> Optional[int]:
    """Device/host address of a torch tensor, numpy array, int or None."""
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "ctypes"):
        return x.ctypes.data
    raise TypeError(f"cannot take the address of {type(x)!r}")


# ---------------------------------------------------------------------------
# Drop-in CPU-API functions (host fp32 buffers, same contract as the reference)
# ---------------------------------------------------------------------------

def rope_f32(values, heads: int, head_dim: int, position: int, theta: float) -> None:
    """In-place te_rope_f32 on a float32 numpy array (runs on the current CUDA device)."""
    lib = load_library()
    _check(lib, lib.te_rope_f32(values.ctypes.data_as(_f32p), heads, head_dim, position, theta))


def attention_decode_f32(query, key_cache, value_cache, position: int, heads: int, kv_heads: int,
                         head_dim: int, out) -> None:
    """te_attention_decode_f32 on float32 numpy arrays."""
    lib = load_library()
    _check(lib, lib.te_attention_decode_f32(
        query.ctypes.data_as(_f32p), key_cache.ctypes.data_as(_f32p), value_cache.ctypes.data_as(_f32p),
        position, heads, kv_heads, head_dim, out.ctypes.data_as(_f32p)))


# ---------------------------------------------------------------------------
# Device-resident engine
# ---------------------------------------------------------------------------

class AttnEngine:
    """One engine per GPU: owns a stream (or uses the given one) and decode scratch."""

    def __init__(self, device: int = 0, stream: Optional[int] = None, decode_chunk_tokens: int = 0):
        self.lib = load_library()
        opts = self.lib.te_attn_default_options()
        opts.device = device
        opts.stream = stream
        opts.decode_chunk_tokens = decode_chunk_tokens
        handle = _vp()
        _check(self.lib, self.lib.te_attn_engine_create(ctypes.byref(opts), ctypes.byref(handle)))
        self.handle = handle
        self.device = device
        self._caches = weakref.WeakSet()

    def close(self) -> None:
        """Frees the engine; caches created from it are freed first (the C
        library frees a cache through its engine)."""
        if getattr(self, "handle", None):
            for cache in list(getattr(self, "_caches", ())):
                cache.close()
            self.lib.te_attn_engine_free(self.handle)
            self.handle = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    def check(self, status: int) -> None:
        _check(self.lib, status, self.handle)

    @property
    def stream(self) -> int:
        return self.lib.te_attn_engine_stream(self.handle) or 0

    def set_stream(self, stream: Optional[int]) -> None:
        self.check(self.lib.te_attn_engine_set_stream(self.handle, stream))

    def synchronize(self) -> None:
        self.check(self.lib.te_attn_engine_synchronize(self.handle))

    @property
    def launch_count(self) -> int:
        return int(self.lib.te_attn_engine_launch_count(self.handle))

    def time_kernels(self, enable: bool = True) -> None:
        """Record CUDA events around te_attention_prefill's attention kernel."""
        self.check(self.lib.te_attn_engine_time_kernels(self.handle, 1 if enable else 0))

    def last_kernel_ms(self) -> float:
        ms = ctypes.c_float(0.0)
        self.check(self.lib.te_attn_engine_last_kernel_ms(self.handle, ctypes.byref(ms)))
        return float(ms.value)

    def set_wait_limit(self, milliseconds: int) -> None:
        """Bound of the waits for other GPUs (the NVLink exchange); see te_attn_engine_set_wait_limit."""
        self.check(self.lib.te_attn_engine_set_wait_limit(self.handle, int(milliseconds)))

    def profile(self, enable: bool = True) -> None:
        """Per-kernel device-time profile of this engine's launches (TINYENGINE_PROFILE)."""
        self.check(self.lib.te_attn_engine_profile(self.handle, 1 if enable else 0))

    def profile_report(self) -> str:
        """The profile's 'tinyengine_profile: device_ms=... decode=ms/calls ...' line (synchronises)."""
        buf = ctypes.create_string_buffer(512)
        self.check(self.lib.te_attn_engine_profile_report(self.handle, buf, len(buf)))
        return buf.value.decode()

    def merge_partials(self, partials, n_parts: int, rows: int, head_dim: int, out, partial_out: bool = False):
        self.check(self.lib.te_attention_merge_partials(
            self.handle, _addr(partials), n_parts, rows, head_dim, _addr(out),
            TE_ATTN_PARTIAL if partial_out else 0))

    def kv_cache(self, **kw) -> "KVCache":
        return KVCache(self, **kw)

    def matvec_gguf_fused(self, quant: int, w, rows: int, cols: int, x, y, flags: int, norm_weight=None,
                          eps: float = 0.0, n_vectors: int = 1) -> None:
        """y[v] = W p(x[v]) (or y[v] += that, with TE_ATTN_ACCUMULATE), p the RMSNorm (TE_ATTN_RMSNORM_INPUT,
        with norm_weight and eps) or the SwiGLU of x[v] = [gate | up] (TE_ATTN_SWIGLU_INPUT); 1..8 vectors."""
        self.check(self.lib.te_matvec_gguf_fused(self.handle, quant, _addr(w), rows, cols, _addr(x), n_vectors,
                                                 _addr(norm_weight), eps, _addr(y), flags))

    def matvec_gguf(self, quant: int, w, rows: int, cols: int, x, y, n_vectors: int = 1, flags: int = 0) -> None:
        """y[v][r] = sum_c W[r][c] x[v][c] (or y += that, with TE_ATTN_ACCUMULATE) for a GGUF Q4_0 / Q8_0
        matrix (raw bytes, device)."""
        self.check(self.lib.te_matvec_gguf(self.handle, quant, _addr(w), rows, cols, _addr(x), n_vectors, _addr(y),
                                           flags))


IPC_HANDLE_BYTES = 64


class Exchange:
    """NVLink exchange + merge of KV-split partial records (te_attn_exchange_*): one
    per rank, all ranks with the same world, rows and head_dim, each on its own GPU."""

    def __init__(self, engine: "AttnEngine", world: int, rank: int, rows: int, head_dim: int):
        self.engine = engine
        self.lib = engine.lib
        handle = _vp()
        buf = (ctypes.c_ubyte * IPC_HANDLE_BYTES)()
        engine.check(self.lib.te_attn_exchange_create(engine.handle, world, rank, rows, head_dim,
                                                      ctypes.byref(handle), ctypes.addressof(buf)))
        self.handle = handle
        self.ipc_handle = bytes(buf)
        self.world, self.rank = world, rank

    def connect(self, handles: Sequence[bytes]) -> None:
        """handles: every rank's ipc_handle, in rank order."""
        blob = b"".join(handles)
        if len(blob) != self.world * IPC_HANDLE_BYTES:
            raise ValueError("need one 64-byte handle per rank")
        buf = (ctypes.c_ubyte * len(blob)).from_buffer_copy(blob)
        self.engine.check(self.lib.te_attn_exchange_connect(self.handle, ctypes.addressof(buf)))

    def merge(self, partial, out) -> None:
        self.engine.check(self.lib.te_attn_exchange_merge(self.handle, _addr(partial), _addr(out)))

    def decode_kv_split(self, cache: "KVCache", layer_begin: int, n_layers: int, seq: int, q_position: int, q,
                        k_new, v_new, heads: int, flags: int = 0) -> None:
        """te_attention_decode_kv_split: this rank's share of one fused KV-split decode step."""
        self.engine.check(self.lib.te_attention_decode_kv_split(
            self.handle, cache.handle, layer_begin, n_layers, seq, int(q_position), _addr(q), _addr(k_new),
            _addr(v_new), heads, flags))

    def output(self, shape):
        """The merged output region as a float32 CUDA tensor of `shape` (a view, not a copy)."""
        import torch
        ptr = ctypes.c_void_p()
        self.engine.check(self.lib.te_attn_exchange_output(self.handle, ctypes.byref(ptr)))

        class _View:  # __cuda_array_interface__ lets torch wrap the library's memory without a copy
            __cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr.value, False),
                                        "version": 2, "strides": None}
        return torch.as_tensor(_View(), device=f"cuda:{self.engine.device}")

    def close(self) -> None:
        if getattr(self, "handle", None):
            self.lib.te_attn_exchange_free(self.handle)
            self.handle = None


class KVCache:
    """Paged f16 KV cache in HBM: [layers][pages][kv_heads][page_tokens][head_dim] per K and V."""

    def __init__(self, engine: AttnEngine, layers: int, max_seqs: int, max_tokens_per_seq: int, kv_heads: int,
                 head_dim: int, page_tokens: int = 128, total_pages: int = 0, max_position: int = 0,
                 rope_theta: float = 1e6):
        self.engine = engine
        self.lib = engine.lib
        d = self.lib.te_kv_cache_default_desc()
        d.layers, d.max_seqs, d.max_tokens_per_seq = layers, max_seqs, max_tokens_per_seq
        d.kv_heads, d.head_dim, d.page_tokens = kv_heads, head_dim, page_tokens
        d.total_pages, d.max_position, d.rope_theta = total_pages, max_position, rope_theta
        handle = _vp()
        engine.check(self.lib.te_kv_cache_create(engine.handle, ctypes.byref(d), ctypes.byref(handle)))
        self.handle = handle
        engine._caches.add(self)
        self.layers, self.max_seqs, self.kv_heads, self.head_dim = layers, max_seqs, kv_heads, head_dim
        self.page_tokens = page_tokens
        self.max_tokens_per_seq = max_tokens_per_seq
        self.rope_theta = rope_theta
        self._steps = weakref.WeakSet()

    def close(self) -> None:
        # Steps built on this cache go first; an engine that is already gone
        # has freed this cache with itself.
        for step in list(getattr(self, "_steps", ())):
            step.close()
        if getattr(self, "handle", None) and getattr(self.engine, "handle", None):
            self.lib.te_kv_cache_free(self.handle)
        self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def _c(self, status: int) -> None:
        self.engine.check(status)

    def reset(self, seq: int, position_offset: int = 0) -> None:
        self._c(self.lib.te_kv_cache_seq_reset(self.handle, seq, position_offset))

    def truncate(self, seq: int, length: int) -> None:
        self._c(self.lib.te_kv_cache_seq_truncate(self.handle, seq, length))

    def reserve(self, seq: int, tokens: int) -> None:
        """Map pages for `tokens` tokens now (graph-capturable decode steps afterwards)."""
        self._c(self.lib.te_kv_cache_reserve(self.handle, seq, tokens))

    def length(self, seq: int) -> int:
        n = _sz()
        self._c(self.lib.te_kv_cache_seq_length(self.handle, seq, ctypes.byref(n)))
        return n.value

    def write_f16(self, layer: int, seq: int, token_begin: int, k, v) -> None:
        """k, v: [n][kv_heads][head_dim] binary16 (torch f16 tensor, numpy float16/uint16)."""
        n = int(k.shape[0])
        self._c(self.lib.te_kv_cache_write_f16(self.handle, layer, seq, token_begin, n, _addr(k), _addr(v)))

    def set_qkv_bias(self, layer_begin: int, heads: int, q_bias=None, k_bias=None, v_bias=None) -> None:
        """fp32 projection biases of layers [layer_begin, +n): q_bias [n][heads * head_dim], k_bias and
        v_bias [n][kv_heads * head_dim] (numpy or torch; None = zeros).  Calls with TE_ATTN_QKV_BIAS add
        them to the raw q/k/v inputs before RoPE and rounding."""
        import numpy as np
        arrs = []
        n = None
        for b, width in ((q_bias, heads * self.head_dim), (k_bias, self.kv_heads * self.head_dim),
                         (v_bias, self.kv_heads * self.head_dim)):
            if b is None:
                arrs.append(None)
                continue
            if hasattr(b, "detach"):
                b = b.detach().float().contiguous()
            else:
                b = np.ascontiguousarray(np.asarray(b, dtype=np.float32))
            rows = int(b.numel() if hasattr(b, "numel") else b.size) // width
            n = rows if n is None else n
            if rows * width != (b.numel() if hasattr(b, "numel") else b.size) or rows != n:
                raise ValueError("bias shapes disagree with heads / kv_heads * head_dim")
            arrs.append(b)
        if n is None:
            raise ValueError("no bias given")
        ptr = lambda b: None if b is None else _addr(b)  # noqa: E731
        self._c(self.lib.te_kv_cache_set_qkv_bias(self.handle, layer_begin, n, heads, ptr(arrs[0]), ptr(arrs[1]),
                                                  ptr(arrs[2])))

    def read_f16(self, layer: int, seq: int, token_begin: int, n_tokens: int):
        import numpy as np
        k = np.zeros((n_tokens, self.kv_heads, self.head_dim), dtype=np.uint16)
        v = np.zeros_like(k)
        self._c(self.lib.te_kv_cache_read_f16(self.handle, layer, seq, token_begin, n_tokens, k.ctypes.data,
                                              v.ctypes.data))
        return k, v

    def append_rope(self, layer_begin: int, n_layers: int, seq: int, k, v, n_tokens: int, flags: int = 0) -> None:
        self._c(self.lib.te_kv_append_rope(self.handle, layer_begin, n_layers, seq, _addr(k), _addr(v), n_tokens,
                                           flags))

    def decode(self, layer_begin: int, n_layers: int, seq_ids: Sequence[int], q, out, heads: int,
               k_new=None, v_new=None, q_positions: Optional[Sequence[int]] = None, flags: int = 0) -> None:
        n = len(seq_ids)
        ids = (ctypes.c_uint32 * n)(*seq_ids)
        qp = (ctypes.c_int64 * n)(*q_positions) if q_positions is not None else None
        self._c(self.lib.te_attention_decode(self.handle, layer_begin, n_layers, ids, n, qp, _addr(q),
                                             _addr(k_new), _addr(v_new), heads, _addr(out), flags))

    def prefill(self, layer_begin: int, n_layers: int, seq: int, q, k, v, n_tokens: int, heads: int, out,
                flags: int = 0) -> None:
        self._c(self.lib.te_attention_prefill(self.handle, layer_begin, n_layers, seq, _addr(q), _addr(k), _addr(v),
                                              n_tokens, heads, _addr(out), flags))


class QwenStep:
    """te_qwen_step_*: every layer of one qwen2 decode token (and optionally the
    output norm, lm_head and argmax) in one cooperative launch over `cache`.

    Weights are device tensors (or addresses): per-layer lists w_qkv, w_o,
    w_gu, w_down of GGUF Q4_0/Q8_0 rows, w_head, and the fp32 norms and
    embedding table; quants maps "qkv", "o", "gu", "down", "head" to
    TE_ATTN_QUANT_GGUF_*.  The library packs its own copy of the weights at
    creation."""

    def __init__(self, cache: KVCache, *, layers: int, hidden: int, heads: int, ffn: int, vocab: int, eps: float,
                 quants: dict, w_qkv, w_o, w_gu, w_down, w_head, attn_norm, ffn_norm, out_norm, embedding):
        self.cache = cache
        self.engine = cache.engine
        self.lib = cache.lib
        d = QwenStepDesc()
        d.abi_version = TE_ATTN_ABI_VERSION
        d.layers, d.hidden, d.heads, d.ffn, d.vocab, d.eps = layers, hidden, heads, ffn, vocab, eps
        d.quant_qkv, d.quant_o, d.quant_gu = quants["qkv"], quants["o"], quants["gu"]
        d.quant_down, d.quant_head = quants["down"], quants["head"]
        arrays = []
        for name, ws in (("w_qkv", w_qkv), ("w_o", w_o), ("w_gu", w_gu), ("w_down", w_down)):
            if len(ws) != layers:
                raise ValueError(f"{name}: one matrix per layer")
            arr = (ctypes.c_void_p * layers)(*[_addr(w) for w in ws])
            arrays.append(arr)
            setattr(d, name, ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p)))
        d.w_head, d.attn_norm, d.ffn_norm = _addr(w_head), _addr(attn_norm), _addr(ffn_norm)
        d.out_norm, d.embedding = _addr(out_norm), _addr(embedding)
        handle = _vp()
        self.engine.check(self.lib.te_qwen_step_create(cache.handle, ctypes.byref(d), ctypes.byref(handle)))
        self.handle = handle
        cache._steps.add(self)

    def run(self, seq: int, token, hidden, logits=None, next_token=None, flags: int = 0) -> None:
        """token / next_token: one-element int64 device tensors (or addresses); hidden [hidden] fp32."""
        self.engine.check(self.lib.te_qwen_step_run(self.handle, seq, _addr(token), _addr(hidden), _addr(logits),
                                                    _addr(next_token), flags))

    def close(self) -> None:
        if getattr(self, "handle", None) and getattr(self.engine, "handle", None):
            self.lib.te_qwen_step_free(self.handle)
        self.handle = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass
