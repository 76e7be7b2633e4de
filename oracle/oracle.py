"""CPU oracle for the attention stage -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU baseline
import this module.  It loads two C builds through ctypes:

* ``liboracle.so`` -- this repository's restatement (``te_oracle.c``) of
  TinyEngine's CPU path (``c/src/ops.c:295-395``, ``c/src/qwen.c:531-539``,
  ``c/src/qwen.c:810-824``);
* ``_ref/libteref.so`` -- the reference's own ``c/src/ops.c`` compiled from its
  sources by ``oracle/Makefile`` (present where the reference was available at
  build time; the built file travels with the repository snapshot);
* ``_ref/libteqwen.so`` -- the reference's CPU forward pass (``c/src/qwen.c``
  ``te_qwen_forward_token`` / ``te_qwen_project_next`` with its GGUF parser),
  built the same way (``ref_qwen.c``), the checker of the layer step.

ctypes releases the GIL during each foreign call, so the threaded CPU baseline
runs the single-threaded C functions on several cores at once.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libteref.so"
REF_QWEN_LIB = HERE / "_ref" / "libteqwen.so"

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_sz = ctypes.c_size_t


def build() -> None:
    """Compile liboracle.so (and _ref/libteref.so when the reference is present)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _ptr(a: np.ndarray, typ=_f32p):
    return a.ctypes.data_as(typ)


class _Lib:
    def __init__(self, path: Path, prefix: str):
        if not path.is_file():
            raise FileNotFoundError(f"oracle library missing: {path} (run `make -C oracle`)")
        self.lib = ctypes.CDLL(str(path))
        self.path = path
        p = prefix
        self.rope = getattr(self.lib, f"{p}rope_f32")
        self.rope.argtypes = [_f32p, _sz, _sz, _sz, ctypes.c_float]
        self.rope.restype = ctypes.c_int
        self.attn = getattr(self.lib, f"{p}attention_decode_f32")
        self.attn.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _f32p]
        self.attn.restype = ctypes.c_int

    def rope_f32(self, values: np.ndarray, heads: int, head_dim: int, position: int, theta: float) -> int:
        assert values.dtype == np.float32 and values.flags.c_contiguous
        return self.rope(_ptr(values), heads, head_dim, position, theta)

    def attention_decode_f32(self, q, k, v, position, heads, kv_heads, head_dim, out=None):
        q = np.ascontiguousarray(q, dtype=np.float32)
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        if out is None:
            out = np.zeros(heads * head_dim, dtype=np.float32)
        st = self.attn(_ptr(q), _ptr(k), _ptr(v), position, heads, kv_heads, head_dim, _ptr(out))
        if st != 0:
            raise RuntimeError(f"oracle attention status {st}")
        return out


class Port(_Lib):
    """The repository's C restatement (liboracle.so)."""

    def __init__(self):
        super().__init__(PORT_LIB, "or_")
        L = self.lib
        L.or_rope_table.argtypes = [_f32p, _f32p, _sz, _sz, ctypes.c_float]
        L.or_f32_to_f16_array.argtypes = [_f32p, _u16p, _sz]
        L.or_f16_to_f32_array.argtypes = [_u16p, _f32p, _sz]
        L.or_append_rope_f16.argtypes = [_f32p, _f32p, _sz, _sz, _sz, _sz, ctypes.c_float, _u16p, _u16p]
        L.or_causal_prefill_f32.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _f32p]
        L.or_decode_partial_f32.argtypes = [_f32p, _f32p, _f32p, _sz, _sz, _sz, _sz, _sz, _f32p]
        L.or_merge_partials_f32.argtypes = [_f32p, _sz, _sz, _sz, _f32p]
        L.or_matvec_q4_0_f32.argtypes = [ctypes.c_void_p, _sz, _sz, _f32p, _f32p]
        L.or_matvec_q8_0_f32.argtypes = [ctypes.c_void_p, _sz, _sz, _f32p, _f32p]
        for name in ("or_rope_table", "or_append_rope_f16", "or_causal_prefill_f32",
                     "or_decode_partial_f32", "or_merge_partials_f32"):
            getattr(L, name).restype = ctypes.c_int

    def rope_table(self, positions: int, head_dim: int, theta: float):
        half = head_dim // 2
        cos = np.zeros((positions, half), dtype=np.float32)
        sin = np.zeros((positions, half), dtype=np.float32)
        st = self.lib.or_rope_table(_ptr(cos), _ptr(sin), positions, head_dim, theta)
        assert st == 0
        return cos, sin

    def f32_to_f16_bits(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(x.shape, dtype=np.uint16)
        self.lib.or_f32_to_f16_array(_ptr(x), _ptr(out, _u16p), x.size)
        return out

    def f16_bits_to_f32(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.uint16)
        out = np.zeros(x.shape, dtype=np.float32)
        self.lib.or_f16_to_f32_array(_ptr(x, _u16p), _ptr(out), x.size)
        return out

    def append_rope_f16(self, k_raw, v_raw, first_position: int, kv_heads: int, head_dim: int, theta: float):
        """k_raw/v_raw [n][kv_heads][head_dim] fp32 -> (k_bits, v_bits) f16 bit patterns."""
        k_raw = np.ascontiguousarray(k_raw, dtype=np.float32)
        v_raw = np.ascontiguousarray(v_raw, dtype=np.float32)
        n = k_raw.size // (kv_heads * head_dim)
        kb = np.zeros(k_raw.shape, dtype=np.uint16)
        vb = np.zeros(v_raw.shape, dtype=np.uint16)
        st = self.lib.or_append_rope_f16(_ptr(k_raw), _ptr(v_raw), n, first_position, kv_heads,
                                         head_dim, theta, _ptr(kb, _u16p), _ptr(vb, _u16p))
        assert st == 0
        return kb, vb

    def causal_prefill_f32(self, q_rot, k, v, seq_len, heads, kv_heads, head_dim):
        q_rot = np.ascontiguousarray(q_rot, dtype=np.float32)
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        out = np.zeros((seq_len, heads, head_dim), dtype=np.float32)
        st = self.lib.or_causal_prefill_f32(_ptr(q_rot), _ptr(k), _ptr(v), seq_len, heads,
                                            kv_heads, head_dim, _ptr(out))
        assert st == 0
        return out

    def decode_partial_f32(self, q, k, v, begin, end, heads, kv_heads, head_dim):
        q = np.ascontiguousarray(q, dtype=np.float32)
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        out = np.zeros((heads, head_dim + 2), dtype=np.float32)
        st = self.lib.or_decode_partial_f32(_ptr(q), _ptr(k), _ptr(v), begin, end, heads,
                                            kv_heads, head_dim, _ptr(out))
        assert st == 0
        return out

    def matvec_q4_0_f32(self, w, rows, cols, x):
        w = np.ascontiguousarray(w, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(rows, dtype=np.float32)
        assert self.lib.or_matvec_q4_0_f32(w.ctypes.data, rows, cols, _ptr(x), _ptr(out)) == 0
        return out

    def matvec_q8_0_f32(self, w, rows, cols, x):
        w = np.ascontiguousarray(w, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(rows, dtype=np.float32)
        assert self.lib.or_matvec_q8_0_f32(w.ctypes.data, rows, cols, _ptr(x), _ptr(out)) == 0
        return out

    def merge_partials_f32(self, partials, heads, head_dim):
        partials = np.ascontiguousarray(partials, dtype=np.float32)
        n_parts = partials.size // (heads * (head_dim + 2))
        out = np.zeros((heads, head_dim), dtype=np.float32)
        st = self.lib.or_merge_partials_f32(_ptr(partials), n_parts, heads, head_dim, _ptr(out))
        assert st == 0
        return out


class Ref(_Lib):
    """The reference's own ops.c, compiled by oracle/Makefile into _ref/libteref.so."""

    def __init__(self):
        super().__init__(REF_LIB, "te_")
        self.lib.ref_stub_model.restype = ctypes.c_void_p
        self.lib.ref_stub_register_tensor.argtypes = [ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint64,
                                                     ctypes.c_void_p, ctypes.c_size_t]
        self.lib.te_model_matvec_f32.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_float),
                                                 ctypes.c_size_t, ctypes.POINTER(ctypes.c_float), ctypes.c_size_t,
                                                 ctypes.POINTER(ctypes.c_size_t)]
        self.lib.te_model_matvec_f32.restype = ctypes.c_int

    def model_matvec_f32(self, ggml_type: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        """te_model_matvec_f32 of the reference on a GGUF-typed matrix given as raw bytes
        (ggml type 2 = Q4_0, 8 = Q8_0); its Metal path is stubbed out, so this is its CPU row loop."""
        w = np.ascontiguousarray(w, dtype=np.uint8)
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(rows, dtype=np.float32)
        written = ctypes.c_size_t(0)
        self.lib.ref_stub_register_tensor(ggml_type, cols, rows, w.ctypes.data, w.size)
        st = self.lib.te_model_matvec_f32(self.lib.ref_stub_model(), b"w", _ptr(x), cols, _ptr(out), rows,
                                          ctypes.byref(written))
        self.lib.ref_stub_register_tensor(0, 0, 0, None, 0)
        assert st == 0 and written.value == rows, st
        return out


class RefQwen:
    """The reference's per-token forward pass on a GGUF file (one model per process: the
    harness keeps it in file-scope state).  forward(token, position) -> hidden [hidden] fp32;
    project() -> (logits [vocab], greedy token)."""

    def __init__(self, path, context_tokens: int):
        if not REF_QWEN_LIB.is_file():
            raise FileNotFoundError(f"oracle library missing: {REF_QWEN_LIB}")
        self.lib = ctypes.CDLL(str(REF_QWEN_LIB))
        self.lib.rq_open.argtypes = [ctypes.c_char_p, ctypes.c_uint32]
        self.lib.rq_forward.argtypes = [ctypes.c_uint32, ctypes.c_size_t, _f32p]
        self.lib.rq_project.argtypes = [_f32p, ctypes.POINTER(ctypes.c_uint32)]
        self.lib.rq_dims.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
        st = self.lib.rq_open(str(path).encode(), context_tokens)
        if st != 0:
            raise RuntimeError(f"reference model load failed: status {st}")
        d = (ctypes.c_uint64 * 8)()
        self.lib.rq_dims(d)
        keys = ("hidden", "ffn", "layers", "heads", "kv_heads", "head_dim", "vocab", "context")
        self.dims = {k: int(v) for k, v in zip(keys, d)}

    def forward(self, token: int, position: int) -> np.ndarray:
        h = np.zeros(self.dims["hidden"], np.float32)
        st = self.lib.rq_forward(token, position, _ptr(h))
        assert st == 0, st
        return h

    def project(self):
        logits = np.zeros(self.dims["vocab"], np.float32)
        tok = ctypes.c_uint32()
        st = self.lib.rq_project(_ptr(logits), ctypes.byref(tok))
        assert st == 0, st
        return logits, int(tok.value)

    def close(self) -> None:
        self.lib.rq_close()


def ref_qwen_available() -> bool:
    return REF_QWEN_LIB.is_file()


_port = None
_ref = None


def port() -> Port:
    global _port
    if _port is None:
        _port = Port()
    return _port


def ref_available() -> bool:
    return REF_LIB.is_file()


def ref() -> Ref:
    global _ref
    if _ref is None:
        _ref = Ref()
    return _ref


def f16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even f16 -> fp32 (numpy's float16 cast is round-to-nearest-even)."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
