"""GGUF reader for the layer-step integration (host side).

Reads what the reference's parser reads (c/src/gguf.c: te_parse_gguf
:221-300 -- magic "GGUF", version 2 or 3, tensor and key-value counts; the
key-values, every GGUF value type including arrays; the tensor infos, name,
dims (innermost first), ggml type and offset; the data section at the
general.alignment boundary, 32 by default) and the model dimensions it
derives (te_extract_model_info, :370-520: the "<arch>." keys, head_dim =
embedding_length / head_count, head_count_kv defaulting to head_count,
rope.freq_base defaulting to 1e6 for qwen2, the vocabulary from the
tokenizer tokens or else from token_embd.weight).  The file is memory-mapped;
tensors come back as numpy views of their bytes.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8
# bytes per block and weights per block of the types the integration reads
_TYPE_LAYOUT = {GGML_F32: (4, 1), GGML_F16: (2, 1), GGML_Q4_0: (18, 32), GGML_Q8_0: (34, 32)}

_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


class GGUFError(ValueError):
    pass


@dataclass
class Tensor:
    name: str
    ggml_type: int
    dims: tuple  # innermost first, as stored
    offset: int  # absolute, in bytes
    nbytes: int
    data: np.ndarray = field(repr=False)  # uint8 view

    @property
    def rows(self) -> int:
        return int(np.prod(self.dims[1:])) if len(self.dims) > 1 else 1

    @property
    def cols(self) -> int:
        return int(self.dims[0])


class GGUFFile:
    def __init__(self, path: str | Path):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            self._mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        self._buf = memoryview(self._mm)
        self._pos = 0
        magic = self._read(4)
        if magic != b"GGUF":
            raise GGUFError("not a GGUF file")
        (self.version,) = self._unpack("<I")
        if self.version not in (2, 3):
            raise GGUFError(f"unsupported GGUF version {self.version}")
        n_tensors, n_kv = self._unpack("<QQ")
        self.metadata: dict = {}
        for _ in range(n_kv):
            key = self._string()
            (vtype,) = self._unpack("<I")
            self.metadata[key] = self._value(vtype)
        infos = []
        for _ in range(n_tensors):
            name = self._string()
            (nd,) = self._unpack("<I")
            dims = self._unpack(f"<{nd}Q")
            ttype, rel = self._unpack("<IQ")
            infos.append((name, ttype, tuple(int(d) for d in dims), rel))
        align = int(self.metadata.get("general.alignment", 32))
        if align <= 0 or align & (align - 1):
            raise GGUFError("bad general.alignment")
        base = (self._pos + align - 1) // align * align
        raw = np.frombuffer(self._mm, dtype=np.uint8)
        self.tensors: dict[str, Tensor] = {}
        for name, ttype, dims, rel in infos:
            if ttype not in _TYPE_LAYOUT:
                nbytes = 0  # a type the integration does not read; kept for listing
            else:
                bb, per = _TYPE_LAYOUT[ttype]
                n = int(np.prod(dims))
                if n % per:
                    raise GGUFError(f"{name}: {n} elements not whole blocks")
                nbytes = n // per * bb
            off = base + rel
            if off + nbytes > raw.size:
                raise GGUFError(f"{name}: data past the end of the file")
            self.tensors[name] = Tensor(name, ttype, dims, off, nbytes, raw[off:off + nbytes])

    # ---- primitive readers -------------------------------------------------
    def _read(self, n: int) -> bytes:
        if self._pos + n > len(self._buf):
            raise GGUFError("truncated GGUF file")
        b = bytes(self._buf[self._pos:self._pos + n])
        self._pos += n
        return b

    def _unpack(self, fmt: str):
        size = struct.calcsize(fmt)
        return struct.unpack(fmt, self._read(size))

    def _string(self) -> str:
        (n,) = self._unpack("<Q")
        return self._read(n).decode("utf-8", errors="replace")

    def _value(self, vtype: int):
        if vtype in _SCALARS:
            return self._unpack(_SCALARS[vtype])[0]
        if vtype == _STRING:
            return self._string()
        if vtype == _ARRAY:
            etype, n = self._unpack("<IQ")
            if etype in _SCALARS and etype != 7:
                fmt = _SCALARS[etype]
                size = struct.calcsize(fmt)
                arr = np.frombuffer(self._read(size * n), dtype=np.dtype(fmt))
                return arr
            return [self._value(etype) for _ in range(n)]
        raise GGUFError(f"unknown GGUF value type {vtype}")

    # ---- model dimensions (te_extract_model_info) --------------------------
    def qwen2_dims(self) -> dict:
        md = self.metadata
        arch = md.get("general.architecture")
        if arch != "qwen2":
            raise GGUFError(f"architecture {arch!r} is not qwen2")
        p = "qwen2."
        hidden = int(md.get(p + "embedding_length", 0))
        heads = int(md.get(p + "attention.head_count", 0))
        kv_heads = int(md.get(p + "attention.head_count_kv", heads))
        vocab = len(md["tokenizer.ggml.tokens"]) if "tokenizer.ggml.tokens" in md else 0
        emb = self.tensors.get("token_embd.weight")
        if vocab == 0 and emb is not None and len(emb.dims) >= 2:
            vocab = emb.dims[1]
        d = {
            "hidden": hidden,
            "layers": int(md.get(p + "block_count", 0)),
            "ffn": int(md.get(p + "feed_forward_length", 0)),
            "heads": heads,
            "kv_heads": kv_heads,
            "head_dim": hidden // heads if heads else 0,
            "vocab": int(vocab),
            "context": int(md.get(p + "context_length", 0)),
            "eps": float(md.get(p + "attention.layer_norm_rms_epsilon", 0.0)),
            "rope_base": float(md.get(p + "rope.freq_base", 1e6)),
        }
        if min(d["hidden"], d["layers"], d["ffn"], d["heads"], d["kv_heads"], d["vocab"]) == 0 or d["eps"] == 0.0 \
                or hidden % heads:
            raise GGUFError("incomplete qwen2 metadata")
        return d

    def close(self) -> None:
        self.tensors = {}
        self._buf.release()
        try:
            self._mm.close()
        except BufferError:
            pass  # tensor views still held elsewhere keep the mapping until they go
