"""Qwen2 decode step on one GPU: the layer-step integration.

Mirrors the reference's per-token forward pass, te_qwen_forward_token
(c/src/qwen.c:907-1112), and its greedy projection, te_qwen_project_next
(:1303-1377), on a GGUF model, with this repository's kernels on the hot
path:

  per layer   RMSNorm(x, attn_norm)                          glue (below)
              q|k|v = W_qkv n            one te_matvec_gguf over the q, k and v
                                         rows stacked (they share the input)
              bias + RoPE + f16 append + GQA decode
                                         one te_attention_decode launch
                                         (TE_ATTN_QKV_BIAS: the biases are added
                                         in fp32 inside it, :998-1011)
              x += W_o attn              te_matvec_gguf + TE_ATTN_ACCUMULATE
              RMSNorm(x, ffn_norm)                           glue
              g|u = W_gate|up n          one te_matvec_gguf (rows stacked)
              s = SwiGLU(g, u)                               glue
              x += W_down s              te_matvec_gguf + TE_ATTN_ACCUMULATE
  head        RMSNorm(x, output_norm); logits = W_out n (te_matvec_gguf); argmax

The glue -- the embedding row, RMSNorm, SwiGLU, argmax -- is elementwise work
on a few thousand values per token, done with device tensor operations in the
reference's arithmetic: RMSNorm sums squares in double, then
scale = 1 / sqrt(float(mean) + eps) and out = (x * scale) * w (te_rmsnorm_f32,
ops.c:272-293); SwiGLU is g / (1 + exp(-g)) * u (te_swiglu_f32, ops.c:397-406);
argmax takes the first maximum (te_argmax_f32).

One difference from the reference's CPU pass is by design: the KV cache is
the engine's f16 cache (the reference's Metal path's layout), where the CPU
pass keeps fp32 keys and values, so outputs agree to f16 rounding of K/V, not
bit for bit.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from .gguf import GGML_F32, GGML_Q4_0, GGML_Q8_0, GGUFError, GGUFFile
from .runtime import TE_ATTN_ACCUMULATE, TE_ATTN_ADVANCE, TE_ATTN_QKV_BIAS, AttnEngine

_QUANT = {GGML_Q4_0: 4, GGML_Q8_0: 8}  # ggml type -> TE_ATTN_QUANT_GGUF_*


class QwenDecoder:
    """One sequence of a qwen2 GGUF model on the engine's device.

    forward_token(token, position) runs every layer for one token (the token
    at `position` of the sequence; positions must follow one another from 0,
    or restart below the current length, which truncates the cache there) and
    returns the hidden state (a device tensor [hidden]); project_next()
    returns the greedy next token and leaves the logits in `self.logits`.
    """

    def __init__(self, engine: AttnEngine, model: str | Path | GGUFFile, context_tokens: int):
        import torch

        self.engine = engine
        self.gguf = model if isinstance(model, GGUFFile) else GGUFFile(model)
        d = self.gguf.qwen2_dims()
        self.dims = d
        H, L, F = d["hidden"], d["layers"], d["ffn"]
        heads, kvh, hd = d["heads"], d["kv_heads"], d["head_dim"]
        self.kv = kvh * hd
        if hd not in (64, 128) or heads % kvh or heads // kvh > 16 or H % 32 or F % 32:
            raise GGUFError("model shape outside the engine's decode kernel (head_dim 64/128, group <= 16)")
        if context_tokens < 1:
            raise ValueError("context_tokens must be positive")
        self.context_tokens = context_tokens
        dev = torch.device("cuda", engine.device)
        self._dev = dev
        # every tensor operation here runs on the engine's stream, in order
        # with its kernels
        self._stream = torch.cuda.ExternalStream(engine.stream, device=dev)
        t = self.gguf.tensors

        def raw(name):
            return torch.from_numpy(np.array(t[name].data)).to(dev)  # a writable copy of the mapped bytes

        def f32(name, n):
            tt = t[name]
            if tt.ggml_type != GGML_F32 or int(np.prod(tt.dims)) != n:
                raise GGUFError(f"{name}: expected {n} fp32 values")
            return torch.from_numpy(tt.data.view(np.float32).copy()).to(dev)

        def quant_of(*names):
            types = {t[n].ggml_type for n in names}
            if len(types) != 1 or next(iter(types)) not in _QUANT:
                raise GGUFError(f"{names}: projections must share one of Q4_0 / Q8_0")
            return _QUANT[types.pop()]

        def stacked(*names):
            # rows of several matrices with the same input, one after another
            return torch.from_numpy(np.concatenate([t[n].data for n in names])).to(dev)

        with torch.cuda.stream(self._stream):
            self._load(d, t, raw, f32, quant_of, stacked)
        self._stream.synchronize()

    def _load(self, d, t, raw, f32, quant_of, stacked):
        import torch
        H, L, F = d["hidden"], d["layers"], d["ffn"]
        heads, kvh, hd = d["heads"], d["kv_heads"], d["head_dim"]
        dev = self._dev
        self.layers = []
        qb = np.zeros((L, H), np.float32)
        kb = np.zeros((L, self.kv), np.float32)
        vb = np.zeros((L, self.kv), np.float32)
        for layer in range(L):
            p = f"blk.{layer}."
            names_qkv = (p + "attn_q.weight", p + "attn_k.weight", p + "attn_v.weight")
            names_gu = (p + "ffn_gate.weight", p + "ffn_up.weight")
            self.layers.append({
                "attn_norm": f32(p + "attn_norm.weight", H),
                "ffn_norm": f32(p + "ffn_norm.weight", H),
                "qkv": stacked(*names_qkv), "q_qkv": quant_of(*names_qkv),
                "o": raw(p + "attn_output.weight"), "q_o": quant_of(p + "attn_output.weight"),
                "gu": stacked(*names_gu), "q_gu": quant_of(*names_gu),
                "down": raw(p + "ffn_down.weight"), "q_down": quant_of(p + "ffn_down.weight"),
            })
            qb[layer] = t[p + "attn_q.bias"].data.view(np.float32)
            kb[layer] = t[p + "attn_k.bias"].data.view(np.float32)
            vb[layer] = t[p + "attn_v.bias"].data.view(np.float32)
        emb = t["token_embd.weight"]
        if emb.ggml_type not in (GGML_Q8_0, GGML_Q4_0, GGML_F32):
            raise GGUFError("token_embd.weight: unsupported type")
        self._emb_type = emb.ggml_type
        self._emb = raw("token_embd.weight")
        head = "output.weight" if "output.weight" in t else "token_embd.weight"
        self._head = raw(head)
        self._q_head = quant_of(head)
        self._out_norm = f32("output_norm.weight", H)

        self.cache = self.engine.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=self.context_tokens,
                                          kv_heads=kvh, head_dim=hd, max_position=self.context_tokens,
                                          rope_theta=d["rope_base"])
        self.cache.set_qkv_bias(0, heads, qb, kb, vb)
        self.x = torch.zeros(H, dtype=torch.float32, device=dev)
        self._qkv = torch.empty(H + 2 * self.kv, dtype=torch.float32, device=dev)
        self._attn = torch.empty(H, dtype=torch.float32, device=dev)
        self._gu = torch.empty(2 * F, dtype=torch.float32, device=dev)
        self.logits = torch.empty(d["vocab"], dtype=torch.float32, device=dev)

    # ---- glue (reference arithmetic) ---------------------------------------
    def _rmsnorm(self, x, w):
        import torch
        ss = torch.sum(x.double() * x.double())
        scale = 1.0 / torch.sqrt((ss / x.numel()).float() + self.dims["eps"])
        return (x * scale) * w

    def _embed(self, token: int):
        import torch
        H = self.dims["hidden"]
        if self._emb_type == GGML_F32:
            return self._emb.view(torch.float32).view(-1, H)[token].clone()
        width = 34 if self._emb_type == GGML_Q8_0 else 18
        row = self._emb.view(-1, H // 32, width)[token]
        scale = row[:, 0:2].contiguous().view(torch.float16).float()  # [blocks, 1]
        if self._emb_type == GGML_Q8_0:
            q = row[:, 2:].contiguous().view(torch.int8).float()
        else:
            b = row[:, 2:].to(torch.int32)
            q = torch.cat([b & 0x0F, b >> 4], dim=1).float() - 8.0
        return (q * scale).reshape(H)

    # ---- the step ----------------------------------------------------------
    def forward_token(self, token: int, position: int):
        import torch
        with torch.cuda.stream(self._stream):
            return self._forward(token, position)

    def _forward(self, token: int, position: int):
        import torch
        d = self.dims
        H, F, L = d["hidden"], d["ffn"], d["layers"]
        heads, kvh, hd = d["heads"], d["kv_heads"], d["head_dim"]
        if not 0 <= token < d["vocab"]:
            raise ValueError("token outside the vocabulary")
        if position >= self.context_tokens:
            raise ValueError("position beyond context_tokens")
        n = self.cache.length(0)
        if position > n:
            raise ValueError("positions must follow one another")
        if position < n:
            self.cache.truncate(0, position)
        eng = self.engine
        self.x.copy_(self._embed(token))
        for layer, w in enumerate(self.layers):
            nrm = self._rmsnorm(self.x, w["attn_norm"])
            eng.matvec_gguf(w["q_qkv"], w["qkv"], H + 2 * self.kv, H, nrm, self._qkv)
            q = self._qkv[:H].view(1, 1, heads, hd)
            k = self._qkv[H:H + self.kv].view(1, 1, kvh, hd)
            v = self._qkv[H + self.kv:].view(1, 1, kvh, hd)
            flags = TE_ATTN_QKV_BIAS | (TE_ATTN_ADVANCE if layer == L - 1 else 0)
            self.cache.decode(layer, 1, [0], q, self._attn.view(1, 1, heads, hd), heads, k_new=k, v_new=v,
                              flags=flags)
            eng.matvec_gguf(w["q_o"], w["o"], H, H, self._attn, self.x, flags=TE_ATTN_ACCUMULATE)
            nrm = self._rmsnorm(self.x, w["ffn_norm"])
            eng.matvec_gguf(w["q_gu"], w["gu"], 2 * F, H, nrm, self._gu)
            g, u = self._gu[:F], self._gu[F:]
            s = (g / (1.0 + torch.exp(-g))) * u
            eng.matvec_gguf(w["q_down"], w["down"], H, F, s, self.x, flags=TE_ATTN_ACCUMULATE)
        return self.x

    def project_next(self) -> int:
        import torch
        d = self.dims
        with torch.cuda.stream(self._stream):
            nrm = self._rmsnorm(self.x, self._out_norm)
            self.engine.matvec_gguf(self._q_head, self._head, d["vocab"], d["hidden"], nrm, self.logits)
            best = torch.argmax(self.logits)
        return int(best.item())

    def close(self) -> None:
        if getattr(self, "cache", None) is not None:
            self.cache.close()
            self.cache = None
