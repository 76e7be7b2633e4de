"""Qwen2 decode step on one GPU: the layer-step integration.

Mirrors the reference's per-token forward pass, te_qwen_forward_token
(c/src/qwen.c:907-1112), and its greedy projection, te_qwen_project_next
(:1303-1377), on a GGUF model, with five launches of this library per layer:

  q|k|v = W_qkv RMSNorm(x)   te_matvec_gguf_fused (TE_ATTN_RMSNORM_INPUT) over
                             the q, k and v rows stacked (they share the input)
  bias + RoPE + f16 append + GQA decode
                             one te_attention_decode launch (TE_ATTN_QKV_BIAS:
                             the biases added in fp32 inside it, :998-1011)
  x += W_o attn              te_matvec_gguf + TE_ATTN_ACCUMULATE
  g|u = W_gate|up RMSNorm(x) te_matvec_gguf_fused (RMSNorm), rows stacked
  x += W_down SwiGLU(g, u)   te_matvec_gguf_fused (TE_ATTN_SWIGLU_INPUT +
                             TE_ATTN_ACCUMULATE)

and for the head logits = W_out RMSNorm(x) (one fused launch) and the argmax
(first maximum, as te_argmax_f32).  The embedding table is dequantised once
into fp32 in HBM (q * scale, exact), so a token's row is a copy.

One difference from the reference's CPU pass is by design: the KV cache is
the engine's f16 cache (the reference's Metal path's layout), where the CPU
pass keeps fp32 keys and values, so outputs agree to f16 rounding of K/V, not
bit for bit.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

from .gguf import GGML_F32, GGML_Q4_0, GGML_Q8_0, GGUFError, GGUFFile
from .runtime import (TE_ATTN_ACCUMULATE, TE_ATTN_ADVANCE, TE_ATTN_QKV_BIAS, TE_ATTN_RMSNORM_INPUT,
                      TE_ATTN_STEP_HEAD, TE_ATTN_SWIGLU_INPUT, AttnEngine, QwenStep)

_QUANT = {GGML_Q4_0: 4, GGML_Q8_0: 8}  # ggml type -> TE_ATTN_QUANT_GGUF_*


class QwenDecoder:
    """One sequence of a qwen2 GGUF model on the engine's device.

    forward_token(token, position) runs every layer for one token (the token
    at `position` of the sequence; positions must follow one another from 0,
    or restart below the current length, which truncates the cache there) and
    returns the hidden state (a device tensor [hidden]); project_next()
    returns the greedy next token and leaves the logits in `self.logits`.
    Work runs on the engine's stream; before returning, both make the
    caller's current stream wait for it, so the results can be used there.

    With fused_step (the default) a decode token runs as ONE launch of the
    library's whole-token step kernel (te_qwen_step_run: every layer, and in
    recorded greedy steps the head and argmax too) instead of five launches
    per layer; the per-op path (fused_step=False) stays available and is what
    prefill_prompt uses.  The fused step needs the same quantisation for a
    projection in every layer; otherwise the decoder takes the per-op path.
    """

    def __init__(self, engine: AttnEngine, model: str | Path | GGUFFile, context_tokens: int,
                 fused_step: bool = True):
        import torch

        self._want_step = fused_step
        self.engine = engine
        self._owns_gguf = not isinstance(model, GGUFFile)
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
        self._emb = self._dequant_table(raw("token_embd.weight"), emb.ggml_type, d["vocab"], H)
        head = "output.weight" if "output.weight" in t else "token_embd.weight"
        self._head = raw(head)
        self._q_head = quant_of(head)
        self._out_norm = f32("output_norm.weight", H)

        self.cache = self.engine.kv_cache(layers=L, max_seqs=1, max_tokens_per_seq=self.context_tokens,
                                          kv_heads=kvh, head_dim=hd, max_position=self.context_tokens,
                                          rope_theta=d["rope_base"])
        self.cache.set_qkv_bias(0, heads, qb, kb, vb)
        self._step = None
        quants = {k: {w["q_" + k] for w in self.layers} for k in ("qkv", "o", "gu", "down")}
        if self._want_step and all(len(v) == 1 for v in quants.values()):
            self._norms = (torch.stack([w["attn_norm"] for w in self.layers]).contiguous(),
                           torch.stack([w["ffn_norm"] for w in self.layers]).contiguous())
            self._step = QwenStep(
                self.cache, layers=L, hidden=H, heads=heads, ffn=F, vocab=d["vocab"], eps=d["eps"],
                quants={**{k: next(iter(v)) for k, v in quants.items()}, "head": self._q_head},
                w_qkv=[w["qkv"] for w in self.layers], w_o=[w["o"] for w in self.layers],
                w_gu=[w["gu"] for w in self.layers], w_down=[w["down"] for w in self.layers], w_head=self._head,
                attn_norm=self._norms[0], ffn_norm=self._norms[1], out_norm=self._out_norm, embedding=self._emb)
        self._tok = torch.zeros(1, dtype=torch.int64, device=dev)
        self.x = torch.zeros(H, dtype=torch.float32, device=dev)
        self._qkv = torch.empty(H + 2 * self.kv, dtype=torch.float32, device=dev)
        self._attn = torch.empty(H, dtype=torch.float32, device=dev)
        self._gu = torch.empty(2 * F, dtype=torch.float32, device=dev)
        self.logits = torch.empty(d["vocab"], dtype=torch.float32, device=dev)

    # ---- embedding table ----------------------------------------------------
    @staticmethod
    def _dequant_table(raw, ggml_type, rows, cols):
        """[rows][cols] fp32 from GGUF bytes, as te_model_dequantize_row_f32:
        q * scale (Q8_0), (q - 8) * scale (Q4_0; low nibbles are weights 0-15
        of a block, high nibbles 16-31) -- exact products in fp32."""
        import torch
        if ggml_type == GGML_F32:
            return raw.view(torch.float32).view(rows, cols).clone()
        width = 34 if ggml_type == GGML_Q8_0 else 18
        blocks = raw.view(rows, cols // 32, width)
        out = torch.empty((rows, cols), dtype=torch.float32, device=raw.device)
        step = 8192
        for r0 in range(0, rows, step):
            b = blocks[r0:r0 + step]
            scale = b[:, :, 0:2].contiguous().view(torch.float16).float()  # [n, blocks, 1]
            if ggml_type == GGML_Q8_0:
                q = b[:, :, 2:].contiguous().view(torch.int8).float()
            else:
                c = b[:, :, 2:].to(torch.int32)
                q = torch.cat([c & 0x0F, c >> 4], dim=2).float() - 8.0
            out[r0:r0 + step] = (q * scale).reshape(-1, cols)
        return out

    def _embed(self, token):
        """The token's fp32 row; token is an int or a one-element device tensor
        (the graph-captured steps read it from device memory)."""
        return self._emb[token] if isinstance(token, int) else self._emb.index_select(0, token)[0]

    @property
    def fused_step(self) -> bool:
        """True when decode tokens run as one te_qwen_step_run launch."""
        return self._step is not None

    # ---- the step ----------------------------------------------------------
    def forward_token(self, token: int, position: int):
        import torch
        with torch.cuda.stream(self._stream):
            x = self._forward(token, position)
        # the caller's stream sees x only after the engine's stream wrote it
        torch.cuda.current_stream(self._dev).wait_stream(self._stream)
        return x

    def _forward(self, token: int, position: int, next_token=None):
        """Every layer for one token; with next_token (a one-element int64
        device tensor, fused step only) also the head, the logits in
        self.logits and the greedy choice in next_token."""
        import torch
        d = self.dims
        H, F, L = d["hidden"], d["ffn"], d["layers"]
        heads, kvh, hd = d["heads"], d["kv_heads"], d["head_dim"]
        if isinstance(token, int) and not 0 <= token < d["vocab"]:
            raise ValueError("token outside the vocabulary")
        if position >= self.context_tokens:
            raise ValueError("position beyond context_tokens")
        n = self.cache.length(0)
        if position > n:
            raise ValueError("positions must follow one another")
        if position < n:
            self.cache.truncate(0, position)
        eng = self.engine
        eps = d["eps"]
        if self._step is not None:
            if isinstance(token, int):
                self._tok.fill_(token)
                token = self._tok
            flags = TE_ATTN_QKV_BIAS | TE_ATTN_ADVANCE
            if next_token is not None:
                self._step.run(0, token, self.x, self.logits, next_token, flags | TE_ATTN_STEP_HEAD)
            else:
                self._step.run(0, token, self.x, flags=flags)
            return self.x
        self.x.copy_(self._embed(token))
        for layer, w in enumerate(self.layers):
            eng.matvec_gguf_fused(w["q_qkv"], w["qkv"], H + 2 * self.kv, H, self.x, self._qkv, TE_ATTN_RMSNORM_INPUT,
                                  w["attn_norm"], eps)
            q = self._qkv[:H].view(1, 1, heads, hd)
            k = self._qkv[H:H + self.kv].view(1, 1, kvh, hd)
            v = self._qkv[H + self.kv:].view(1, 1, kvh, hd)
            flags = TE_ATTN_QKV_BIAS | (TE_ATTN_ADVANCE if layer == L - 1 else 0)
            self.cache.decode(layer, 1, [0], q, self._attn.view(1, 1, heads, hd), heads, k_new=k, v_new=v,
                              flags=flags)
            eng.matvec_gguf(w["q_o"], w["o"], H, H, self._attn, self.x, flags=TE_ATTN_ACCUMULATE)
            eng.matvec_gguf_fused(w["q_gu"], w["gu"], 2 * F, H, self.x, self._gu, TE_ATTN_RMSNORM_INPUT,
                                  w["ffn_norm"], eps)
            eng.matvec_gguf_fused(w["q_down"], w["down"], H, F, self._gu, self.x,
                                  TE_ATTN_SWIGLU_INPUT | TE_ATTN_ACCUMULATE)
        return self.x

    # ---- a whole prompt at once -----------------------------------------------
    def prefill_prompt(self, tokens, position: int = 0):
        """The prompt's tokens at positions position .. position + T - 1, every
        layer once for all T (the reference's batched prompt pass,
        te_qwen_prefill_prompt_batch, qwen.c:630-906): projections of up to 8
        tokens per launch (te_matvec_gguf_fused / te_matvec_gguf with
        n_vectors), one te_attention_prefill launch per layer (bias, RoPE, f16
        append and causal attention over the cache; head_dim 64 or 128).
        Returns the last token's hidden state, like forward_token."""
        import torch
        toks = [int(t) for t in tokens]
        d = self.dims
        if not toks:
            raise ValueError("empty prompt")
        if any(not 0 <= t < d["vocab"] for t in toks):
            raise ValueError("token outside the vocabulary")
        if position + len(toks) > self.context_tokens:
            raise ValueError("prompt beyond context_tokens")
        n = self.cache.length(0)
        if position > n:
            raise ValueError("positions must follow one another")
        if position < n:
            self.cache.truncate(0, position)
        with torch.cuda.stream(self._stream):
            self._prefill(toks)
        torch.cuda.current_stream(self._dev).wait_stream(self._stream)
        return self.x

    def _prefill(self, toks) -> None:
        import torch
        d = self.dims
        H, F, L = d["hidden"], d["ffn"], d["layers"]
        heads, kv, eps = d["heads"], self.kv, d["eps"]
        T = len(toks)
        eng = self.engine
        idx = torch.tensor(toks, dtype=torch.int64).to(self._dev, non_blocking=True)
        X = self._emb.index_select(0, idx)  # [T][H], the residual stream of every token
        qkv = torch.empty((T, H + 2 * kv), dtype=torch.float32, device=self._dev)
        attn = torch.empty((T, H), dtype=torch.float32, device=self._dev)
        gu = torch.empty((T, 2 * F), dtype=torch.float32, device=self._dev)
        chunks = [(c, min(8, T - c)) for c in range(0, T, 8)]
        for layer, w in enumerate(self.layers):
            for c, m in chunks:
                eng.matvec_gguf_fused(w["q_qkv"], w["qkv"], H + 2 * kv, H, X[c:c + m], qkv[c:c + m],
                                      TE_ATTN_RMSNORM_INPUT, w["attn_norm"], eps, n_vectors=m)
            q = qkv[:, :H].contiguous()
            k = qkv[:, H:H + kv].contiguous()
            v = qkv[:, H + kv:].contiguous()
            flags = TE_ATTN_QKV_BIAS | (TE_ATTN_ADVANCE if layer == L - 1 else 0)
            self.cache.prefill(layer, 1, 0, q, k, v, T, heads, attn, flags)
            for c, m in chunks:
                eng.matvec_gguf(w["q_o"], w["o"], H, H, attn[c:c + m], X[c:c + m], n_vectors=m,
                                flags=TE_ATTN_ACCUMULATE)
            for c, m in chunks:
                eng.matvec_gguf_fused(w["q_gu"], w["gu"], 2 * F, H, X[c:c + m], gu[c:c + m],
                                      TE_ATTN_RMSNORM_INPUT, w["ffn_norm"], eps, n_vectors=m)
            for c, m in chunks:
                eng.matvec_gguf_fused(w["q_down"], w["down"], H, F, gu[c:c + m], X[c:c + m],
                                      TE_ATTN_SWIGLU_INPUT | TE_ATTN_ACCUMULATE, n_vectors=m)
        self.x.copy_(X[T - 1])

    def project_next(self) -> int:
        import torch
        d = self.dims
        with torch.cuda.stream(self._stream):
            self._head_logits()
            best = int(torch.argmax(self.logits).item())  # read back in the engine stream's order
        torch.cuda.current_stream(self._dev).wait_stream(self._stream)
        return best

    def _head_logits(self) -> None:
        d = self.dims
        self.engine.matvec_gguf_fused(self._q_head, self._head, d["vocab"], d["hidden"], self.x, self.logits,
                                      TE_ATTN_RMSNORM_INPUT, self._out_norm, d["eps"])

    # ---- many steps as one CUDA graph ----------------------------------------
    def capture_greedy(self, start_position: int, n_steps: int) -> None:
        """Record n_steps greedy decode steps as one CUDA graph.  Step i reads
        its token from the device tensor self.tokens[i], runs every layer at
        position start_position + i and writes the argmax of its logits to
        self.tokens[i + 1]: no host work between steps.  The sequence must
        already hold start_position tokens.  Every position of the window is
        first run eagerly once (mapping its cache pages and sizing the
        engine's scratch, so that nothing is allocated while recording); the
        graph's kernel arguments fix the positions, so each replay restarts
        at start_position.  Afterwards the cache's length counts the window."""
        import torch
        if n_steps < 1 or start_position + n_steps > self.context_tokens:
            raise ValueError("window beyond context_tokens")
        if self.cache.length(0) < start_position:
            raise ValueError("the sequence does not hold start_position tokens yet")
        self.cache.reserve(0, start_position + n_steps)
        for i in range(n_steps):  # eager pass over the window
            self.forward_token(0, start_position + i)
        self.project_next()
        with torch.cuda.stream(self._stream):
            self.tokens = torch.zeros(n_steps + 1, dtype=torch.int64, device=self._dev)
        self._stream.synchronize()
        self.cache.truncate(0, start_position)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=self._stream):
            for i in range(n_steps):
                if self._step is not None:  # one launch per token: layers, head and argmax
                    self._forward(self.tokens[i:i + 1], start_position + i, next_token=self.tokens[i + 1:i + 2])
                    continue
                self._forward(self.tokens[i:i + 1], start_position + i)
                self._head_logits()
                self.tokens[i + 1:i + 2].copy_(torch.argmax(self.logits).reshape(1))
        self._graph = graph
        self._graph_window = (start_position, n_steps)

    def replay_greedy(self, first_token: int):
        """Run the captured window from its start with first_token as the token
        at start_position; returns self.tokens (device; tokens[1:] are the
        greedy choices), ordered before the caller's stream.  The recording
        already counted the window in the cache's length, and each replay
        rewrites those positions, so eager steps may follow a replay at
        start_position + n_steps; a cache changed since the recording (other
        steps, a truncation) is refused."""
        import torch
        if getattr(self, "_graph", None) is None:
            raise RuntimeError("capture_greedy first")
        if not 0 <= first_token < self.dims["vocab"]:
            raise ValueError("token outside the vocabulary")
        start, n = self._graph_window
        if self.cache.length(0) != start + n:
            raise RuntimeError("the cache changed since the capture; capture again")
        with torch.cuda.stream(self._stream):
            self.tokens[0:1].fill_(first_token)
            self._graph.replay()
        torch.cuda.current_stream(self._dev).wait_stream(self._stream)
        return self.tokens

    def close(self) -> None:
        """Releases the cache, the device weights and (when this decoder opened
        it) the GGUF mapping; pending work on the engine's stream completes first."""
        if getattr(self, "_stream", None) is not None:
            self._stream.synchronize()
        self._graph = None
        if getattr(self, "_step", None) is not None:
            self._step.close()
            self._step = None
        if getattr(self, "cache", None) is not None:
            self.cache.close()
            self.cache = None
        self.layers = []
        self._emb = self._head = self._out_norm = None
        if getattr(self, "_owns_gguf", False) and self.gguf is not None:
            self.gguf.close()
            self.gguf = None
