"""GPU tests of the whole-token decode step (te_qwen_step_*, csrc/k_step.cu).

The step kernel runs te_qwen_forward_token (c/src/qwen.c:907-1112) for every
layer of a token, and optionally te_qwen_project_next (:1303-1377), in one
cooperative launch.  Parity is checked against the reference's own CPU
forward pass (oracle/_ref/libteqwen.so) and against this library's per-op
path (five launches per layer) on synthetic qwen2 GGUF models:
  * contexts beyond one 256-token attention chunk, so that several CTAs
    share a kv head's tokens and the last one merges their records;
  * one library launch per token, with the head and argmax in the same
    launch when recorded as greedy steps;
  * a token outside the vocabulary on the device: the kernel reports it
    through the engine's error word (no fault), and the next step runs.
Bars as in test_gpu_qwen.py: hidden |h - ref| <= 2e-2 + 2e-2 |ref| against
the reference (f16 K/V against its fp32 ones), and 2e-3 + 2e-3 |h| against
the per-op path (same f16 cache, sums in another order).
"""
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from gguf_synth import GGML_Q4_0, GGML_Q8_0, write_qwen2  # noqa: E402

LONG = dict(layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=512, quant_attn=GGML_Q8_0,
            quant_ffn=GGML_Q4_0, seed=31)
LONG128 = dict(layers=2, hidden=512, heads=8, kv_heads=2, ffn=768, vocab=384, quant_attn=GGML_Q4_0,
               quant_ffn=GGML_Q8_0, seed=32)


def close(got, ref, atol, rtol, what):
    err = np.abs(got - ref) - (atol + rtol * np.abs(ref))
    assert err.max() <= 0, f"{what}: max excess {err.max():.3e}, max abs diff {np.abs(got - ref).max():.3e}"


@pytest.mark.parametrize("spec", [LONG, LONG128], ids=["hd64", "hd128"])
def test_long_context_matches_reference_and_per_op(tmp_path, spec):
    """700 teacher-forced tokens (three attention chunks per kv head), then greedy steps."""
    from oracle import oracle as O
    if not O.ref_qwen_available():
        pytest.skip("reference forward pass not built")
    from tinymetalagent_b200 import AttnEngine
    from tinymetalagent_b200.qwen import QwenDecoder
    path = tmp_path / "m.gguf"
    write_qwen2(path, **spec)
    ctx = 720
    ref = O.RefQwen(path, ctx)
    eng = AttnEngine(0)
    step = QwenDecoder(eng, path, ctx)
    per_op = QwenDecoder(eng, path, ctx, fused_step=False)
    assert step.fused_step and not per_op.fused_step
    try:
        toks = np.random.default_rng(3).integers(0, spec["vocab"], 700)
        for pos, t in enumerate(toks):
            h_ref = ref.forward(int(t), pos)
            h = step.forward_token(int(t), pos).cpu().numpy()
            h2 = per_op.forward_token(int(t), pos).cpu().numpy()
            if pos % 97 == 0 or pos in (255, 256, 257, 511, 512, 513) or pos >= 695:
                close(h, h_ref, 2e-2, 2e-2, f"hidden at position {pos} against the reference")
                close(h, h2, 2e-3, 2e-3, f"hidden at position {pos} against the per-op path")
        for pos in range(700, 708):
            logits_ref, tok_ref = ref.project()
            tok = step.project_next()
            close(step.logits.cpu().numpy(), logits_ref, 5e-2, 2e-2, f"logits after position {pos - 1}")
            assert tok == tok_ref, f"greedy token at position {pos}"
            h_ref = ref.forward(tok_ref, pos)
            close(step.forward_token(tok, pos).cpu().numpy(), h_ref, 2e-2, 2e-2, f"hidden at position {pos}")
    finally:
        step.close()
        per_op.close()
        eng.close()
        ref.close()


def test_one_launch_per_token_and_recorded_head(tmp_path):
    """forward_token is one library launch; a recorded greedy step (layers, head, argmax) is one launch
    too, and its tokens and logits equal the eager per-op head's."""
    import torch
    from tinymetalagent_b200 import AttnEngine
    from tinymetalagent_b200.qwen import QwenDecoder
    path = tmp_path / "m.gguf"
    write_qwen2(path, **LONG)
    eng = AttnEngine(0)
    try:
        dec = QwenDecoder(eng, path, 300)
        prompt = [int(t) for t in np.random.default_rng(4).integers(0, 512, 270)]
        n0 = eng.launch_count
        for pos, t in enumerate(prompt):
            dec.forward_token(t, pos)
        assert eng.launch_count - n0 == len(prompt)
        first = dec.project_next()
        logits_eager = dec.logits.cpu().numpy()
        toks, tok = [], first
        for i in range(6):
            dec.forward_token(tok, len(prompt) + i)
            tok = dec.project_next()
            toks.append(tok)
        dec.close()

        g = QwenDecoder(eng, path, 300)
        for pos, t in enumerate(prompt):
            g.forward_token(t, pos)
        assert g.project_next() == first
        np.testing.assert_allclose(g.logits.cpu().numpy(), logits_eager, rtol=0, atol=0)
        g.capture_greedy(len(prompt), 6)
        n0 = eng.launch_count
        got = g.replay_greedy(first).cpu().numpy()
        assert eng.launch_count == n0  # a replay issues no library call
        assert got[1:].tolist() == toks
        torch.cuda.synchronize()
        g.close()
    finally:
        eng.close()


def test_bad_device_token_sets_error_word(tmp_path):
    """A token id outside the vocabulary that reaches the kernel from device memory is reported by the
    next synchronisation as TE_STATUS_RUNTIME_ERROR; the engine and the decoder keep working."""
    import torch
    from tinymetalagent_b200 import AttnEngine, TinyEngineError
    from tinymetalagent_b200.qwen import QwenDecoder
    from tinymetalagent_b200.runtime import TE_ATTN_QKV_BIAS, TE_STATUS_RUNTIME_ERROR
    path = tmp_path / "m.gguf"
    write_qwen2(path, **LONG)
    eng = AttnEngine(0)
    try:
        dec = QwenDecoder(eng, path, 64)
        h0 = dec.forward_token(5, 0).cpu().numpy().copy()
        bad = torch.full((1,), 10 ** 6, dtype=torch.int64, device="cuda:0")
        dec._step.run(0, bad, dec.x, flags=TE_ATTN_QKV_BIAS)  # no advance: the cache length stays 1
        with pytest.raises(TinyEngineError) as ei:
            eng.synchronize()
        assert ei.value.status == TE_STATUS_RUNTIME_ERROR
        eng.synchronize()  # reported once
        ref = QwenDecoder(eng, path, 64, fused_step=False)
        ref.forward_token(5, 0)
        h1 = dec.forward_token(9, 1).cpu().numpy()
        r1 = ref.forward_token(9, 1).cpu().numpy()
        close(h1, r1, 2e-3, 2e-3, "step after the reported error")
        assert np.isfinite(h0).all()
        dec.close()
        ref.close()
    finally:
        eng.close()
