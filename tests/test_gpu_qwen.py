"""GPU parity of the layer-step integration (tinymetalagent_b200/qwen.py).

The oracle is the reference's own CPU forward pass (c/src/qwen.c
te_qwen_forward_token :907-1112 and te_qwen_project_next :1303-1377, built
from its sources into oracle/_ref/libteqwen.so) on the same synthetic qwen2
GGUF file.  The reference keeps fp32 keys and values where the engine keeps
f16 (its Metal path's cache), and sums in another order, so hidden states
agree to f16 rounding of K/V carried through the layers: the bar is
|h - ref| <= 2e-2 + 2e-2 |ref| per element (hidden values are O(1); the
measured worst differences over 48 positions are 5.5e-4 and 1.2e-3), logits
within 5e-2 + 2e-2 |ref|, and the greedy tokens equal at every step (the test
also checks that each step's top-two logit margin in the reference exceeds
0.1, so equality is the expected outcome, not luck).
"""
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from gguf_synth import GGML_Q4_0, GGML_Q8_0, write_qwen2  # noqa: E402

MODELS = {
    # hidden 256, 4 heads of 64, 2 KV heads; Q8_0 attention, Q4_0 MLP
    "hd64": dict(layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=512, quant_attn=GGML_Q8_0,
                 quant_ffn=GGML_Q4_0, seed=11),
    # hidden 512, 4 heads of 128, 1 KV head (group 4); Q4_0 attention, Q8_0 MLP
    "hd128": dict(layers=3, hidden=512, heads=4, kv_heads=1, ffn=1024, vocab=640, quant_attn=GGML_Q4_0,
                  quant_ffn=GGML_Q8_0, seed=12),
    # tied embeddings: no output.weight, the lm_head is token_embd.weight; 7 query heads per KV head
    "tied": dict(layers=2, hidden=448, heads=7, kv_heads=1, ffn=640, vocab=384, quant_attn=GGML_Q8_0,
                 quant_ffn=GGML_Q4_0, seed=13, tied=True),
}


def close(got, ref, atol, rtol, what):
    err = np.abs(got - ref) - (atol + rtol * np.abs(ref))
    assert err.max() <= 0, f"{what}: max excess {err.max():.3e}, max abs diff {np.abs(got - ref).max():.3e}"


def margin(logits):
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0])


@pytest.mark.parametrize("fused", [True, False], ids=["step", "per_op"])
@pytest.mark.parametrize("name", list(MODELS))
def test_decode_steps_match_reference(tmp_path, name, fused):
    from oracle import oracle as O
    if not O.ref_qwen_available():
        pytest.skip("reference forward pass not built")
    from tinymetalagent_b200 import AttnEngine
    from tinymetalagent_b200.qwen import QwenDecoder
    path = tmp_path / f"{name}.gguf"
    write_qwen2(path, **MODELS[name])
    ctx = 48
    ref = O.RefQwen(path, ctx)
    eng = AttnEngine(0)
    dec = QwenDecoder(eng, path, ctx, fused_step=fused)
    assert dec.fused_step == fused
    try:
        vocab = ref.dims["vocab"]
        rng = np.random.default_rng(5)
        # teacher-forced prompt: both sides see the same tokens
        prompt = rng.integers(0, vocab, 20)
        worst = 0.0
        for pos, tok in enumerate(prompt):
            h_ref = ref.forward(int(tok), pos)
            h = dec.forward_token(int(tok), pos).cpu().numpy()
            close(h, h_ref, 2e-2, 2e-2, f"hidden at position {pos}")
            worst = max(worst, float(np.abs(h - h_ref).max()))
        # greedy continuation: each side feeds its own choice
        tok_ref = tok_gpu = None
        for pos in range(len(prompt), ctx):
            logits_ref, tok_ref = ref.project()
            tok_gpu = dec.project_next()
            close(dec.logits.cpu().numpy(), logits_ref, 5e-2, 2e-2, f"logits after position {pos - 1}")
            assert margin(logits_ref) > 0.1, "synthetic model gave an ambiguous greedy step"
            assert tok_gpu == tok_ref, f"greedy token at position {pos}"
            h_ref = ref.forward(tok_ref, pos)
            h = dec.forward_token(tok_gpu, pos).cpu().numpy()
            close(h, h_ref, 2e-2, 2e-2, f"hidden at position {pos}")
            worst = max(worst, float(np.abs(h - h_ref).max()))
        print(f"{name}: worst hidden abs diff {worst:.3e}")
        # restart below the current length: the cache is truncated there
        h_ref = ref.forward(7, 10)
        h = dec.forward_token(7, 10).cpu().numpy()
        close(h, h_ref, 2e-2, 2e-2, "hidden after restarting at position 10")
    finally:
        dec.close()
        eng.close()
        ref.close()


def test_decoder_rejects_gaps_and_bad_tokens(tmp_path):
    from tinymetalagent_b200 import AttnEngine
    from tinymetalagent_b200.qwen import QwenDecoder
    path = tmp_path / "m.gguf"
    write_qwen2(path, **MODELS["hd64"])
    eng = AttnEngine(0)
    dec = QwenDecoder(eng, path, 16)
    try:
        with pytest.raises(ValueError):
            dec.forward_token(1, 3)     # position 3 before positions 0..2
        with pytest.raises(ValueError):
            dec.forward_token(10 ** 6, 0)  # outside the vocabulary
        with pytest.raises(ValueError):
            dec.forward_token(1, 16)    # beyond the context
    finally:
        dec.close()
        eng.close()


@pytest.mark.parametrize("fused", [True, False], ids=["step", "per_op"])
def test_graph_replay_matches_eager_steps(tmp_path, fused):
    """capture_greedy / replay_greedy: the same kernels as the eager steps, recorded once; the tokens and
    the final hidden state equal the eager run's, replaying twice gives the same tokens, and eager steps
    continue after a replay."""
    import torch
    from tinymetalagent_b200 import AttnEngine
    from tinymetalagent_b200.qwen import QwenDecoder
    path = tmp_path / "m.gguf"
    write_qwen2(path, **MODELS["hd64"])
    prompt = [int(t) for t in np.random.default_rng(8).integers(0, 512, 12)]
    n = 16
    eng = AttnEngine(0)
    try:
        eager = QwenDecoder(eng, path, 40, fused_step=fused)
        for pos, t in enumerate(prompt):
            eager.forward_token(t, pos)
        first = eager.project_next()
        toks, tok = [], first
        for i in range(n):
            eager.forward_token(tok, len(prompt) + i)
            tok = eager.project_next()
            toks.append(tok)
        h_eager = eager.x.cpu().numpy()
        after = eager.forward_token(tok, len(prompt) + n).cpu().numpy()
        eager.close()

        g = QwenDecoder(eng, path, 40, fused_step=fused)
        for pos, t in enumerate(prompt):
            g.forward_token(t, pos)
        assert g.project_next() == first
        g.capture_greedy(len(prompt), n)
        for _ in range(2):
            got = g.replay_greedy(first).cpu().numpy()
            assert got[0] == first and got[1:].tolist() == toks
            np.testing.assert_allclose(g.x.cpu().numpy(), h_eager, rtol=0, atol=1e-6)
        np.testing.assert_allclose(g.forward_token(tok, len(prompt) + n).cpu().numpy(), after, rtol=0, atol=1e-6)
        with pytest.raises(RuntimeError):
            g.replay_greedy(first)  # the cache moved on since the capture
        g.close()
        torch.cuda.synchronize()
    finally:
        eng.close()


@pytest.mark.parametrize("name", list(MODELS))
def test_prefill_prompt_matches_reference(tmp_path, name):
    """prefill_prompt (batched projections + one te_attention_prefill launch per layer; head_dim 64 and 128,
    groups 2, 4 and 7) against the reference's token-by-token forward pass; then greedy steps continue from
    the prefilled cache, and a prompt prefilled in two calls (the second over the first's cache) gives the
    same state."""
    from oracle import oracle as O
    if not O.ref_qwen_available():
        pytest.skip("reference forward pass not built")
    from tinymetalagent_b200 import AttnEngine
    from tinymetalagent_b200.qwen import QwenDecoder
    path = tmp_path / "m.gguf"
    write_qwen2(path, **MODELS[name])
    prompt = [int(t) for t in np.random.default_rng(21).integers(0, MODELS[name]["vocab"], 21)]
    ctx = 40
    ref = O.RefQwen(path, ctx)
    eng = AttnEngine(0)
    try:
        for pos, t in enumerate(prompt):
            h_ref = ref.forward(t, pos)
        dec = QwenDecoder(eng, path, ctx)
        h = dec.prefill_prompt(prompt).cpu().numpy()
        close(h, h_ref, 2e-2, 2e-2, "hidden after the prompt")
        for pos in range(len(prompt), len(prompt) + 8):
            logits_ref, tok_ref = ref.project()
            tok = dec.project_next()
            close(dec.logits.cpu().numpy(), logits_ref, 5e-2, 2e-2, f"logits after position {pos - 1}")
            assert margin(logits_ref) > 0.1 and tok == tok_ref, f"greedy token at position {pos}"
            h_ref = ref.forward(tok_ref, pos)
            close(dec.forward_token(tok, pos).cpu().numpy(), h_ref, 2e-2, 2e-2, f"hidden at position {pos}")
        dec.close()

        two = QwenDecoder(eng, path, ctx)
        two.prefill_prompt(prompt[:12])
        h2 = two.prefill_prompt(prompt[12:], position=12).cpu().numpy()
        np.testing.assert_allclose(h2, h, rtol=2e-3, atol=2e-3)
        two.close()
    finally:
        eng.close()
        ref.close()
