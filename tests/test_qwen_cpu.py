"""Host side of the layer-step integration, on CPU.

The GGUF reader (tinymetalagent_b200/gguf.py) against the reference's own
parser (c/src/gguf.c te_parse_gguf / te_extract_model_info, built into
oracle/_ref/libteqwen.so) on a synthetic qwen2 file, and the reference's
forward pass on that file (the checker the GPU parity test uses): it loads,
runs, and is deterministic.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from gguf_synth import GGML_Q4_0, GGML_Q8_0, write_qwen2  # noqa: E402


def test_gguf_reader_dims_and_tensors(tmp_path):
    from tinymetalagent_b200.gguf import GGUFFile
    want = write_qwen2(tmp_path / "m.gguf", layers=3, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=320)
    g = GGUFFile(tmp_path / "m.gguf")
    d = g.qwen2_dims()
    for k in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ffn", "vocab", "context"):
        assert d[k] == want[k], k
    assert abs(d["eps"] - 1e-6) < 1e-12 and d["rope_base"] == 1e6
    q = g.tensors["blk.1.attn_q.weight"]
    assert q.ggml_type == GGML_Q8_0 and q.dims == (256, 256) and q.nbytes == 256 * 8 * 34
    down = g.tensors["blk.2.ffn_down.weight"]
    assert down.ggml_type == GGML_Q4_0 and down.dims == (512, 256) and down.nbytes == 256 * 16 * 18
    assert g.tensors["blk.0.attn_k.bias"].data.view(np.float32).shape == (128,)
    g.close()


def test_gguf_reader_rejects_bad_files(tmp_path):
    from tinymetalagent_b200.gguf import GGUFError, GGUFFile
    (tmp_path / "bad.gguf").write_bytes(b"GGUX" + bytes(28))
    with pytest.raises(GGUFError):
        GGUFFile(tmp_path / "bad.gguf")
    write_qwen2(tmp_path / "m.gguf")
    data = (tmp_path / "m.gguf").read_bytes()
    (tmp_path / "cut.gguf").write_bytes(data[: len(data) // 2])
    with pytest.raises(GGUFError):
        GGUFFile(tmp_path / "cut.gguf")


def test_reference_forward_on_synthetic_model(tmp_path):
    from oracle import oracle as O
    if not O.ref_qwen_available():
        pytest.skip("reference forward pass not built (its sources were absent at build time)")
    from tinymetalagent_b200.gguf import GGUFFile
    write_qwen2(tmp_path / "m.gguf")
    d = GGUFFile(tmp_path / "m.gguf").qwen2_dims()
    runs = []
    for _ in range(2):
        r = O.RefQwen(tmp_path / "m.gguf", 32)
        for k in ("hidden", "ffn", "layers", "heads", "kv_heads", "head_dim", "vocab"):
            assert r.dims[k] == d[k], k
        hs, toks = [], []
        tok = 3
        for pos in range(5):
            hs.append(r.forward(tok, pos))
            _, tok = r.project()
            toks.append(tok)
        r.close()
        runs.append((np.stack(hs), toks))
    assert np.isfinite(runs[0][0]).all() and 0.3 < float(runs[0][0].std()) < 10
    assert np.array_equal(runs[0][0], runs[1][0]) and runs[0][1] == runs[1][1]


@pytest.mark.parametrize("variant", [dict(tokenizer=True), dict(alignment=64), dict(version=2, alignment=128),
                                     dict(tokenizer=True, tied=True, alignment=256)])
def test_gguf_reader_matches_reference_parser(tmp_path, variant):
    """Files with tokenizer arrays (strings, int32), a general.alignment, GGUF v2, tied embeddings: the reader
    and the reference's own parser (te_model_parse_gguf + te_qwen_state_init) agree on every dimension, and
    the bytes of a tensor the reader returns are the ones the writer put there."""
    from tinymetalagent_b200.gguf import GGUFFile
    want = write_qwen2(tmp_path / "m.gguf", vocab=320, **variant)
    g = GGUFFile(tmp_path / "m.gguf")
    d = g.qwen2_dims()
    assert d["vocab"] == 320 and d["hidden"] == want["hidden"] and d["layers"] == want["layers"]
    if variant.get("tokenizer"):
        toks = g.metadata["tokenizer.ggml.tokens"]
        assert len(toks) == 320 and toks[5] == "tok5"
        assert g.metadata["tokenizer.ggml.token_type"].dtype == np.int32
    if variant.get("alignment"):
        assert all(t.offset % variant["alignment"] == 0 for t in g.tensors.values())
    assert ("output.weight" in g.tensors) == (not variant.get("tied"))
    from oracle import oracle as O
    if O.ref_qwen_available():
        r = O.RefQwen(tmp_path / "m.gguf", 16)
        for k in ("hidden", "ffn", "layers", "heads", "kv_heads", "head_dim", "vocab"):
            assert r.dims[k] == d[k], k
        h = r.forward(3, 0)
        assert np.isfinite(h).all()
        r.close()
    g.close()
