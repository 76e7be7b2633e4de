"""GPU parity of the GGUF Q4_0 / Q8_0 matrix-vector kernel (te_matvec_gguf).

Reference: te_model_matvec_f32's CPU row loop (c/src/ops.c:216-262, dot
products :584-620), restated in the oracle (pinned bit-for-bit to the
reference in tests/test_oracle.py).  The kernel forms the same products and
sums them in another order, so the bar is fp32 summation error:
|y - ref| <= 1e-5 * sum_c |w_rc x_c| + 1e-6.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from make_golden import quant_matrix  # noqa: E402

Q4, Q8 = 4, 8          # TE_ATTN_QUANT_GGUF_Q4_0 / _Q8_0
GGML = {Q4: 2, Q8: 8}  # ggml type ids of the fixture generator


def dequant(quant, w, rows, cols):
    blocks = cols // 32
    width = 18 if quant == Q4 else 34
    b = w.reshape(rows, blocks, width)
    scale = b[:, :, 0:2].copy().view(np.float16).astype(np.float32)[..., 0]
    if quant == Q4:
        qs = b[:, :, 2:]
        q = np.concatenate([(qs & 0x0F), (qs >> 4)], axis=2).astype(np.float32) - 8.0
    else:
        q = b[:, :, 2:].view(np.int8).astype(np.float32)
    return (q * scale[..., None]).reshape(rows, cols)


def check(port, quant, w, rows, cols, x, y):
    ref_fn = port.matvec_q4_0_f32 if quant == Q4 else port.matvec_q8_0_f32
    wd = np.abs(dequant(quant, w, rows, cols))
    for v in range(x.shape[0]):
        ref = ref_fn(w, rows, cols, x[v])
        bound = 1e-5 * (wd @ np.abs(x[v])) + 1e-6
        err = np.abs(y[v] - ref)
        assert (err <= bound).all(), (v, float(err.max()), float((err - bound).max()))


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("quant", [Q4, Q8])
@pytest.mark.parametrize("shape", [(1, 32, 1), (37, 896, 1), (300, 2048, 3), (4096, 2048, 1), (2048, 11008, 2),
                                   (5, 3584, 8), (129, 160, 5),
                                   # long rows: fewer rows per staged group, and (99 968 columns of
                                   # Q8_0) stages so large that one CTA per SM holds them
                                   (40, 29568, 3), (4, 99968, 1)])
def test_matvec_matches_oracle(port, quant, shape):
    import torch
    from tinymetalagent_b200 import AttnEngine
    rows, cols, nv = shape
    rng = np.random.default_rng(rows * 7 + cols + quant)
    w = quant_matrix(rng, GGML[quant], rows, cols)
    x = rng.standard_normal((nv, cols)).astype(np.float32)
    eng = AttnEngine(0)
    try:
        y = torch.full((nv, rows), float("nan"), dtype=torch.float32, device="cuda")
        eng.matvec_gguf(quant, dev(w), rows, cols, dev(x), y, nv)
        eng.synchronize()
        check(port, quant, w, rows, cols, x, y.cpu().numpy())
    finally:
        eng.close()


def test_matvec_golden_fixture(port):
    """The committed outputs of the reference's te_model_matvec_f32."""
    import torch
    from tinymetalagent_b200 import AttnEngine
    g = dict(np.load(Path(__file__).resolve().parent / "golden" / "golden_matvec.npz"))
    eng = AttnEngine(0)
    try:
        for i in range(4):
            ggml_type, rows, cols = (int(v) for v in g[f"mv{i}_meta"])
            quant = Q4 if ggml_type == 2 else Q8
            y = torch.zeros((1, rows), dtype=torch.float32, device="cuda")
            eng.matvec_gguf(quant, dev(g[f"mv{i}_w"]), rows, cols, dev(g[f"mv{i}_x"][None]), y, 1)
            eng.synchronize()
            wd = np.abs(dequant(quant, g[f"mv{i}_w"], rows, cols))
            bound = 1e-5 * (wd @ np.abs(g[f"mv{i}_x"])) + 1e-6
            assert (np.abs(y.cpu().numpy()[0] - g[f"mv{i}_out"]) <= bound).all()
    finally:
        eng.close()


def test_matvec_rejects_bad_arguments():
    import torch
    from tinymetalagent_b200 import AttnEngine, TinyEngineError
    eng = AttnEngine(0)
    try:
        w = torch.zeros(18 * 4 + 16, dtype=torch.uint8, device="cuda")
        x = torch.zeros((1, 64), dtype=torch.float32, device="cuda")
        y = torch.zeros((1, 2), dtype=torch.float32, device="cuda")
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf(Q4, w[2:], 2, 64, x, y)      # w not 16-byte aligned
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf(Q4, w, 2, 48, x, y)          # cols not a multiple of 32
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf(3, w, 2, 64, x, y)           # not Q4_0 / Q8_0
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf(Q4, w, 2, 64, x, y, 9)       # more than 8 vectors
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf(Q4, w, 2, 64, x, y, 1, 1 << 3)  # a flag other than TE_ATTN_ACCUMULATE
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf(Q8, w, 2, 110016, x, y)      # a row too long for two shared-memory stages
    finally:
        eng.close()


@pytest.mark.parametrize("quant", [Q4, Q8])
def test_matvec_residual_accumulate(port, quant):
    """Output projection + residual (c/src/qwen.c:1072-1079): y = residual + (W x), the add in fp32
    after the dot product."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ACCUMULATE, AttnEngine
    rows, cols, nv = 2048, 2048, 2
    rng = np.random.default_rng(99 + quant)
    w = quant_matrix(rng, GGML[quant], rows, cols)
    x = rng.standard_normal((nv, cols)).astype(np.float32)
    res = rng.standard_normal((nv, rows)).astype(np.float32)
    eng = AttnEngine(0)
    try:
        y = dev(res)
        eng.matvec_gguf(quant, dev(w), rows, cols, dev(x), y, nv, TE_ATTN_ACCUMULATE)
        eng.synchronize()
        got = y.cpu().numpy()
        ref_fn = port.matvec_q4_0_f32 if quant == Q4 else port.matvec_q8_0_f32
        wd = np.abs(dequant(quant, w, rows, cols))
        for v in range(nv):
            exp = (res[v] + ref_fn(w, rows, cols, x[v])).astype(np.float32)
            bound = 1e-5 * (wd @ np.abs(x[v])) + 1e-6 + 1e-7 * np.abs(exp)
            assert (np.abs(got[v] - exp) <= bound).all()
    finally:
        eng.close()


@pytest.mark.parametrize("quant", [Q4, Q8])
@pytest.mark.parametrize("shape", [(896 + 256, 896, 1), (4864 * 2, 896, 3), (300, 2048, 8), (7, 160, 2)])
def test_matvec_fused_rmsnorm_input(port, quant, shape):
    """te_matvec_gguf_fused + TE_ATTN_RMSNORM_INPUT: y[v] = W te_rmsnorm_f32(x[v], w_norm, eps) (c/src/ops.c:272-293:
    double sum of squares, fp32 scale, (x * scale) * w), one scale per vector."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_RMSNORM_INPUT, AttnEngine
    rows, cols, nv = shape
    rng = np.random.default_rng(rows + cols + quant + nv)
    w = quant_matrix(rng, GGML[quant], rows, cols)
    x = (rng.standard_normal((nv, cols)) * rng.uniform(0.5, 4.0, (nv, 1))).astype(np.float32)
    nw = (1.0 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    eps = np.float32(1e-6)
    xn = np.empty_like(x)
    for v in range(nv):
        ss = np.sum(x[v].astype(np.float64) ** 2)
        scale = np.float32(1.0) / np.sqrt(np.float32(ss / cols) + eps)
        xn[v] = (x[v] * scale) * nw
    eng = AttnEngine(0)
    try:
        y = torch.full((nv, rows), float("nan"), dtype=torch.float32, device="cuda")
        eng.matvec_gguf_fused(quant, dev(w), rows, cols, dev(x), y, TE_ATTN_RMSNORM_INPUT, dev(nw), float(eps),
                              n_vectors=nv)
        eng.synchronize()
        check(port, quant, w, rows, cols, xn, y.cpu().numpy())
    finally:
        eng.close()


@pytest.mark.parametrize("quant", [Q4, Q8])
@pytest.mark.parametrize("shape", [(896, 4864, 1), (2048, 2048, 4), (33, 96, 8)])
def test_matvec_fused_swiglu_input_accumulate(port, quant, shape):
    """te_matvec_gguf_fused + TE_ATTN_SWIGLU_INPUT + TE_ATTN_ACCUMULATE: y[v] += W te_swiglu_f32(gate, up)
    (ops.c:397-406), x[v] = [gate | up] -- the down projection and its residual add (qwen.c:1933-1941,
    :1105-1108)."""
    import torch
    from tinymetalagent_b200 import TE_ATTN_ACCUMULATE, TE_ATTN_SWIGLU_INPUT, AttnEngine
    rows, cols, nv = shape
    rng = np.random.default_rng(3 * rows + cols + quant + nv)
    w = quant_matrix(rng, GGML[quant], rows, cols)
    gu = (rng.standard_normal((nv, 2 * cols)) * 2.0).astype(np.float32)
    res = rng.standard_normal((nv, rows)).astype(np.float32)
    eng = AttnEngine(0)
    try:
        y = dev(res)
        eng.matvec_gguf_fused(quant, dev(w), rows, cols, dev(gu), y, TE_ATTN_SWIGLU_INPUT | TE_ATTN_ACCUMULATE,
                              n_vectors=nv)
        eng.synchronize()
        got = y.cpu().numpy()
        ref_fn = port.matvec_q4_0_f32 if quant == Q4 else port.matvec_q8_0_f32
        wd = np.abs(dequant(quant, w, rows, cols))
        for v in range(nv):
            g, u = gu[v, :cols], gu[v, cols:]
            s = ((g / (np.float32(1.0) + np.exp(-g))) * u).astype(np.float32)
            exp = (res[v] + ref_fn(w, rows, cols, s)).astype(np.float32)
            bound = 2e-5 * (wd @ np.abs(s)) + 1e-6 + 1e-7 * np.abs(exp)  # fp32 sums + device expf (a few ulp)
            assert (np.abs(got[v] - exp) <= bound).all(), v
    finally:
        eng.close()


def test_matvec_fused_rejects_bad_arguments():
    import torch
    from tinymetalagent_b200 import (TE_ATTN_RMSNORM_INPUT, TE_ATTN_SWIGLU_INPUT, AttnEngine, TinyEngineError)
    eng = AttnEngine(0)
    try:
        w = torch.zeros(18 * 4, dtype=torch.uint8, device="cuda")
        x = torch.zeros(128, dtype=torch.float32, device="cuda")
        y = torch.zeros(2, dtype=torch.float32, device="cuda")
        nw = torch.ones(64, dtype=torch.float32, device="cuda")
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf_fused(Q4, w, 2, 64, x, y, 0)                                  # no prologue
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf_fused(Q4, w, 2, 64, x, y, TE_ATTN_RMSNORM_INPUT | TE_ATTN_SWIGLU_INPUT, nw, 1e-6)
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf_fused(Q4, w, 2, 64, x, y, TE_ATTN_RMSNORM_INPUT, None, 1e-6)  # no norm weight
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf_fused(Q4, w, 2, 64, x, y, TE_ATTN_RMSNORM_INPUT, nw, 0.0)     # eps must be > 0
        with pytest.raises(TinyEngineError):
            eng.matvec_gguf_fused(Q4, w, 2, 64, x, y, TE_ATTN_RMSNORM_INPUT, nw[1:], 1e-6)  # unaligned weight
    finally:
        eng.close()
