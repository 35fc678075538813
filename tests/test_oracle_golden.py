"""Pin the CPU oracle to fixtures produced by the reference's own Python code.

The fixtures come from tests/golden/make_golden.py, which runs test_mha_golden_model.py's
NumPy functions and model/gpt.py's MultiHeadAttention (forward + NumPy backward) unchanged.
Tolerances follow the reference's own checks: rtol=1e-4, atol=1e-5
(test_mha_golden_model.py:45, test_mha_integration_parity.py:37).
"""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import mha_oracle as O

TOL = dict(rtol=1e-4, atol=1e-5)


def test_kernel_level_golden():
    g = np.load(os.path.join(GOLDEN, "kernel_h3_m17_d8.npz"))
    scale = float(g["scale"])
    out, lse, probs = O.causal_attention_forward(g["Q"], g["K"], g["V"], scale)
    np.testing.assert_allclose(probs, g["probs"], **TOL)
    np.testing.assert_allclose(out, g["out"], **TOL)
    # lse reproduces the probabilities: P = exp(s - lse) on and below the diagonal
    s = np.einsum("hid,hjd->hij", g["Q"].astype(np.float64), g["K"].astype(np.float64)) * scale
    p_from_lse = np.where(O.causal_mask(int(g["M"])), np.exp(s - lse[..., None]), 0.0)
    np.testing.assert_allclose(p_from_lse, g["probs"], **TOL)
    # the golden backward leaves the softmax scale out of dS (test_mha_golden_model.py:75-91)
    dq, dk, dv, ds = O.causal_attention_backward(g["probs"], g["Q"], g["K"], g["V"], g["dOut"],
                                                 scale, apply_scale=False)
    np.testing.assert_allclose(dv, g["dV"], **TOL)
    np.testing.assert_allclose(ds, g["dScores_pre"], **TOL)
    np.testing.assert_allclose(dq, g["dQ"], **TOL)
    np.testing.assert_allclose(dk, g["dK"], **TOL)
    # the production convention (model/gpt.py:677) is exactly scale × the golden one
    dq2, dk2, dv2, _ = O.causal_attention_backward(g["probs"], g["Q"], g["K"], g["V"], g["dOut"],
                                                   scale, apply_scale=True)
    np.testing.assert_allclose(dq2, scale * dq, rtol=1e-12)
    np.testing.assert_allclose(dk2, scale * dk, rtol=1e-12)
    np.testing.assert_allclose(dv2, dv, rtol=1e-12)


MHA_FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "mha_*.npz")))


@pytest.mark.parametrize("path", MHA_FIXTURES, ids=[os.path.basename(p) for p in MHA_FIXTURES])
def test_mha_golden(path):
    g = np.load(path)
    B, T, C, NH = (int(g[k]) for k in ("B", "T", "C", "NH"))
    out, cache = O.mha_forward(g["x"], g["w_qkv"], g["b_qkv"], g["w_o"], g["b_o"], B, T, NH)
    np.testing.assert_allclose(out, g["out"], **TOL)
    np.testing.assert_allclose(cache["q"], g["cache_q"], **TOL)
    np.testing.assert_allclose(cache["k"], g["cache_k"], **TOL)
    np.testing.assert_allclose(cache["v"], g["cache_v"], **TOL)
    np.testing.assert_allclose(cache["context"], g["cache_context"], **TOL)
    if "cache_attn_weights" in g:
        np.testing.assert_allclose(cache["probs"], g["cache_attn_weights"], **TOL)
    din, daw, dab, dpw, dpb = O.mha_backward(cache, g["dy"], g["w_qkv"], g["w_o"], B, T, NH)
    np.testing.assert_allclose(din, g["din"], **TOL)
    np.testing.assert_allclose(daw, g["d_attn_w"], **TOL)
    np.testing.assert_allclose(dab, g["d_attn_b"], **TOL)
    np.testing.assert_allclose(dpw, g["d_proj_w"], **TOL)
    np.testing.assert_allclose(dpb, g["d_proj_b"], **TOL)


def test_oracle_fp32_mirror_matches_fp64():
    """The fp32 restatement (timed as the CPU baseline) agrees with the fp64 oracle."""
    inp = O.make_config_inputs(1, 2, 128, 64, 4)
    out64, c64 = O.mha_forward(inp["x"], inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], 2, 128, 4)
    out32, c32 = O.mha_forward(inp["x"], inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], 2, 128, 4,
                               dtype=np.float32)
    assert O.rel_err(out32, out64) < 1e-5
    g64 = O.mha_backward(c64, inp["dy"], inp["w_qkv"], inp["w_o"], 2, 128, 4)
    g32 = O.mha_backward(c32, inp["dy"], inp["w_qkv"], inp["w_o"], 2, 128, 4, dtype=np.float32)
    for a, b in zip(g32, g64):
        assert O.rel_err(a, b) < 1e-5


def test_decode_is_last_causal_row():
    rng = np.random.default_rng(7)
    q = rng.standard_normal((2, 3, 40, 16))
    k = rng.standard_normal((2, 3, 40, 16))
    v = rng.standard_normal((2, 3, 40, 16))
    out, lse, _ = O.causal_attention_forward(q, k, v, 0.25)
    dout, dlse = O.decode_attention(q[:, :, -1], k, v, 0.25)
    np.testing.assert_allclose(dout, out[:, :, -1], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(dlse, lse[:, :, -1], rtol=1e-12)


def test_rel_err_catches_planted_mistake():
    """A mistake planted in the oracle's output (on the CPU) is caught at the stated tolerance."""
    g = np.load(os.path.join(GOLDEN, "kernel_h3_m17_d8.npz"))
    out, _, _ = O.causal_attention_forward(g["Q"], g["K"], g["V"], float(g["scale"]))
    bad = out.copy()
    bad[1, 16, 3] += 1e-3 * np.abs(out).max()
    assert O.rel_err(bad, g["out"]) > 1e-5
    assert O.rel_err(out, g["out"]) < 1e-6


@pytest.mark.parametrize("name", ["ffn_c16_m6", "ffn_c64_m40"])
def test_ffn_oracle_matches_reference_feedforward(name):
    """The FFN restatement against model/gpt.py's FeedForward run with its NumPy backward; the
    reference's own parity tolerance (test_ffn_gpu_backward.py:25)."""
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    out, cache = O.ffn_forward(g["x"], g["w_fc"], g["b_fc"], g["w_proj"], g["b_proj"])
    np.testing.assert_allclose(cache["pre"], g["pre"], **TOL)
    np.testing.assert_allclose(cache["act"], g["act"], **TOL)
    np.testing.assert_allclose(out, g["out"], **TOL)
    d_in, dfw, dfb, dpw, dpb = O.ffn_backward(cache, g["dy"], g["w_fc"], g["w_proj"])
    for got, key in ((d_in, "din"), (dfw, "d_fc_w"), (dfb, "d_fc_b"), (dpw, "d_proj_w"), (dpb, "d_proj_b")):
        np.testing.assert_allclose(got, g[key], **TOL, err_msg=key)
