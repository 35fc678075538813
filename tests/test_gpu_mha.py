"""API-level parity of the drop-in MultiHeadAttention (model/gpt.py:478-707).

Mirrors test_mha_integration_parity.py: same seeds, same shapes, same checked quantities (forward
output, the forward caches, dIn and the four parameter gradients), against fixtures produced by
the reference's own MultiHeadAttention, with its tolerance rtol=1e-4, atol=1e-5 for the float32
path, plus max-relative 1e-5.  The bf16 tensor-core path is checked against the oracle at 2e-2.
"""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-4, atol=1e-5)


def _torch():
    import torch
    return torch


def _load_weights(attn, g):
    torch = _torch()
    for p, key in ((attn.c_attn_w, "w_qkv"), (attn.c_attn_b, "b_qkv"), (attn.c_proj_w, "w_o"),
                   (attn.c_proj_b, "b_o")):
        p.weights.copy_(torch.from_numpy(g[key]))


def _run(attn, x, dy, B, T, accumulate=False):
    torch = _torch()
    gx = torch.from_numpy(x).cuda()
    out = attn.forward(gx, B, T)
    gdy = torch.from_numpy(dy).cuda()
    din = attn.backward(gdy, B, T, accumulate=accumulate)
    torch.cuda.synchronize()
    res = dict(out=out.get(), din=din.get(), d_attn_w=attn.c_attn_w.grads.cpu().numpy(),
               d_attn_b=attn.c_attn_b.grads.cpu().numpy(), d_proj_w=attn.c_proj_w.grads.cpu().numpy(),
               d_proj_b=attn.c_proj_b.grads.cpu().numpy())
    out.free()
    din.free()
    return res


def test_integration_oracle_scenario(pkg, cuda_dev):
    """capture_mha_oracle.py / test_mha_integration_parity.py: seed 4242, B=2 T=5 C=8 NH=2.
    Construction from the seeded global NumPy generator reproduces the reference's weights."""
    g = np.load(os.path.join(GOLDEN, "mha_b2_t5_c8_nh2.npz"))
    B, T, C, NH = (int(g[k]) for k in ("B", "T", "C", "NH"))
    np.random.seed(4242)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T))
    np.testing.assert_array_equal(attn.c_attn_w.weights.cpu().numpy(), g["w_qkv"])
    np.testing.assert_array_equal(attn.c_proj_w.weights.cpu().numpy(), g["w_o"])
    rng = np.random.RandomState(4243)
    x = rng.normal(0.0, 1.0, size=(B * T, C)).astype(np.float32)
    dy = rng.normal(0.0, 1.0, size=(B * T, C)).astype(np.float32)
    np.testing.assert_array_equal(x, g["x"])
    torch = _torch()
    out = attn.forward(torch.from_numpy(x).cuda(), B, T)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.get(), g["out"], **TOL)
    for name in ("cache_q", "cache_k", "cache_v", "cache_attn_weights", "cache_context"):
        np.testing.assert_allclose(getattr(attn, name), g[name], **TOL, err_msg=name)
    din = attn.backward(torch.from_numpy(dy).cuda(), B, T)
    torch.cuda.synchronize()
    np.testing.assert_allclose(din.get(), g["din"], **TOL)
    np.testing.assert_allclose(attn.c_attn_w.grads.cpu().numpy(), g["d_attn_w"], **TOL)
    np.testing.assert_allclose(attn.c_attn_b.grads.cpu().numpy(), g["d_attn_b"], **TOL)
    np.testing.assert_allclose(attn.c_proj_w.grads.cpu().numpy(), g["d_proj_w"], **TOL)
    np.testing.assert_allclose(attn.c_proj_b.grads.cpu().numpy(), g["d_proj_b"], **TOL)


FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "mha_*.npz")))


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(p) for p in FIXTURES])
def test_mha_fp32_matches_reference_fixture(pkg, cuda_dev, path):
    g = np.load(path)
    B, T, C, NH = (int(g[k]) for k in ("B", "T", "C", "NH"))
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T))
    _load_weights(attn, g)
    res = _run(attn, g["x"], g["dy"], B, T)
    for k, v in res.items():
        ref = g["out"] if k == "out" else g["din"] if k == "din" else g[k]
        np.testing.assert_allclose(v, ref, **TOL, err_msg=k)
        assert O.rel_err(v, ref) < 1e-5, (k, O.rel_err(v, ref))


@pytest.mark.parametrize("cfg,B,T,C,NH,prec,tol", [
    (1, 8, 128, 64, 4, "fp32", 1e-5),      # the 'small' preset, full size
    (2, 16, 128, 256, 8, "fp32", 1e-5),    # training-batch shape, batch slice
    (2, 16, 128, 256, 8, "bf16", 2e-2),    # the same on the tensor cores (head_dim 32)
    (2, 16, 128, 256, 8, "tf32", 2e-2),    # float32 storage, tf32 tensor-core products
    (5, 2, 512, 768, 12, "tf32", 2e-2),    # data-parallel step shape in tf32, batch slice
    (1, 4, 100, 128, 2, "tf32", 2e-2),     # ragged T in tf32
    (3, 2, 1024, 512, 8, "bf16", 2e-2),    # long context, batch slice
    (5, 2, 512, 768, 12, "bf16", 2e-2),    # data-parallel step shape, batch slice
    (1, 4, 100, 128, 2, "bf16", 2e-2),     # ragged T on the tensor-core path
])
def test_mha_config_against_oracle(pkg, cuda_dev, cfg, B, T, C, NH, prec, tol):
    inp = O.make_config_inputs(cfg, B, T, C, NH)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=prec))
    _load_weights(attn, inp)
    res = _run(attn, inp["x"], inp["dy"], B, T)
    out, cache = O.mha_forward(inp["x"], inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], B, T, NH)
    din, daw, dab, dpw, dpb = O.mha_backward(cache, inp["dy"], inp["w_qkv"], inp["w_o"], B, T, NH)
    ref = dict(out=out, din=din, d_attn_w=daw, d_attn_b=dab, d_proj_w=dpw, d_proj_b=dpb)
    for k in ref:
        assert O.rel_err(res[k], ref[k]) < tol, (k, O.rel_err(res[k], ref[k]))


@pytest.mark.parametrize("prec", ["fp32", "bf16"])
def test_accumulate_adds_to_existing_grads(pkg, cuda_dev, prec):
    B, T, C, NH = 2, 64, 128, 2
    inp = O.make_config_inputs(9, B, T, C, NH)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=prec))
    _load_weights(attn, inp)
    first = _run(attn, inp["x"], inp["dy"], B, T, accumulate=False)
    second = _run(attn, inp["x"], inp["dy"], B, T, accumulate=True)
    for k in ("d_attn_w", "d_attn_b", "d_proj_w", "d_proj_b"):
        np.testing.assert_allclose(second[k], 2 * first[k], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(second["din"], first["din"], rtol=0, atol=0)


def test_backward_without_forward_raises(pkg, cuda_dev):
    torch = _torch()
    attn = pkg.MultiHeadAttention(16, 2)
    with pytest.raises(RuntimeError, match="without forward caches"):
        attn.backward(torch.zeros(4 * 16, device="cuda"), 1, 4)
    attn.forward(torch.zeros(4 * 16, device="cuda"), 1, 4)
    attn.free_forward_caches()
    with pytest.raises(RuntimeError, match="without forward caches"):
        attn.backward(torch.zeros(4 * 16, device="cuda"), 1, 4)


def test_native_library_is_what_runs(pkg, cuda_dev):
    """Every op of a forward+backward is a launch of libattn_b200.so kernels."""
    torch = _torch()
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=64, num_heads=4, max_len=32))
    before = pkg.launch_count()
    out = attn.forward(torch.randn(2 * 32 * 64, device="cuda"), 2, 32)
    attn.backward(torch.randn(2 * 32 * 64, device="cuda"), 2, 32)
    torch.cuda.synchronize()
    assert pkg.launch_count() - before >= 8
    out.free()


@pytest.mark.parametrize("prec,tol,B,T0,steps,C,NH", [
    ("fp32", 1e-5, 2, 5, 4, 64, 4),      # the reference's 'small' head_dim 16
    ("bf16", 2e-2, 3, 130, 3, 256, 4),   # head_dim 64 on the tensor cores, prompt past one tile
    ("bf16", 2e-2, 2, 17, 2, 256, 8),    # head_dim 32
])
def test_kv_cache_decode_matches_full_forward(pkg, cuda_dev, prec, tol, B, T0, steps, C, NH):
    """Prompt forward with a KV cache, then one forward_decode per new token: each decode output
    equals the corresponding row of one causal forward over the whole sequence (what
    GenerationSession.generate recomputes per token, generate.py:611-628)."""
    torch = _torch()
    T = T0 + steps
    inp = O.make_config_inputs(4, B, T, C, NH)
    rng = np.random.default_rng(T * C)
    inp["b_qkv"] = (rng.standard_normal(3 * C) * 0.1).astype(np.float32)  # exercise the biases too
    inp["b_o"] = (rng.standard_normal(C) * 0.1).astype(np.float32)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=prec))
    _load_weights(attn, inp)
    x = inp["x"].reshape(B, T, C)
    full = attn.forward(torch.from_numpy(np.ascontiguousarray(x.reshape(B * T, C))).cuda(), B, T)
    ref = full.get().reshape(B, T, C)
    full.free()
    cache = attn.new_kv_cache(B, T)
    prompt = attn.forward(torch.from_numpy(np.ascontiguousarray(x[:, :T0].reshape(B * T0, C))).cuda(), B, T0,
                          kv_cache=cache)
    assert O.rel_err(prompt.get().reshape(B, T0, C), ref[:, :T0]) < tol
    prompt.free()
    assert cache.length == T0
    for t in range(T0, T):
        y = attn.forward_decode(torch.from_numpy(np.ascontiguousarray(x[:, t])).cuda(), B, cache)
        torch.cuda.synchronize()
        assert O.rel_err(y.get(), ref[:, t]) < tol, (t, O.rel_err(y.get(), ref[:, t]))
        y.free()
    assert cache.length == T
    with pytest.raises(RuntimeError):
        attn.forward_decode(torch.zeros((B, C), device="cuda"), B, cache)  # cache full


@pytest.mark.parametrize("prec,tol,B,T,C,NH", [
    ("fp32", 1e-5, 2, 33, 64, 4),
    ("bf16", 2e-2, 2, 200, 256, 4),
    ("bf16", 2e-2, 1, 130, 768, 12),
])
def test_forward_residual_matches_block_sequence(pkg, cuda_dev, prec, tol, B, T, C, NH):
    """forward_residual(x) == x + attn(ln_1(x)) of TransformerBlock.forward (model/gpt.py:778-783),
    with the LayerNorm of layernorm_kernel (core/kernels.py:75-110); the backward that follows
    sees the LayerNorm output as the attention input, exactly as after the unfused sequence."""
    torch = _torch()
    inp = O.make_config_inputs(5, B, T, C, NH)
    rng = np.random.default_rng(C + T)
    gamma = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    inp["b_qkv"] = (rng.standard_normal(3 * C) * 0.1).astype(np.float32)
    inp["b_o"] = (rng.standard_normal(C) * 0.1).astype(np.float32)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=prec))
    _load_weights(attn, inp)
    gx = torch.from_numpy(inp["x"].copy()).cuda()
    attn.forward_residual(gx, B, T, torch.from_numpy(gamma).cuda(), torch.from_numpy(beta).cuda())
    ln = O.layernorm(inp["x"], gamma, beta)
    out, cache = O.mha_forward(ln, inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], B, T, NH)
    torch.cuda.synchronize()
    assert O.rel_err(gx.cpu().numpy(), inp["x"] + out) < tol
    assert O.rel_err(attn.cache_input, ln) < (tol if prec == "fp32" else 1e-2)
    din = attn.backward(torch.from_numpy(inp["dy"]).cuda(), B, T)
    torch.cuda.synchronize()
    ref_din, ref_daw, ref_dab, ref_dpw, ref_dpb = O.mha_backward(cache, inp["dy"], inp["w_qkv"], inp["w_o"], B, T, NH)
    got = dict(din=din.get(), daw=attn.c_attn_w.grads.cpu().numpy(), dab=attn.c_attn_b.grads.cpu().numpy(),
               dpw=attn.c_proj_w.grads.cpu().numpy(), dpb=attn.c_proj_b.grads.cpu().numpy())
    ref = dict(din=ref_din, daw=ref_daw, dab=ref_dab, dpw=ref_dpw, dpb=ref_dpb)
    din.free()
    for k in ref:
        assert O.rel_err(got[k], ref[k]) < tol, (k, O.rel_err(got[k], ref[k]))



@pytest.mark.parametrize("prec,tol,B,T,C,NH", [("fp32", 1e-5, 2, 33, 64, 4), ("bf16", 2e-2, 2, 130, 256, 4)])
def test_backward_residual_matches_block_sequence(pkg, cuda_dev, prec, tol, B, T, C, NH):
    """forward_residual + backward_residual against the attention half of TransformerBlock:
    x1 = x + attn(ln_1(x)); dX0 = dX1 + ln_1 backward of attn.backward(dX1) (model/gpt.py:825-838)."""
    torch = _torch()
    inp = O.make_config_inputs(5, B, T, C, NH)
    rng = np.random.default_rng(C * 3 + T)
    gamma = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=prec))
    _load_weights(attn, inp)
    gx = torch.from_numpy(inp["x"].copy()).cuda()
    tg = torch.from_numpy(gamma).cuda()
    attn.forward_residual(gx, B, T, tg, torch.from_numpy(beta).cuda())
    gd = torch.from_numpy(inp["dy"].copy()).cuda()
    dgamma = torch.full((C,), 5.0, device="cuda")
    dbeta = torch.full((C,), 5.0, device="cuda")
    attn.backward_residual(gd, B, T, tg, dgamma, dbeta)
    torch.cuda.synchronize()
    ln = O.layernorm(inp["x"], gamma, beta)
    _, cache = O.mha_forward(ln, inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], B, T, NH)
    dln, daw, dab, dpw, dpb = O.mha_backward(cache, inp["dy"], inp["w_qkv"], inp["w_o"], B, T, NH)
    dx_ln, dg_ref, db_ref = O.layernorm_backward(dln, inp["x"], gamma)
    checks = dict(dx=(gd, inp["dy"] + dx_ln), dgamma=(dgamma, dg_ref), dbeta=(dbeta, db_ref),
                  d_attn_w=(attn.c_attn_w.grads, daw), d_proj_b=(attn.c_proj_b.grads, dpb))
    for k, (got, want) in checks.items():
        assert O.rel_err(got.cpu().numpy(), want) < tol, (k, O.rel_err(got.cpu().numpy(), want))


@pytest.mark.parametrize("H,M,D,Din,seed", [(3, 17, 8, 6, 1337), (4, 200, 32, 48, 7)])
def test_mha_controller_matches_oracle(pkg, cuda_dev, H, M, D, Din, seed):
    """MHAController.forward (core/mha_ops.py:84-138) as the reference's golden test drives it in
    its Layer 3 (test_mha_golden_model.py:285-308, 511-517: seed 1337, H=3, M=17, D=8, Din=6,
    X ~ N(0, 1), W_qkv ~ N(0, 1/sqrt(Din))), and at a larger shape: out and probs against the
    oracle's fused projection + causal attention, at the reference's tolerance and 1e-5 relative."""
    torch = _torch()
    np.random.seed(seed)
    X = np.random.normal(0.0, 1.0, size=(H, M, Din)).astype(np.float32)
    W = np.random.normal(0.0, 1.0 / np.sqrt(Din), size=(Din, 3 * D)).astype(np.float32)
    ctl = pkg.MHAController(H, M, D)
    out, probs = ctl.forward(X, W)
    assert out.shape == (H, M, D) and probs.shape == (H, M, M)
    fused = X.astype(np.float64) @ W.astype(np.float64)  # matmul_qkv_fused, split_qkv_kernel
    q, k, v = fused[..., :D], fused[..., D:2 * D], fused[..., 2 * D:]
    ref_out, _, ref_probs = O.causal_attention_forward(q, k, v, 1.0 / np.sqrt(D))
    np.testing.assert_allclose(out, ref_out, **TOL)
    np.testing.assert_allclose(probs, ref_probs, **TOL)
    assert O.rel_err(out, ref_out) < 1e-5 and O.rel_err(probs, ref_probs) < 1e-5
    # the pass-through of the fused projection on device buffers
    gX, gW = torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda()
    gF = torch.empty((H, M, 3 * D), dtype=torch.float32, device="cuda")
    ctl.matmul_qkv_fused(gX, gW, gF, Din, block=(256, 1, 1), grid=(1, 1))
    torch.cuda.synchronize()
    assert O.rel_err(gF.cpu().numpy(), fused) < 1e-5
