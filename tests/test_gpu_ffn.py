"""API-level parity of the drop-in FeedForward (model/gpt.py:282-470).

Mirrors test_ffn_gpu_backward.py: the same scenario (seed 1337, C=16, M=6, dOut = output) and the
same checked quantities (dIn and the four parameter gradients, plus the forward output and the
cached activations), against fixtures produced by the reference's own FeedForward with its NumPy
backward, at its tolerance rtol=1e-4, atol=1e-5 for the float32 path.  Wider shapes and the bf16
tensor-core path (2e-2) are checked against the oracle, and the reference's own FFN kernels
(built from their sources into oracle/_ref) run beside the library on the same inputs.
"""
import ctypes
import os

import numpy as np
import pytest

from conftest import GOLDEN, ROOT
from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-4, atol=1e-5)
GRADS = (("d_fc_w", "c_fc_w"), ("d_fc_b", "c_fc_b"), ("d_proj_w", "c_proj_w"), ("d_proj_b", "c_proj_b"))


def _torch():
    import torch
    return torch


def _bf16_round(a):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).bfloat16().float().numpy()


def _load_weights(ffn, g):
    torch = _torch()
    for key, attr in (("w_fc", "c_fc_w"), ("b_fc", "c_fc_b"), ("w_proj", "c_proj_w"), ("b_proj", "c_proj_b")):
        getattr(ffn, attr).weights.copy_(torch.from_numpy(np.ascontiguousarray(g[key], dtype=np.float32)))


def _run(ffn, x, dy, B, T, accumulate=False):
    torch = _torch()
    out = ffn.forward(torch.from_numpy(x).cuda(), B, T)
    pre = ffn.cache_pre_act.tensor.float().cpu().numpy()
    act = ffn.cache_activated.tensor.float().cpu().numpy()
    din = ffn.backward(torch.from_numpy(dy).cuda(), B, T, accumulate=accumulate)
    torch.cuda.synchronize()
    res = dict(out=out.get(), din=din.get(), pre=pre, act=act)
    for key, attr in GRADS:
        res[key] = getattr(ffn, attr).grads.cpu().numpy()
    return res


def _config(pkg, C, prec="fp32"):
    return pkg.GPTConfig(vocab_size=64, embedding_dim=C, num_heads=2, max_len=8, attention_precision=prec)


def _inputs(M, C, seed):
    rng = np.random.default_rng(seed)
    return dict(x=rng.standard_normal((M, C)).astype(np.float32),
                w_fc=(rng.standard_normal((C, 4 * C)) * 0.05).astype(np.float32),
                b_fc=(rng.standard_normal(4 * C) * 0.5).astype(np.float32),
                w_proj=(rng.standard_normal((4 * C, C)) * 0.05).astype(np.float32),
                b_proj=(rng.standard_normal(C) * 0.5).astype(np.float32),
                dy=rng.standard_normal((M, C)).astype(np.float32))


def test_ffn_gpu_backward_scenario(pkg, cuda_dev):
    """test_ffn_gpu_backward.py:35-106: seeded construction reproduces the reference's weights; the
    library's backward matches the reference's NumPy oracle backward at the reference's tolerance."""
    g = np.load(os.path.join(GOLDEN, "ffn_c16_m6.npz"))
    C, M = int(g["C"]), int(g["M"])
    np.random.seed(1337)
    ffn = pkg.FeedForward(_config(pkg, C))
    for key, attr in (("w_fc", "c_fc_w"), ("w_proj", "c_proj_w")):
        np.testing.assert_array_equal(getattr(ffn, attr).weights.cpu().numpy(), g[key])
    x = np.random.normal(0.0, 1.0, size=(M, C)).astype(np.float32)
    np.testing.assert_array_equal(x, g["x"])
    res = _run(ffn, x, g["dy"], 1, M)
    for key in ("out", "pre", "act", "din", "d_fc_w", "d_fc_b", "d_proj_w", "d_proj_b"):
        np.testing.assert_allclose(res[key], g[key], **TOL, err_msg=key)
        assert O.rel_err(res[key], g[key]) < 1e-5, key


def test_ffn_fixture_with_biases(pkg, cuda_dev):
    g = np.load(os.path.join(GOLDEN, "ffn_c64_m40.npz"))
    C, M = int(g["C"]), int(g["M"])
    ffn = pkg.FeedForward(_config(pkg, C))
    _load_weights(ffn, g)
    res = _run(ffn, g["x"], g["dy"], 2, M // 2)
    for key in ("out", "pre", "act", "din", "d_fc_w", "d_fc_b", "d_proj_w", "d_proj_b"):
        np.testing.assert_allclose(res[key], g[key], **TOL, err_msg=key)
    # accumulate=True adds a second backward's gradients onto the first's (model/gpt.py:451-456)
    torch = _torch()
    ffn.forward(torch.from_numpy(g["x"]).cuda(), 2, M // 2).free()
    ffn.backward(torch.from_numpy(g["dy"]).cuda(), 2, M // 2, accumulate=True).free()
    torch.cuda.synchronize()
    for key, attr in GRADS:
        np.testing.assert_allclose(getattr(ffn, attr).grads.cpu().numpy(), 2 * g[key], rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("prec,tol,M,C", [
    ("fp32", 1e-5, 74, 64), ("bf16", 2e-2, 74, 64), ("bf16", 2e-2, 1024, 256), ("bf16", 2e-2, 600, 768),
    ("fp32", 1e-5, 300, 96),
    # edge shapes: one token, tiny widths (CUDA-core paths), hidden sizes that leave partial 256-column
    # tiles and partial 64- or 32-column epilogue chunks on the tensor cores (4C = 288, 544), and a
    # contraction (C = 136) that is not a multiple of the 64-deep K block
    ("fp32", 1e-5, 2, 8), ("bf16", 2e-2, 2, 8), ("fp32", 1e-5, 6, 24), ("bf16", 2e-2, 130, 40),
    ("bf16", 2e-2, 1000, 72), ("bf16", 2e-2, 4098, 136)])
def test_ffn_matches_oracle(pkg, cuda_dev, prec, tol, M, C):
    inp = _inputs(M, C, M + C)
    if prec == "bf16":  # the oracle sees the operands the tensor cores see
        for k in ("x", "w_fc", "w_proj", "dy"):
            inp[k] = _bf16_round(inp[k])
    ffn = pkg.FeedForward(_config(pkg, C, prec))
    _load_weights(ffn, inp)
    res = _run(ffn, inp["x"], inp["dy"], 2, M // 2)
    out, cache = O.ffn_forward(inp["x"], inp["w_fc"], inp["b_fc"], inp["w_proj"], inp["b_proj"])
    d_in, dfw, dfb, dpw, dpb = O.ffn_backward(cache, inp["dy"], inp["w_fc"], inp["w_proj"])
    want = dict(out=out, pre=cache["pre"], act=cache["act"], din=d_in, d_fc_w=dfw, d_fc_b=dfb, d_proj_w=dpw,
                d_proj_b=dpb)
    for k, v in want.items():
        assert O.rel_err(res[k], v) < tol, (k, O.rel_err(res[k], v))
    assert pkg.lib.attn_device_error(1) == 0


@pytest.mark.parametrize("prec,tol,M,C", [("fp32", 1e-5, 66, 64), ("bf16", 2e-2, 512, 256)])
def test_ffn_residual_matches_block_sequence(pkg, cuda_dev, prec, tol, M, C):
    """forward_residual/backward_residual against the MLP half of TransformerBlock
    (model/gpt.py:785-795, :806-821): x2 = x1 + ffn(ln_2(x1)); dX1 = dX2 + ln_2 backward of
    ffn.backward(dX2)."""
    torch = _torch()
    inp = _inputs(M, C, 7 * M + C)
    rng = np.random.default_rng(C)
    gamma = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    beta = (0.1 * rng.standard_normal(C)).astype(np.float32)
    ffn = pkg.FeedForward(_config(pkg, C, prec))
    _load_weights(ffn, inp)
    gx = torch.from_numpy(inp["x"].copy()).cuda()
    tg = torch.from_numpy(gamma).cuda()
    ffn.forward_residual(gx, 2, M // 2, tg, torch.from_numpy(beta).cuda())
    gd = torch.from_numpy(inp["dy"].copy()).cuda()
    dgamma = torch.full((C,), 3.0, device="cuda")
    dbeta = torch.full((C,), 3.0, device="cuda")
    ffn.backward_residual(gd, 2, M // 2, tg, dgamma, dbeta)
    torch.cuda.synchronize()
    ln = O.layernorm(inp["x"], gamma, beta)
    out, cache = O.ffn_forward(ln, inp["w_fc"], inp["b_fc"], inp["w_proj"], inp["b_proj"])
    dln, dfw, dfb, dpw, dpb = O.ffn_backward(cache, inp["dy"], inp["w_fc"], inp["w_proj"])
    dx_ln, dg_ref, db_ref = O.layernorm_backward(dln, inp["x"], gamma)
    checks = dict(x=(gx, inp["x"] + out), dx=(gd, inp["dy"] + dx_ln), dgamma=(dgamma, dg_ref),
                  dbeta=(dbeta, db_ref), d_fc_w=(ffn.c_fc_w.grads, dfw), d_fc_b=(ffn.c_fc_b.grads, dfb),
                  d_proj_w=(ffn.c_proj_w.grads, dpw))
    for k, (got, want) in checks.items():
        assert O.rel_err(got.cpu().numpy(), want) < tol, (k, O.rel_err(got.cpu().numpy(), want))


def test_ffn_inference_and_errors(pkg, cuda_dev):
    torch = _torch()
    C, M = 64, 40
    inp = _inputs(M, C, 3)
    ffn = pkg.FeedForward(_config(pkg, C, "bf16"))
    _load_weights(ffn, inp)
    x = torch.from_numpy(inp["x"]).cuda()
    with pytest.raises(RuntimeError):
        ffn.backward(x, 1, M)  # no forward caches (model/gpt.py:378-379)
    y_train = ffn.forward(x, 1, M).get()
    ffn.training = False
    y_eval = ffn.forward(x, 1, M).get()
    np.testing.assert_array_equal(y_train, y_eval)  # the pre-activation cache changes nothing
    assert ffn.cache_pre_act is None
    with pytest.raises(RuntimeError):
        ffn.backward(x, 1, M)
    ffn.training = True
    ffn.forward(x, 1, M).free()
    ffn.use_cpu_backward = True
    with pytest.raises(RuntimeError):
        ffn.backward(x, 1, M)


def _ref_lib():
    path = os.path.join(ROOT, "oracle", "_ref", "libref_kernels.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref not built (needs the reference checkout at build time)")
    lib = ctypes.CDLL(path)
    P, I = ctypes.c_void_p, ctypes.c_int
    lib.ref_ffn_forward.argtypes = [P] * 8 + [I, I]
    lib.ref_ffn_backward.argtypes = [P] * 11 + [I, I]
    return lib


@pytest.mark.parametrize("M,C", [(6, 16), (257, 64), (1024, 192)])
def test_ffn_matches_reference_kernels(pkg, cuda_dev, M, C):
    """The reference's FFN kernel sequence (matmul_2d_kernel, activation_kernel,
    matmul_backward_weights/input_kernel, gelu_backward_kernel, reduce_sum_axis0_kernel) run on the
    same inputs: the float32 path agrees within 1e-5."""
    torch = _torch()
    ref = _ref_lib()
    inp = _inputs(M, C, 11 * M + C)
    t = {k: torch.from_numpy(v).cuda() for k, v in inp.items()}
    H = 4 * C
    pre, act = torch.empty((M, H), device="cuda"), torch.empty((M, H), device="cuda")
    out, din = torch.empty((M, C), device="cuda"), torch.empty((M, C), device="cuda")
    g = dict(d_fc_w=torch.empty((C, H), device="cuda"), d_fc_b=torch.empty(H, device="cuda"),
             d_proj_w=torch.empty((H, C), device="cuda"), d_proj_b=torch.empty(C, device="cuda"))
    assert ref.ref_ffn_forward(t["x"].data_ptr(), t["w_fc"].data_ptr(), t["b_fc"].data_ptr(), t["w_proj"].data_ptr(),
                               t["b_proj"].data_ptr(), pre.data_ptr(), act.data_ptr(), out.data_ptr(), M, C) == 0
    assert ref.ref_ffn_backward(t["dy"].data_ptr(), t["x"].data_ptr(), pre.data_ptr(), act.data_ptr(),
                                t["w_fc"].data_ptr(), t["w_proj"].data_ptr(), din.data_ptr(), g["d_fc_w"].data_ptr(),
                                g["d_fc_b"].data_ptr(), g["d_proj_w"].data_ptr(), g["d_proj_b"].data_ptr(), M, C) == 0
    ffn = pkg.FeedForward(_config(pkg, C))
    _load_weights(ffn, inp)
    res = _run(ffn, inp["x"], inp["dy"], 1, M)
    want = dict(out=out, pre=pre, act=act, din=din, **g)
    for k, v in want.items():
        assert O.rel_err(res[k], v.cpu().numpy()) < 1e-5, (k, O.rel_err(res[k], v.cpu().numpy()))
