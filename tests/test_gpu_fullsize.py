"""Parity at the sizes the bench times: the whole workload, not a batch slice.

The bench's data-parallel step (global batch 512, T=512, C=768, 12 heads of 64) on one GPU runs
6,144 heads through the persistent attention kernels (about 41 heads per CTA, the dQ accumulator
reused from head to head) and weight-gradient GEMMs over K = 262,144 tokens (split along K with
reduce-adds).  These tests run MultiHeadAttention.forward + backward at exactly those sizes (and at
the long-context and training-batch configurations' full sizes) and compare against a checker that
evaluates the oracle's formulas (model/gpt.py:652-689 for the backward, the golden model's causal
softmax for the forward) on the device with torch, chunk by chunk over the sequences:

* the four parameter gradients in full, each chunk's contribution summed in float64;
* the output and dX on sampled sequences (the first, the last and two in between).

The checker computes in float64 for the float32 path (tolerance 1e-5, max|diff| / max|ref|) and in
float32 with TF32 disabled for the bf16 and tf32 paths (tolerance 2e-2).  Inputs are seeded
synthetic data with the workloads' distributions: x, dY ~ N(0, 1), weights ~ N(0, 0.02), biases
0.1 * N(0, 1).
"""
import math

import numpy as np
import pytest

from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(B, T, C, seed):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    r = lambda *shape: torch.randn(shape, generator=g, device="cuda")  # noqa: E731
    return dict(x=r(B * T, C), dy=r(B * T, C), w_qkv=0.02 * r(C, 3 * C), b_qkv=0.1 * r(3 * C),
                w_o=0.02 * r(C, C), b_o=0.1 * r(C))


def checker(inp, B, T, NH, dt, sample, chunk):
    """The oracle's forward and backward on the device, in ``dt``, over chunks of ``chunk``
    sequences.  Returns the parameter gradients (float64) and out / dX of the sampled sequences."""
    import torch
    C = inp["x"].shape[1]
    D = C // NH
    scale = 1.0 / math.sqrt(D)
    wq, bq, wo, bo = (inp[k].to(dt) for k in ("w_qkv", "b_qkv", "w_o", "b_o"))
    mask = torch.ones(T, T, dtype=torch.bool, device="cuda").tril()
    f64 = dict(dtype=torch.float64, device="cuda")
    grads = dict(d_attn_w=torch.zeros(C, 3 * C, **f64), d_attn_b=torch.zeros(3 * C, **f64),
                 d_proj_w=torch.zeros(C, C, **f64), d_proj_b=torch.zeros(C, **f64))
    outs, dxs = {}, {}
    for b0 in range(0, B, chunk):
        c = min(chunk, B - b0)
        rows = slice(b0 * T, (b0 + c) * T)
        xs, dys = inp["x"][rows].to(dt), inp["dy"][rows].to(dt)
        qkv = xs @ wq + bq                                              # model/gpt.py:558
        q, k, v = qkv.view(c, T, 3, NH, D).permute(2, 0, 3, 1, 4)       # [c, NH, T, D] each
        s = (q @ k.transpose(-1, -2)) * scale
        p = torch.softmax(s.masked_fill(~mask, float("-inf")), dim=-1)
        o = p @ v
        ctx = o.permute(0, 2, 1, 3).reshape(c * T, C)
        grads["d_proj_w"] += (ctx.t() @ dys).double()                 # gpt.py:666-667
        grads["d_proj_b"] += dys.sum(0).double()
        do = (dys @ wo.t()).view(c, T, NH, D).permute(0, 2, 1, 3)      # gpt.py:670
        dv = p.transpose(-1, -2) @ do                                   # gpt.py:672-680
        dp = do @ v.transpose(-1, -2)
        ds = p * (dp - (dp * p).sum(-1, keepdim=True)) * scale
        dq, dk = ds @ k, ds.transpose(-1, -2) @ q
        dqkv = torch.stack([dq, dk, dv]).permute(1, 3, 0, 2, 4).reshape(c * T, 3 * C)
        grads["d_attn_w"] += (xs.t() @ dqkv).double()                  # gpt.py:687-688
        grads["d_attn_b"] += dqkv.sum(0).double()
        for b in sample:
            if b0 <= b < b0 + c:
                r = slice((b - b0) * T, (b - b0 + 1) * T)
                outs[b] = (ctx[r] @ wo + bo).double()                   # gpt.py:629
                dxs[b] = (dqkv[r] @ wq.t()).double()                    # gpt.py:689
        del qkv, q, k, v, s, p, o, ctx, do, dv, dp, ds, dq, dk, dqkv
    return grads, outs, dxs


def _run_and_check(pkg, B, T, C, NH, prec, tol, seed, chunk):
    import torch
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        inp = _inputs(B, T, C, seed)
        attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                    attention_precision=prec))
        for p, key in ((attn.c_attn_w, "w_qkv"), (attn.c_attn_b, "b_qkv"), (attn.c_proj_w, "w_o"),
                       (attn.c_proj_b, "b_o")):
            p.weights.copy_(inp[key])
        out = attn.forward(inp["x"], B, T)
        din = attn.backward(inp["dy"], B, T, accumulate=False)
        attn.wait_grad_sync()
        torch.cuda.synchronize()
        got = dict(d_attn_w=attn.c_attn_w.grads, d_attn_b=attn.c_attn_b.grads, d_proj_w=attn.c_proj_w.grads,
                   d_proj_b=attn.c_proj_b.grads)
        sample = sorted({0, 1, B // 2, B - 1})
        grads, outs, dxs = checker(inp, B, T, NH, torch.float64 if prec == "fp32" else torch.float32, sample,
                                   chunk)
        errs = {k: O.rel_err(got[k].double().cpu().numpy(), grads[k].cpu().numpy()) for k in grads}
        o2, d2 = out.tensor.view(B, T, C), din.tensor.view(B, T, C)
        for b in sample:
            errs[f"out[{b}]"] = O.rel_err(o2[b].double().cpu().numpy(), outs[b].cpu().numpy())
            errs[f"dX[{b}]"] = O.rel_err(d2[b].double().cpu().numpy(), dxs[b].cpu().numpy())
        bad = {k: v for k, v in errs.items() if not np.isfinite(v) or v >= tol}
        assert not bad, f"{prec} B={B} T={T} C={C} NH={NH}: above {tol}: {bad}"
        assert pkg.lib.attn_device_error(0) == 0
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32


@pytest.mark.parametrize("prec,tol", [("bf16", 2e-2), ("fp32", 1e-5)])
def test_data_parallel_step_full_batch_512(pkg, cuda_dev, prec, tol):
    """The bench's workload on one GPU: global batch 512, T=512, C=768, NH=12 (head_dim 64)."""
    _run_and_check(pkg, 512, 512, 768, 12, prec, tol, seed=1005, chunk=32)


def test_long_context_full_batch_32(pkg, cuda_dev):
    """Long-context configuration at full size: B=32, T=1024, C=512, NH=8, bf16."""
    _run_and_check(pkg, 32, 1024, 512, 8, "bf16", 2e-2, seed=1003, chunk=8)


@pytest.mark.parametrize("prec,tol", [("fp32", 1e-5), ("tf32", 2e-2)])
def test_training_batch_full_256(pkg, cuda_dev, prec, tol):
    """Training-batch configuration at full size: B=256, T=128, C=256, NH=8 (head_dim 32), float32
    inputs, with float32 arithmetic and with tf32 tensor-core products."""
    _run_and_check(pkg, 256, 128, 256, 8, prec, tol, seed=1002, chunk=64)
