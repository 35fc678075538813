"""CPU oracle for the causal multi-head attention path (test infrastructure only).

This module is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py`` (its ``cpu_baseline`` leg and ``--impl reference`` arm) import it.  The
shipped path is the CUDA library behind ``include/attn_b200.h``; it never calls in here.

It restates, in NumPy, the reference trainer's own NumPy math for the path:

* forward: ``numpy_causal_attention_forward`` (test_mha_golden_model.py:60-72) wrapped in the
  projections of ``MultiHeadAttention.forward`` (model/gpt.py:531-631): ``qkv = x·Wqkv + b``
  (``matmul_2d_kernel``, core/kernels.py:119-140, bias added after the dot), the head split of
  ``split_heads_kernel`` (core/mha_kernels.py:534-558), the merge of ``merge_heads_kernel``
  (core/mha_kernels.py:567-584) and ``out = ctx·Wo + bo`` (model/gpt.py:629);
* backward: ``MultiHeadAttention.backward`` (model/gpt.py:652-689) step for step, including the
  softmax scale applied to dS (model/gpt.py:677).  The golden-model backward
  (test_mha_golden_model.py:75-91) omits that scale; ``causal_attention_backward`` exposes it
  through ``apply_scale`` so both conventions can be checked.

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against fixtures
that ``tests/golden/make_golden.py`` produced by running the reference's own Python code
(its ``MultiHeadAttention`` and golden-model functions) in this container.

Two precisions: ``np.float64`` for parity checks (the golden model computes in float64),
``np.float32`` to time the reference's own fp32 NumPy backward as the CPU baseline.
"""

from __future__ import annotations

import numpy as np

# The fused forward kernel seeds its running row max with -1e30 (core/mha_kernels.py:450).
ROW_MAX_INIT = -1e30


def causal_mask(T: int) -> np.ndarray:
    """Lower-triangular mask: key j is visible to query i iff j <= i
    (test_mha_golden_model.py:64, core/mha_kernels.py:429 ``valid_cols = i + 1``)."""
    return np.tril(np.ones((T, T), dtype=bool))


def causal_attention_forward(q, k, v, scale, dtype=np.float64):
    """Causal softmax attention for q, k, v of shape [..., T, D].

    Follows test_mha_golden_model.py:60-72: scores = scale·q·kᵀ, mask j > i, subtract the row
    max, exp, normalise, out = P·V.  Returns ``(out, lse, probs)`` where ``lse`` is the
    natural-log log-sum-exp of the scaled, masked scores per row (the quantity the B200 kernels
    store instead of P; reconstruct P as exp(s - lse)).
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    T = q.shape[-2]
    mask = causal_mask(T)
    scores = np.einsum("...id,...jd->...ij", q, k) * dtype(scale)
    masked = np.where(mask, scores, -np.inf)
    row_max = np.max(masked, axis=-1, keepdims=True)
    ex = np.where(mask, np.exp(masked - row_max), 0.0).astype(dtype)
    row_sum = np.sum(ex, axis=-1, keepdims=True)
    probs = ex / row_sum
    out = np.einsum("...ij,...jd->...id", probs, v)
    lse = (row_max + np.log(row_sum))[..., 0]
    return out, lse, probs


def causal_attention_backward(probs, q, k, v, dout, scale, apply_scale=True, dtype=np.float64):
    """VJP of causal attention given the forward probabilities.

    dV = Pᵀ·dO, dP = dO·Vᵀ, dS = P ⊙ (dP − rowsum(dP ⊙ P)), dQ = dS·K, dK = dSᵀ·Q
    (test_mha_golden_model.py:75-91; model/gpt.py:672-680).  With ``apply_scale`` dS is
    multiplied by ``scale`` as the production backward does (model/gpt.py:677); without it the
    result matches the golden model, which leaves the scale out.
    Returns ``(dq, dk, dv, ds)``.
    """
    p = np.asarray(probs, dtype=dtype)
    do = np.asarray(dout, dtype=dtype)
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    T = q.shape[-2]
    mask = causal_mask(T)
    dv = np.einsum("...ij,...id->...jd", p, do)
    dp = np.einsum("...id,...jd->...ij", do, v)
    row_dot = np.sum(dp * p * mask, axis=-1, keepdims=True)
    ds = np.where(mask, p * (dp - row_dot), 0.0)
    if apply_scale:
        ds = ds * dtype(scale)
    dq = np.einsum("...ij,...jd->...id", ds, k)
    dk = np.einsum("...ij,...id->...jd", ds, q)
    return dq, dk, dv, ds


def split_heads(qkv, B, T, NH, D):
    """[B·T, 3C] with columns [Q | K | V], each NH consecutive D-chunks, -> three
    [B, NH, T, D] arrays (split_heads_kernel, core/mha_kernels.py:534-558)."""
    C = NH * D
    x = np.asarray(qkv).reshape(B, T, 3, NH, D)
    q = np.ascontiguousarray(x[:, :, 0].transpose(0, 2, 1, 3))
    k = np.ascontiguousarray(x[:, :, 1].transpose(0, 2, 1, 3))
    v = np.ascontiguousarray(x[:, :, 2].transpose(0, 2, 1, 3))
    assert q.shape == (B, NH, T, D) and C * 3 == np.asarray(qkv).shape[-1]
    return q, k, v


def merge_heads(ctx_heads, B, T, NH, D):
    """[B, NH, T, D] -> [B·T, NH·D] (merge_heads_kernel, core/mha_kernels.py:567-584)."""
    return np.ascontiguousarray(np.asarray(ctx_heads).reshape(B, NH, T, D)
                                .transpose(0, 2, 1, 3).reshape(B * T, NH * D))


def linear(x, w, b, dtype=np.float64):
    """``C = A·B + bias`` with the bias added after the dot (core/kernels.py:132-138)."""
    return np.asarray(x, dtype=dtype) @ np.asarray(w, dtype=dtype) + np.asarray(b, dtype=dtype)


def mha_forward(x, w_qkv, b_qkv, w_o, b_o, B, T, NH, dtype=np.float64):
    """``MultiHeadAttention.forward`` (model/gpt.py:531-631) on host arrays.

    Returns ``(out, cache)``; ``cache`` holds what the reference keeps for backward
    (model/gpt.py:554-619): input, q/k/v as [B, NH, T, D], probs, merged context, plus the lse.
    """
    C = np.asarray(x).shape[1]
    D = C // NH
    scale = 1.0 / np.sqrt(D)
    qkv = linear(x, w_qkv, b_qkv, dtype)
    q, k, v = split_heads(qkv, B, T, NH, D)
    o, lse, probs = causal_attention_forward(q, k, v, scale, dtype)
    ctx = merge_heads(o, B, T, NH, D)
    out = linear(ctx, w_o, b_o, dtype)
    cache = dict(input=np.asarray(x, dtype=dtype), q=q, k=k, v=v, probs=probs, lse=lse,
                 context=ctx, o=o)
    return out, cache


def mha_backward(cache, dout, w_qkv, w_o, B, T, NH, dtype=np.float64):
    """``MultiHeadAttention.backward`` math (model/gpt.py:652-689), same order of operations.

    Returns ``(d_in, d_attn_w, d_attn_b, d_proj_w, d_proj_b)``.
    """
    dout = np.asarray(dout, dtype=dtype)
    w_qkv = np.asarray(w_qkv, dtype=dtype)
    w_o = np.asarray(w_o, dtype=dtype)
    C = dout.shape[1]
    D = C // NH
    M = B * T
    ctx = np.asarray(cache["context"], dtype=dtype)
    attn = np.asarray(cache["probs"], dtype=dtype)
    q = np.asarray(cache["q"], dtype=dtype)
    k = np.asarray(cache["k"], dtype=dtype)
    v = np.asarray(cache["v"], dtype=dtype)

    d_proj_w = ctx.T @ dout                                                  # gpt.py:666
    d_proj_b = np.sum(dout, axis=0)                                          # gpt.py:667
    d_ctx = dout @ w_o.T                                                     # gpt.py:669
    d_ctx = np.ascontiguousarray(d_ctx.reshape(B, T, NH, D).transpose(0, 2, 1, 3))
    d_attn = np.einsum("bhtd,bhsd->bhts", d_ctx, v, optimize=True)           # gpt.py:672
    d_v = np.einsum("bhts,bhtd->bhsd", attn, d_ctx, optimize=True)           # gpt.py:673
    inner = np.sum(d_attn * attn, axis=-1, keepdims=True)                    # gpt.py:675
    d_scores = (d_attn - inner) * attn                                       # gpt.py:676
    d_scores *= dtype(1.0 / np.sqrt(D))                                      # gpt.py:677
    d_q = np.einsum("bhts,bhsd->bhtd", d_scores, k, optimize=True)           # gpt.py:679
    d_k = np.einsum("bhts,bhtd->bhsd", d_scores, q, optimize=True)           # gpt.py:680
    d_q_seq = d_q.transpose(0, 2, 1, 3).reshape(B, T, C)
    d_k_seq = d_k.transpose(0, 2, 1, 3).reshape(B, T, C)
    d_v_seq = d_v.transpose(0, 2, 1, 3).reshape(B, T, C)
    d_qkv = np.concatenate([d_q_seq, d_k_seq, d_v_seq], axis=2).reshape(M, C * 3)  # gpt.py:682-685
    x = np.asarray(cache["input"], dtype=dtype)
    d_attn_w = x.T @ d_qkv                                                   # gpt.py:687
    d_attn_b = np.sum(d_qkv, axis=0)                                         # gpt.py:688
    d_in = d_qkv @ w_qkv.T                                                   # gpt.py:689
    return d_in, d_attn_w, d_attn_b, d_proj_w, d_proj_b


def decode_attention(q, k_cache, v_cache, scale, dtype=np.float64):
    """One new query row per (batch, head) attending over an L-token cached prefix.

    q: [B, NH, D]; k_cache/v_cache: [B, NH, L, D].  The new token is the last position of the
    causal sequence, so every cached key is visible: this equals the last row of
    ``causal_attention_forward`` (the row generate.py:628 keeps after a full re-forward).
    Returns ``(out [B, NH, D], lse [B, NH])``.
    """
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k_cache, dtype=dtype)
    v = np.asarray(v_cache, dtype=dtype)
    s = np.einsum("bhd,bhld->bhl", q, k) * dtype(scale)
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp(s - m)
    z = np.sum(e, axis=-1, keepdims=True)
    out = np.einsum("bhl,bhld->bhd", e / z, v)
    return out, (m + np.log(z))[..., 0]


def layernorm(x, gamma, beta, eps=1e-5, dtype=np.float64):
    """Row LayerNorm as layernorm_kernel (core/kernels.py:75-110): per row, mean = sum / C, then
    the biased variance sum((x - mean)^2) / C in a second pass, rstd = 1 / sqrt(var + 1e-5) (the
    kernel's rsqrtf), y = (x - mean) * rstd * gamma + beta.  The reference has this only as CUDA
    source; tests/test_gpu_reference_kernels.py runs that source next to this restatement."""
    x = np.asarray(x, dtype=dtype)
    mean = x.mean(axis=-1, keepdims=True)
    var = ((x - mean) ** 2).mean(axis=-1, keepdims=True)
    return (x - mean) / np.sqrt(var + dtype(eps)) * np.asarray(gamma, dtype) + np.asarray(beta, dtype)


def layernorm_backward(dy, x, gamma, eps=1e-5, dtype=np.float64):
    """layernorm_backward_kernel (core/kernels.py:361-416): mean and variance recomputed per row,
    x_hat = (x - mean) * rstd, g = dy * gamma, dx = rstd / C * (C * g - sum(g) - x_hat * sum(g * x_hat)),
    dgamma = sum over rows of dy * x_hat, dbeta = sum over rows of dy.  Returns (dx, dgamma, dbeta)."""
    x = np.asarray(x, dtype=dtype)
    dy = np.asarray(dy, dtype=dtype)
    C = x.shape[-1]
    mean = x.mean(axis=-1, keepdims=True)
    rstd = 1.0 / np.sqrt(((x - mean) ** 2).mean(axis=-1, keepdims=True) + dtype(eps))
    xh = (x - mean) * rstd
    g = dy * np.asarray(gamma, dtype)
    dx = rstd / C * (C * g - g.sum(-1, keepdims=True) - xh * (g * xh).sum(-1, keepdims=True))
    return dx, (dy * xh).sum(0), dy.sum(0)


# The tanh form of GELU the reference uses in activation_kernel and gelu_backward_kernel
# (core/kernels.py:243-248, :432-440; model/gpt.py:403-410): sqrt(2/pi) and 3 * 0.044715.
GELU_K0 = 0.7978845608
GELU_K1 = 0.044715
GELU_K1x3 = 0.134145


def gelu(x, dtype=np.float64):
    """activation_kernel (core/kernels.py:237-250): 0.5 x (1 + tanh(K0 (x + K1 x^3)))."""
    x = np.asarray(x, dtype=dtype)
    return 0.5 * x * (1.0 + np.tanh(GELU_K0 * (x + GELU_K1 * x ** 3)))


def gelu_grad(x, dtype=np.float64):
    """d gelu / dx as FeedForward's NumPy backward writes it (model/gpt.py:403-410) and
    gelu_backward_kernel computes it (core/kernels.py:424-447)."""
    x = np.asarray(x, dtype=dtype)
    t = np.tanh(GELU_K0 * (x + GELU_K1 * x ** 3))
    return 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * (GELU_K0 * (1.0 + GELU_K1x3 * x * x))


def ffn_forward(x, w_fc, b_fc, w_proj, b_proj, dtype=np.float64):
    """FeedForward.forward (model/gpt.py:327-365): pre = x W_fc + b_fc (matmul_2d_kernel, bias after
    the dot), act = gelu(pre) in place, out = act W_proj + b_proj.  Returns (out, cache) with the
    three cached activations of the reference (cache_input, cache_pre_act, cache_activated)."""
    x = np.asarray(x, dtype=dtype)
    pre = linear(x, w_fc, b_fc, dtype)
    act = gelu(pre, dtype)
    out = linear(act, w_proj, b_proj, dtype)
    return out, dict(x=x, pre=pre, act=act)


def ffn_backward(cache, dout, w_fc, w_proj, dtype=np.float64):
    """FeedForward.backward's NumPy path (model/gpt.py:381-426) step for step:
    dProjW = act^T dOut, dProjB = sum(dOut), dHidden = dOut W_proj^T, dPre = dHidden * gelu'(pre),
    dFcW = x^T dPre, dFcB = sum(dPre), dIn = dPre W_fc^T.
    Returns (dIn, dFcW, dFcB, dProjW, dProjB)."""
    dout = np.asarray(dout, dtype=dtype)
    w_fc = np.asarray(w_fc, dtype=dtype)
    w_proj = np.asarray(w_proj, dtype=dtype)
    d_proj_w = cache["act"].T @ dout
    d_proj_b = dout.sum(0)
    d_pre = (dout @ w_proj.T) * gelu_grad(cache["pre"], dtype)
    d_fc_w = cache["x"].T @ d_pre
    d_fc_b = d_pre.sum(0)
    d_in = d_pre @ w_fc.T
    return d_in, d_fc_w, d_fc_b, d_proj_w, d_proj_b


def rel_err(actual, ref) -> float:
    """max|actual - ref| / max|ref|: the per-tensor relative error the tolerances are stated in."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    denom = float(np.max(np.abs(r))) if r.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(a))) if a.size else 0.0
    return float(np.max(np.abs(a - r)) / denom)


def make_config_inputs(cfg: int, B: int, T: int, C: int, NH: int, seed: int | None = None):
    """Seeded synthetic inputs of one attention configuration:
    x ~ N(0,1), Wqkv/Wo ~ N(0,0.02), biases 0, upstream grad dY ~ N(0,1),
    generator ``np.random.default_rng(1000 + cfg)``.  All fp32 [B·T, C] / [C, 3C] / [C, C]."""
    rng = np.random.default_rng(1000 + cfg if seed is None else seed)
    x = rng.standard_normal((B * T, C), dtype=np.float32)
    w_qkv = (rng.standard_normal((C, 3 * C), dtype=np.float32) * np.float32(0.02))
    w_o = (rng.standard_normal((C, C), dtype=np.float32) * np.float32(0.02))
    dy = rng.standard_normal((B * T, C), dtype=np.float32)
    return dict(x=x, w_qkv=w_qkv, b_qkv=np.zeros(3 * C, np.float32), w_o=w_o,
                b_o=np.zeros(C, np.float32), dy=dy)
