"""The library's two modules inside a transformer block and a short training loop.

Mirrors the reference's integration smoke run (smoke_train_mha_integration.py: 2 layers, 4 heads,
B=2, T=16, C=32, 5 steps, all losses finite). The block is TransformerBlock.forward/backward
(model/gpt.py:754-838) written with the fused residual forms: x += attn(ln_1(x)); x += mlp(ln_2(x))
and, backward, dX += LN_bwd(sublayer_bwd(dX)), MLP first. The embedding, readout, loss and
optimizer are outside the library and are plain torch here (test scaffolding).
"""
import numpy as np
import pytest

from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    return torch


class _Block:
    def __init__(self, pkg, C, NH, T, prec, rng):
        torch = _torch()
        cfg = pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T, attention_precision=prec)
        self.attn = pkg.MultiHeadAttention(cfg)
        self.mlp = pkg.FeedForward(cfg)
        for p in (self.attn.c_attn_b, self.attn.c_proj_b, self.mlp.c_fc_b, self.mlp.c_proj_b):
            p.weights.copy_(torch.from_numpy((0.1 * rng.standard_normal(p.shape)).astype(np.float32)))
        mk = lambda a: torch.from_numpy(a.astype(np.float32)).cuda()  # noqa: E731
        self.g1, self.b1 = mk(1 + 0.1 * rng.standard_normal(C)), mk(0.1 * rng.standard_normal(C))
        self.g2, self.b2 = mk(1 + 0.1 * rng.standard_normal(C)), mk(0.1 * rng.standard_normal(C))
        self.dg1, self.db1, self.dg2, self.db2 = (torch.zeros(C, device="cuda") for _ in range(4))

    def forward(self, x, B, T):
        self.attn.forward_residual(x, B, T, self.g1, self.b1)
        self.mlp.forward_residual(x, B, T, self.g2, self.b2)

    def backward(self, d, B, T):
        self.mlp.backward_residual(d, B, T, self.g2, self.dg2, self.db2)
        self.attn.backward_residual(d, B, T, self.g1, self.dg1, self.db1)

    def params(self):
        return [(p.weights, p.grads) for p in (self.attn.c_attn_w, self.attn.c_attn_b, self.attn.c_proj_w,
                                               self.attn.c_proj_b, self.mlp.c_fc_w, self.mlp.c_fc_b,
                                               self.mlp.c_proj_w, self.mlp.c_proj_b)] + \
               [(self.g1, self.dg1), (self.b1, self.db1), (self.g2, self.dg2), (self.b2, self.db2)]


@pytest.mark.parametrize("prec,tol", [("fp32", 1e-5), ("bf16", 2e-2)])
def test_block_matches_oracle(pkg, cuda_dev, prec, tol):
    """One block forward + backward against the oracle's unfused sequence of the same block."""
    torch = _torch()
    B, T, C, NH = 2, 40, 64, 4
    rng = np.random.default_rng(91)
    np.random.seed(91)
    blk = _Block(pkg, C, NH, T, prec, rng)
    x = rng.standard_normal((B * T, C)).astype(np.float32)
    dy = rng.standard_normal((B * T, C)).astype(np.float32)
    gx, gd = torch.from_numpy(x.copy()).cuda(), torch.from_numpy(dy.copy()).cuda()
    blk.forward(gx, B, T)
    blk.backward(gd, B, T)
    torch.cuda.synchronize()
    h = lambda t: t.detach().cpu().numpy().astype(np.float64)  # noqa: E731
    a, m = blk.attn, blk.mlp
    w = dict(wqkv=h(a.c_attn_w.weights), bqkv=h(a.c_attn_b.weights), wo=h(a.c_proj_w.weights), bo=h(a.c_proj_b.weights),
             wfc=h(m.c_fc_w.weights), bfc=h(m.c_fc_b.weights), wpr=h(m.c_proj_w.weights), bpr=h(m.c_proj_b.weights))
    g1, b1, g2, b2 = h(blk.g1), h(blk.b1), h(blk.g2), h(blk.b2)
    # oracle: x1 = x + attn(ln_1(x)); x2 = x1 + mlp(ln_2(x1)) and the backward in the block's order
    ao, ac = O.mha_forward(O.layernorm(x, g1, b1), w["wqkv"], w["bqkv"], w["wo"], w["bo"], B, T, NH)
    x1 = x + ao
    fo, fc = O.ffn_forward(O.layernorm(x1, g2, b2), w["wfc"], w["bfc"], w["wpr"], w["bpr"])
    x2 = x1 + fo
    dln2, dfw, dfb, dpw, dpb = O.ffn_backward(fc, dy, w["wfc"], w["wpr"])
    dx1_ln, dg2, db2 = O.layernorm_backward(dln2, x1, g2)
    dx1 = dy + dx1_ln
    dln1, daw, dab, dow, dob = O.mha_backward(ac, dx1, w["wqkv"], w["wo"], B, T, NH)
    dx_ln, dg1, db1 = O.layernorm_backward(dln1, x, g1)
    want = dict(x2=(gx, x2), dx=(gd, dx1 + dx_ln), d_attn_w=(a.c_attn_w.grads, daw), d_attn_b=(a.c_attn_b.grads, dab),
                d_attn_proj_w=(a.c_proj_w.grads, dow), d_fc_w=(m.c_fc_w.grads, dfw), d_fc_b=(m.c_fc_b.grads, dfb),
                d_mlp_proj_w=(m.c_proj_w.grads, dpw), d_mlp_proj_b=(m.c_proj_b.grads, dpb),
                dg1=(blk.dg1, dg1), db1=(blk.db1, db1), dg2=(blk.dg2, dg2), db2=(blk.db2, db2))
    for k, (got, ref) in want.items():
        assert O.rel_err(h(got), ref) < tol, (k, O.rel_err(h(got), ref))
    assert pkg.lib.attn_device_error(1) == 0


@pytest.mark.parametrize("prec", ["fp32", "bf16"])
def test_two_block_training_smoke(pkg, cuda_dev, prec):
    """smoke_train_mha_integration.py's shape: 2 blocks, 4 heads, B=2, T=16, C=32, 5 steps.  A
    regression readout on the last block (torch) gives the loss; SGD on every parameter of both
    blocks.  All losses finite, and the loss falls."""
    torch = _torch()
    B, T, C, NH, steps = 2, 16, 32, 4, 5
    rng = np.random.default_rng(777)
    np.random.seed(777)
    blocks = [_Block(pkg, C, NH, T, prec, rng) for _ in range(2)]
    gen = torch.Generator(device="cuda")
    gen.manual_seed(778)
    x0 = torch.randn((B * T, C), generator=gen, device="cuda")
    w_out = 0.2 * torch.randn((C, 8), generator=gen, device="cuda")
    target = torch.randn((B * T, 8), generator=gen, device="cuda")
    losses = []
    for _ in range(steps):
        x = x0.clone()
        for blk in blocks:
            blk.forward(x, B, T)
        y = x @ w_out
        diff = y - target
        losses.append(float((diff * diff).mean()))
        d = (2.0 / diff.numel()) * diff @ w_out.t()  # dL/dx
        d = d.contiguous()
        for blk in reversed(blocks):
            blk.backward(d, B, T)
        with torch.no_grad():
            for blk in blocks:
                for wt, gr in blk.params():
                    wt.sub_(0.05 * gr)
    torch.cuda.synchronize()
    assert all(np.isfinite(losses)), losses
    assert losses[-1] < losses[0], losses
    assert pkg.lib.attn_device_error(1) == 0
