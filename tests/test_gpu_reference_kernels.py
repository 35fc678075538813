"""The library's kernels next to the reference's own CUDA kernels, on the same inputs.

``oracle/build_ref.py`` compiles the reference's kernel sources (the strings that PyCUDA compiles at
run time, core/kernels.py and core/mha_kernels.py) for sm_100a into oracle/_ref/libref_kernels.so
with launchers that use the reference's launch configurations.  These tests load that library as
the checker: ``layernorm_kernel`` (core/kernels.py:75-110) against attn_layernorm, and
``fused_attention_forward_kernel`` (core/mha_kernels.py:404-521) against attn_fwd (float32 and the
bf16 tensor-core path), attn_probs (its Scores output) and the LSE (its row_max + log row_sum).
The kernel-level backward chain of the reference's GPU golden test (matmul_score_kernel,
softmax_fused_backward, matmul_grad_q/k/v; core/mha_kernels.py:62-87, 195-236, 592-680) is run
against attn_bwd, and split_heads_kernel / merge_heads_kernel (core/mha_kernels.py:534-584)
against attn_split_heads / attn_merge_heads.  They are skipped where the reference library was
not built.
"""
import ctypes
import math
import os

import numpy as np
import pytest

from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu
REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "libref_kernels.so")


@pytest.fixture(scope="module")
def ref():
    if not os.path.exists(REF):
        pytest.skip("oracle/_ref/libref_kernels.so not built (python oracle/build_ref.py <reference>)")
    lib = ctypes.CDLL(REF)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    lib.ref_layernorm.argtypes = [P, P, P, P, I, I]
    lib.ref_layernorm.restype = I
    lib.ref_layernorm_backward.argtypes = [P, P, P, P, P, P, I, I]
    lib.ref_layernorm_backward.restype = I
    lib.ref_fused_attention_forward.argtypes = [P, P, P, P, P, P, P, I, I, I, F]
    lib.ref_fused_attention_forward.restype = I
    lib.ref_attention_backward.argtypes = [P, P, P, P, P, P, P, P, I, I, I]
    lib.ref_attention_backward.restype = I
    lib.ref_split_heads.argtypes = [P, P, P, P, I, I, I, I]
    lib.ref_split_heads.restype = I
    lib.ref_merge_heads.argtypes = [P, P, I, I, I, I]
    lib.ref_merge_heads.restype = I
    return lib


@pytest.mark.parametrize("M,C", [(1, 8), (257, 64), (1000, 768), (33, 100), (64, 2048)])
def test_layernorm_matches_reference_kernel(pkg, cuda_dev, ref, M, C):
    import torch
    rng = np.random.default_rng(M + C)
    x = (rng.standard_normal((M, C)) * 3 + 1).astype(np.float32)
    g = rng.standard_normal(C).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    tx, tg, tb = (torch.from_numpy(a).cuda() for a in (x, g, b))
    y_ref = torch.empty_like(tx)
    assert ref.ref_layernorm(tx.data_ptr(), y_ref.data_ptr(), tg.data_ptr(), tb.data_ptr(), M, C) == 0
    y = pkg.mha_ops.layernorm(tx, tg, tb)
    torch.cuda.synchronize()
    yr, yo = y_ref.cpu().numpy(), y.cpu().numpy()
    assert O.rel_err(yo, yr) < 1e-5
    # the oracle restatement agrees with the reference kernel too
    assert O.rel_err(O.layernorm(x, g, b), yr) < 1e-5
    # bf16 output with the ones column: the same values rounded, then 1, then zeros
    yb = pkg.mha_ops.layernorm(tx, tg, tb, out_dtype=torch.bfloat16, ones_col=True)
    torch.cuda.synchronize()
    assert yb.shape[1] % 8 == 0 and yb.shape[1] > C
    assert O.rel_err(yb[:, :C].float().cpu().numpy(), yr) < 1e-2
    assert torch.all(yb[:, C] == 1) and torch.all(yb[:, C + 1:] == 0)


@pytest.mark.parametrize("H,M,D", [(3, 17, 8), (4, 128, 16), (2, 200, 64), (2, 129, 32)])
def test_attention_forward_matches_reference_kernel(pkg, cuda_dev, ref, H, M, D):
    import torch
    ops = pkg.mha_ops
    rng = np.random.default_rng(H * 1000 + M + D)
    q, k, v = (rng.standard_normal((H, M, D)).astype(np.float32) for _ in range(3))
    scale = 1.0 / math.sqrt(D)
    tq, tk, tv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    scores = torch.empty((H, M, M), dtype=torch.float32, device="cuda")
    o_ref = torch.empty((H, M, D), dtype=torch.float32, device="cuda")
    rmax = torch.empty((H, M), dtype=torch.float32, device="cuda")
    rsum = torch.empty((H, M), dtype=torch.float32, device="cuda")
    assert ref.ref_fused_attention_forward(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), scores.data_ptr(),
                                           o_ref.data_ptr(), rmax.data_ptr(), rsum.data_ptr(), H, M, D, scale) == 0
    lse_ref = (rmax + torch.log(rsum)).cpu().numpy()
    # float32 path of the library, on the reference's [H, M, D] head layout
    view = lambda t: ops.HeadView.heads(t.data_ptr(), H, M, D)  # noqa: E731
    o = torch.empty_like(tq)
    lse = torch.empty((1, H, M), dtype=torch.float32, device="cuda")
    ops.attention_forward(view(tq), view(tk), view(tv), view(o), lse, 1, H, M, D, scale, torch.float32)
    p = ops.attention_probs(view(tq), view(tk), lse, 1, H, M, D, scale, torch.float32)
    torch.cuda.synchronize()
    assert O.rel_err(o.cpu().numpy(), o_ref.cpu().numpy()) < 1e-5
    assert O.rel_err(lse.cpu().numpy()[0], lse_ref) < 1e-5
    assert O.rel_err(p.cpu().numpy()[0], scores.cpu().numpy()) < 1e-5
    # bf16 tensor-core path against the same kernel on the bf16-rounded inputs
    bq, bk, bv = (t.to(torch.bfloat16) for t in (tq, tk, tv))
    fq, fk, fv = (t.float().contiguous() for t in (bq, bk, bv))
    assert ref.ref_fused_attention_forward(fq.data_ptr(), fk.data_ptr(), fv.data_ptr(), scores.data_ptr(),
                                           o_ref.data_ptr(), rmax.data_ptr(), rsum.data_ptr(), H, M, D, scale) == 0
    ob = torch.empty_like(bq)
    ops.attention_forward(view(bq), view(bk), view(bv), view(ob), lse, 1, H, M, D, scale, torch.bfloat16)
    torch.cuda.synchronize()
    assert O.rel_err(ob.float().cpu().numpy(), o_ref.cpu().numpy()) < 2e-2


@pytest.mark.parametrize("H,M,D", [(3, 17, 8), (4, 128, 16), (2, 130, 64)])
def test_attention_backward_matches_reference_kernels(pkg, cuda_dev, ref, H, M, D):
    """dQ, dK, dV of attn_bwd against the reference's own gradient kernels.  Those follow the
    golden test and leave the softmax scale out of dS, which production applies
    (model/gpt.py:677); dQ and dK are linear in dS, so the library's equal the reference's times
    the scale."""
    import torch
    ops = pkg.mha_ops
    rng = np.random.default_rng(H * 7 + M + D)
    q, k, v, do = (rng.standard_normal((H, M, D)).astype(np.float32) for _ in range(4))
    scale = 1.0 / math.sqrt(D)
    tq, tk, tv, tdo = (torch.from_numpy(a).cuda() for a in (q, k, v, do))
    probs = torch.empty((H, M, M), dtype=torch.float32, device="cuda")
    o_ref = torch.empty_like(tq)
    rmax = torch.empty((H, M), dtype=torch.float32, device="cuda")
    rsum = torch.empty((H, M), dtype=torch.float32, device="cuda")
    assert ref.ref_fused_attention_forward(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), probs.data_ptr(),
                                           o_ref.data_ptr(), rmax.data_ptr(), rsum.data_ptr(), H, M, D, scale) == 0
    rdq, rdk, rdv = (torch.empty_like(tq) for _ in range(3))
    assert ref.ref_attention_backward(tq.data_ptr(), tk.data_ptr(), tv.data_ptr(), tdo.data_ptr(), probs.data_ptr(),
                                      rdq.data_ptr(), rdk.data_ptr(), rdv.data_ptr(), H, M, D) == 0
    view = lambda t: ops.HeadView.heads(t.data_ptr(), H, M, D)  # noqa: E731
    o = torch.empty_like(tq)
    lse = torch.empty((1, H, M), dtype=torch.float32, device="cuda")
    ops.attention_forward(view(tq), view(tk), view(tv), view(o), lse, 1, H, M, D, scale, torch.float32)
    dq, dk, dv = (torch.empty_like(tq) for _ in range(3))
    ops.attention_backward(view(tq), view(tk), view(tv), view(o), view(tdo), lse, view(dq), view(dk), view(dv),
                           1, H, M, D, scale, torch.float32)
    torch.cuda.synchronize()
    assert O.rel_err(dv.cpu().numpy(), rdv.cpu().numpy()) < 1e-5
    assert O.rel_err(dq.cpu().numpy(), scale * rdq.cpu().numpy()) < 1e-5
    assert O.rel_err(dk.cpu().numpy(), scale * rdk.cpu().numpy()) < 1e-5


def test_split_merge_heads_match_reference_kernels(pkg, cuda_dev, ref):
    import torch
    B, T, NH, HD = 2, 37, 3, 16
    C = NH * HD
    qkv = torch.from_numpy(np.random.default_rng(5).standard_normal((B * T, 3 * C)).astype(np.float32)).cuda()
    outs = [torch.empty((B * NH, T, HD), dtype=torch.float32, device="cuda") for _ in range(6)]
    assert ref.ref_split_heads(qkv.data_ptr(), *(t.data_ptr() for t in outs[:3]), B, T, NH, HD) == 0
    pkg.mha_ops.split_heads(qkv.data_ptr(), *(t.data_ptr() for t in outs[3:]), B, T, NH, HD)
    ctx_ref = torch.empty((B * T, C), dtype=torch.float32, device="cuda")
    ctx = torch.empty_like(ctx_ref)
    assert ref.ref_merge_heads(outs[0].data_ptr(), ctx_ref.data_ptr(), B, T, NH, HD) == 0
    pkg.mha_ops.merge_heads(outs[0].data_ptr(), ctx.data_ptr(), B, T, NH, HD)
    torch.cuda.synchronize()
    for a, b in zip(outs[:3], outs[3:]):
        assert torch.equal(a, b)
    assert torch.equal(ctx, ctx_ref)


@pytest.mark.parametrize("M,C", [(1, 8), (300, 64), (1000, 768), (33, 100), (7, 2000), (9, 30)])
def test_layernorm_backward_matches_reference_kernel(pkg, cuda_dev, ref, M, C):
    import torch
    rng = np.random.default_rng(M * 3 + C)
    x = (rng.standard_normal((M, C)) * 2 - 0.5).astype(np.float32)
    dy = rng.standard_normal((M, C)).astype(np.float32)
    g = rng.standard_normal(C).astype(np.float32)
    tx, tdy, tg = (torch.from_numpy(a).cuda() for a in (x, dy, g))
    rdx, rdg, rdb = torch.empty_like(tx), torch.empty_like(tg), torch.empty_like(tg)
    assert ref.ref_layernorm_backward(tdy.data_ptr(), tx.data_ptr(), tg.data_ptr(), rdx.data_ptr(), rdg.data_ptr(),
                                      rdb.data_ptr(), M, C) == 0
    dx, dg, db = torch.empty_like(tx), torch.full_like(tg, 7.0), torch.full_like(tg, 7.0)
    pkg.mha_ops.layernorm_backward(tdy, tx, tg, dx, dg, db)
    torch.cuda.synchronize()
    assert O.rel_err(dx.cpu().numpy(), rdx.cpu().numpy()) < 1e-5
    assert O.rel_err(dg.cpu().numpy(), rdg.cpu().numpy()) < 1e-5
    assert O.rel_err(db.cpu().numpy(), rdb.cpu().numpy()) < 1e-5
    odx, odg, odb = O.layernorm_backward(dy, x, g)  # the restatement agrees with the kernel too
    assert O.rel_err(odx, rdx.cpu().numpy()) < 1e-5 and O.rel_err(odg, rdg.cpu().numpy()) < 1e-5
    # accumulating forms: dx += dLN (the residual branch), parameter gradients added
    base = torch.from_numpy(rng.standard_normal((M, C)).astype(np.float32)).cuda()
    dx2 = base.clone()
    pkg.mha_ops.layernorm_backward(tdy, tx, tg, dx2, dg, db, accumulate_dx=True, accumulate_params=True)
    torch.cuda.synchronize()
    assert O.rel_err(dx2.cpu().numpy(), base.cpu().numpy() + rdx.cpu().numpy()) < 1e-5
    assert O.rel_err(dg.cpu().numpy(), 2 * rdg.cpu().numpy()) < 1e-5
