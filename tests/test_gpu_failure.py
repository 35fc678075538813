"""Failure detection on the GPU without a fault: a bounded wait that runs out reports and returns.

Every mbarrier wait in the tensor-core kernels has a time limit; a wait that reaches it records
its site in the library's device error word and the kernel skips its remaining work and returns
(no trap, no hang).  attn_wait_selftest runs that path on purpose: one warp waits for an mbarrier
arrival that nothing ever makes, with a 20 ms limit.  The test reads the recorded code, and then
checks that the context still runs the library's kernels correctly.
"""
import time

import numpy as np
import pytest

from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_reports_and_leaves_the_context_usable(pkg, cuda_dev):
    import torch
    L = pkg.lib
    L.attn_device_error(1)  # start from a clear word
    assert L.attn_device_error(0) == 0
    t0 = time.perf_counter()
    assert L.attn_wait_selftest(20000, None) == 0
    code = L.attn_device_error(1)  # synchronises, then clears
    waited = time.perf_counter() - t0
    assert code == pkg._lib.ATTN_SELFTEST_SITE
    assert waited >= 0.015, waited  # the wait held for about its limit before giving up
    assert L.attn_device_error(0) == 0
    # the context is intact: a tensor-core GEMM and an attention step run and are right
    rng = np.random.default_rng(3)
    a = torch.from_numpy(rng.standard_normal((256, 128)).astype(np.float32)).bfloat16().cuda()
    b = torch.from_numpy(rng.standard_normal((128, 512)).astype(np.float32)).bfloat16().cuda()
    c = torch.empty((256, 512), device="cuda")
    pkg.mha_ops.gemm(a.data_ptr(), 128, False, b.data_ptr(), 512, False, torch.bfloat16, c.data_ptr(), 512,
                     torch.float32, 256, 512, 128)
    torch.cuda.synchronize()
    want = a.float().cpu().numpy().astype(np.float64) @ b.float().cpu().numpy().astype(np.float64)
    assert O.rel_err(c.cpu().numpy(), want) < 1e-3
    inp = O.make_config_inputs(5, 2, 130, 128, 2)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=128, num_heads=2, max_len=130,
                                                attention_precision="bf16"))
    for p, k in ((attn.c_attn_w, "w_qkv"), (attn.c_attn_b, "b_qkv"), (attn.c_proj_w, "w_o"), (attn.c_proj_b, "b_o")):
        p.weights.copy_(torch.from_numpy(inp[k]))
    out = attn.forward(torch.from_numpy(inp["x"]).cuda(), 2, 130)
    attn.backward(torch.from_numpy(inp["dy"]).cuda(), 2, 130).free()
    torch.cuda.synchronize()
    ref, _ = O.mha_forward(inp["x"], inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], 2, 130, 2)
    assert O.rel_err(out.get(), ref) < 2e-2
    assert L.attn_device_error(0) == 0


def test_selftest_rejects_bad_limits(pkg, cuda_dev):
    L = pkg.lib
    before = pkg.launch_count()
    assert L.attn_wait_selftest(0, None) == -1
    assert L.attn_wait_selftest(2000000, None) == -1
    assert pkg.launch_count() == before


def _bf16_module(pkg, B, T, C, NH, seed):
    import torch
    inp = O.make_config_inputs(seed, B, T, C, NH)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision="bf16"))
    for p, k in ((attn.c_attn_w, "w_qkv"), (attn.c_attn_b, "b_qkv"), (attn.c_proj_w, "w_o"), (attn.c_proj_b, "b_o")):
        p.weights.copy_(torch.from_numpy(inp[k]))
    return attn, inp


def test_module_raises_at_its_next_call_after_a_wait_gave_up(pkg, cuda_dev):
    """A kernel whose bounded wait gave up inside a module call makes the module's next call raise
    DeviceWaitError (the reference raises on a failed launch, model/gpt.py:649-650); after
    clear_device_error() the module computes correctly again."""
    import torch
    B, T, C, NH = 2, 130, 128, 2
    pkg.clear_device_error()
    attn, inp = _bf16_module(pkg, B, T, C, NH, 5)
    x, dy = torch.from_numpy(inp["x"]).cuda(), torch.from_numpy(inp["dy"]).cuda()
    # a forward whose stream also runs a wait that gives up (as a timed-out kernel of that call would)
    assert pkg.lib.attn_wait_selftest(20000, torch.cuda.current_stream().cuda_stream) == 0
    attn.forward(x, B, T).free()  # its status copy, enqueued after its kernels, sees the code
    torch.cuda.synchronize()
    with pytest.raises(pkg.DeviceWaitError) as ei:
        attn.backward(dy, B, T)
    assert ei.value.site == pkg._lib.ATTN_SELFTEST_SITE
    with pytest.raises(pkg.DeviceWaitError):
        attn.wait_grad_sync()
    assert pkg.clear_device_error() == pkg._lib.ATTN_SELFTEST_SITE
    out = attn.forward(x, B, T)
    din = attn.backward(dy, B, T)
    attn.wait_grad_sync()
    torch.cuda.synchronize()
    ref, cache = O.mha_forward(inp["x"], inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], B, T, NH)
    ref_din, *_ = O.mha_backward(cache, inp["dy"], inp["w_qkv"], inp["w_o"], B, T, NH)
    assert O.rel_err(out.get(), ref) < 2e-2
    assert O.rel_err(din.get(), ref_din) < 2e-2
    assert pkg.lib.attn_device_error(0) == 0


def test_a_code_left_in_the_word_does_not_cut_later_launches_short(pkg, cuda_dev):
    """With the status word still holding an earlier code, a tensor-core attention forward and
    backward over long rows (T = 4096: the backward's drain warps wait far longer than the 0.2 ms
    between a wait's checks of the word) still run to completion and are correct."""
    import torch
    pkg.clear_device_error()
    assert pkg.lib.attn_wait_selftest(20000, torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    B, NH, T, D = 1, 2, 4096, 64
    rng = np.random.default_rng(11)
    q, k, v, do = (torch.from_numpy(rng.standard_normal((B, NH, T, D)).astype(np.float32)).bfloat16().cuda()
                   for _ in range(4))
    ops = pkg.mha_ops
    hv = lambda t: ops.HeadView.heads(t.data_ptr(), NH, T, D)  # noqa: E731
    o = torch.empty_like(q)
    lse = torch.empty((B, NH, T), dtype=torch.float32, device="cuda")
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    scale = 1.0 / np.sqrt(D)
    ops.attention_forward(hv(q), hv(k), hv(v), hv(o), lse, B, NH, T, D, scale, torch.bfloat16)
    ops.attention_backward(hv(q), hv(k), hv(v), hv(o), hv(do), lse, hv(dq), hv(dk), hv(dv), B, NH, T, D, scale,
                           torch.bfloat16)
    torch.cuda.synchronize()
    assert pkg.lib.attn_device_error(0) == pkg._lib.ATTN_SELFTEST_SITE  # only the self-test's code
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ro, _, probs = O.causal_attention_forward(f(q), f(k), f(v), scale)
    rdq, rdk, rdv, _ = O.causal_attention_backward(probs, f(q), f(k), f(v), f(do), scale)
    for got, want in ((o, ro), (dq, rdq), (dk, rdk), (dv, rdv)):
        assert O.rel_err(f(got), want) < 2e-2
    assert pkg.clear_device_error() == pkg._lib.ATTN_SELFTEST_SITE
