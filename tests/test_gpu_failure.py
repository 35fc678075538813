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
