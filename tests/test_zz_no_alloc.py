"""attn_decode_noalloc: decode for callers that cannot allocate a device workspace.

Callers whose device memory belongs to another allocator (for example a serving process that
reserved the free HBM for its KV cache up front) or thin FFI callers that hold only the q/K/V/o
pointers cannot pass attn_decode a workspace.  attn_decode_noalloc keeps the split partial states
in a fixed 4 MiB device array inside the library instead.  This test calls it through the C ABI
twice in a row, with different shapes and data so that stale contents of the shared array would
show.  Each result must be bit-identical to attn_decode's on the same inputs (attn_decode takes a
caller-allocated workspace and runs the same kernels, so any difference would come from the
shared array), and both must match the oracle's float64 decode of the same bf16 inputs at the
bf16 tolerance the other decode tests use.  It also checks that a problem too large for the array
is refused with a message and launches nothing.  The file name sorts last so that a run stopping
at the first failure has already run every other test.
"""
import ctypes
import math

import numpy as np
import pytest

from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu
BF16_TOL = 2e-2


def _noalloc(pkg, q, kc, vc, out, lse):
    B, NH, D = q.shape
    L = kc.shape[1]
    qs, ks = q.stride(), kc.stride()
    import torch
    return pkg.lib.attn_decode_noalloc(
        q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(), lse.data_ptr(), B, NH, L, D,
        qs[0], qs[1], ks[0], ks[1], ks[2], ctypes.c_float(1.0 / math.sqrt(D)), 1,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("call", [0, 1])
def test_noalloc_decode_matches_workspace_decode(pkg, cuda_dev, call):
    import torch
    for i, (B, NH, L, D) in enumerate([(64, 8, 2048, 64), (3, 5, 1000, 128)]):
        gen = torch.Generator(device="cuda")
        gen.manual_seed(100 * call + i)
        q = torch.randn((B, NH, D), generator=gen, device="cuda").to(torch.bfloat16)
        kc = torch.randn((B, L, NH, D), generator=gen, device="cuda").to(torch.bfloat16)
        vc = torch.randn((B, L, NH, D), generator=gen, device="cuda").to(torch.bfloat16)
        out = torch.empty_like(q)
        lse = torch.empty((B, NH), dtype=torch.float32, device="cuda")
        rc = _noalloc(pkg, q, kc, vc, out, lse)
        assert rc == 0, pkg.lib.attn_last_error_string().decode()
        ref_lse = torch.empty_like(lse)
        ref = pkg.mha_ops.decode(q, kc, vc, lse=ref_lse)  # the entry point with a workspace
        torch.cuda.synchronize()
        assert torch.equal(out, ref), "attn_decode_noalloc differs from attn_decode"
        assert torch.equal(lse, ref_lse)
        f = lambda t: t.float().cpu().numpy()  # noqa: E731
        want, want_lse = O.decode_attention(f(q), f(kc).transpose(0, 2, 1, 3), f(vc).transpose(0, 2, 1, 3),
                                            1.0 / math.sqrt(D))
        assert O.rel_err(f(out), want) < BF16_TOL
        assert O.rel_err(lse.cpu().numpy(), want_lse) < BF16_TOL
    assert pkg.lib.attn_device_error(1) == 0


def test_noalloc_decode_rejects_oversize(pkg, cuda_dev):
    before = pkg.launch_count()
    fake = 1 << 20  # never dereferenced: the size check fails first
    rc = pkg.lib.attn_decode_noalloc(fake, fake, fake, fake, None, 1024, 16, 4096, 128,
                                     16 * 128, 128, 4096 * 16 * 128, 16 * 128, 128,
                                     ctypes.c_float(0.1), 1, None)
    assert rc == -2
    msg = pkg.lib.attn_last_error_string().decode()
    assert "fixed array" in msg and "1048576" in msg
    assert pkg.launch_count() == before
