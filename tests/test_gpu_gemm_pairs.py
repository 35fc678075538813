"""The tensor-core GEMM on CTA pairs (256x256 tiles per pair of SMs, tcgen05.mma.cta_group::2),
which the library runs when ATTN_GEMM_PAIRS=1 is set before its first GEMM.  A child process with
that setting runs every operand layout, ragged M and N (including a pair whose second CTA has no
rows left), K splits with fp32 reduce-adds, bf16 outputs, a bias, accumulation and the two
activation epilogues.  It checks each result against float64 and against the one-CTA kernel of a
second library copy, which the process loads without the setting: bit-identical for bf16 outputs
(never split along K), within float32 rounding for the rest.
"""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent(r"""
    import ctypes, importlib, os, shutil, sys, tempfile
    import numpy as np
    import torch
    sys.path.insert(0, ROOT)
    pkg = importlib.import_module("llm-gpu-5_b200")
    # the library reads ATTN_GEMM_PAIRS at its first GEMM: make one (256 rows, a pair's tile) now,
    # then unset it for a second copy of the library, loaded under another name
    w = torch.zeros((256, 256), dtype=torch.bfloat16, device="cuda")
    o = torch.empty((256, 256), dtype=torch.float32, device="cuda")
    assert pkg.lib.attn_gemm(w.data_ptr(), 256, 0, w.data_ptr(), 256, 0, 1, o.data_ptr(), 256, 0, None,
                             256, 256, 256, 0, torch.cuda.current_stream().cuda_stream) == 0
    os.environ.pop("ATTN_GEMM_PAIRS")
    tmp = tempfile.mkdtemp()
    single_path = os.path.join(tmp, "libattn_single.so")
    shutil.copy(pkg.LIB_PATH, single_path)
    single = ctypes.CDLL(single_path)
    for fn, (res, args) in pkg._lib.SIGNATURES.items():
        f = getattr(single, fn); f.restype = res; f.argtypes = args
    paired = pkg.lib
    BF, F32 = 1, 0
    s = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(7)

    def bf(a):
        return torch.from_numpy(a).cuda().bfloat16()

    def run(L, A, lda, at, Bm, ldb, bt, C, ldc, cd, bias, M, N, K, acc, act=0, aux=None):
        if act:
            rc = L.attn_gemm_act(A.data_ptr(), lda, at, Bm.data_ptr(), ldb, bt, BF, C.data_ptr(), ldc, cd,
                                 None if bias is None else bias.data_ptr(), M, N, K, act,
                                 None if aux is None else aux.data_ptr(), N, cd, s)
        else:
            rc = L.attn_gemm(A.data_ptr(), lda, at, Bm.data_ptr(), ldb, bt, BF, C.data_ptr(), ldc, cd,
                             None if bias is None else bias.data_ptr(), M, N, K, acc, s)
        assert rc == 0, L.attn_last_error_string()

    cases = [  # M, N, K, at, bt, c dtype, bias, accumulate
        (1024, 2304, 768, 0, 1, BF, True, 0),    # the QKV projection's layout
        (1024, 768, 768, 0, 1, F32, True, 0),    # the output projection's
        (1024, 768, 2304, 0, 0, F32, False, 0),  # dX = dQKV W^T
        (768, 768, 8192, 1, 0, F32, False, 0),   # dWo: K splits, fp32 reduce-adds
        (769, 2304, 4096, 1, 0, F32, False, 1),  # dWqkv with the ones row (x^T rows padded to 776)
        (300, 520, 200, 0, 0, BF, True, 0),      # ragged M and N; the second pair's CTA 1 is past M
        (1000, 300, 136, 1, 1, F32, False, 0),
        (384, 256, 128, 1, 1, F32, True, 0),
    ]
    for M, N, K, at, bt, cd, use_bias, acc in cases:
        Mp = (M + 7) // 8 * 8  # a 16-byte row pitch for the transposed A
        A = rng.standard_normal((K, Mp) if at else (M, K)).astype(np.float32)
        Bm = rng.standard_normal((N, K) if bt else (K, N)).astype(np.float32)
        tA, tB = bf(A), bf(Bm)
        A64 = tA.double().cpu().numpy()[:, :M] if at else tA.double().cpu().numpy()
        B64 = tB.double().cpu().numpy()
        ref = (A64.T if at else A64) @ (B64.T if bt else B64)
        bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).cuda() if use_bias else None
        if bias is not None:
            ref = ref + bias.double().cpu().numpy()
        C0 = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).cuda()
        if acc:
            ref = ref + C0.double().cpu().numpy()
        dt = torch.bfloat16 if cd == BF else torch.float32
        outs = []
        for L in (paired, single):
            C = C0.clone().to(dt)
            run(L, tA, A.shape[1], at, tB, Bm.shape[1], bt, C, N, cd, bias, M, N, K, acc)
            torch.cuda.synchronize()
            outs.append(C.double().cpu().numpy())
        err = np.abs(outs[0] - ref).max() / np.abs(ref).max()
        assert err < (1e-2 if cd == BF else 1e-4), (M, N, K, at, bt, err)
        if cd == BF:  # no K splits: the same sums in the same order
            assert np.array_equal(outs[0], outs[1]), (M, N, K, at, bt)
    # activation epilogues (bf16 out): GELU with the pre-activation cache, and GELU' on an aux input
    M, N, K = 512, 3072, 768
    A = bf(rng.standard_normal((M, K)).astype(np.float32))
    Bm = bf(rng.standard_normal((K, N)).astype(np.float32) * 0.05)
    for act in (1, 2):
        res = []
        for L in (paired, single):
            C = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
            aux = (torch.empty((M, N), dtype=torch.bfloat16, device="cuda") if act == 1 else
                   bf(rng.standard_normal((M, N)).astype(np.float32)))
            if act == 2:
                aux.copy_(bf(np.linspace(-3, 3, M * N, dtype=np.float32).reshape(M, N)))
            run(L, A, K, 0, Bm, N, 0, C, N, BF, None, M, N, K, 0, act=act, aux=aux)
            torch.cuda.synchronize()
            res.append((C.clone(), aux.clone()))
        assert torch.equal(res[0][0], res[1][0]), act
        assert torch.equal(res[0][1], res[1][1]), act
    assert paired.attn_device_error(0) == 0 and single.attn_device_error(0) == 0
    print("pairs ok")
""")


def test_gemm_on_cta_pairs_matches_float64_and_the_single_cta_kernel():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    env = dict(os.environ, ATTN_GEMM_PAIRS="1")
    out = subprocess.run([sys.executable, "-c", f"ROOT = {ROOT!r}\n" + CHILD], env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-3000:]
    assert "pairs ok" in out.stdout
