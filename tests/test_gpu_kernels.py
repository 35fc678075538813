"""GPU parity of the attention kernels against the oracle, through the C ABI.

Tolerances (max|Δ|/max|ref| per tensor, ``rel_err``): float32 path 1e-5; bf16 tensor-core path
2e-2, with the oracle evaluated on the same bf16-rounded inputs; tf32 tensor-core path (float32
inputs) 2e-2.  The reference's own
assert_allclose tolerance (rtol=1e-4, atol=1e-5, test_mha_golden_model.py:45) is also applied to
the float32 path on its golden fixture.
"""
import math
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
BF16_TOL = 2e-2


def _torch():
    import torch
    return torch


def _dev(a, dtype=None):
    torch = _torch()
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


def _bf16_round(a):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def _run_attention(pkg, q, k, v, do, dtype, layout):
    """q/k/v/do: float arrays [B, NH, T, D].  Returns (o, lse, dq, dk, dv) as float64 arrays."""
    torch = _torch()
    ops = pkg.mha_ops
    B, NH, T, D = q.shape
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32  # storage (tf32: float32)
    code = "tf32" if dtype == "tf32" else tdt                    # operand type of the calls
    if layout == "heads":
        def put(a):
            return _dev(a.astype(np.float32), tdt).contiguous()

        def view(t):
            return ops.HeadView.heads(t.data_ptr(), NH, T, D)

        def get(t):
            return t.float().cpu().numpy().reshape(B, NH, T, D)
        tq, tk, tv, tdo = put(q), put(k), put(v), put(do)
        to, tdq, tdk, tdv = (torch.empty_like(tq) for _ in range(4))
        qv, kv, vv, ov, dov = view(tq), view(tk), view(tv), view(to), view(tdo)
        dqv, dkv, dvv = view(tdq), view(tdk), view(tdv)
    else:  # token layout of the fused projection: one [B*T, 3C] buffer, context [B*T, C]
        C = NH * D
        qkv = np.concatenate([a.transpose(0, 2, 1, 3).reshape(B * T, C) for a in (q, k, v)], axis=1)
        tqkv = _dev(qkv.astype(np.float32), tdt).contiguous()
        tdo = _dev(do.transpose(0, 2, 1, 3).reshape(B * T, C).astype(np.float32), tdt).contiguous()
        to = torch.empty((B * T, C), dtype=tdt, device="cuda")
        tg = torch.empty((B * T, 3 * C), dtype=tdt, device="cuda")
        es = tqkv.element_size()
        tokv = lambda base: ops.HeadView.tokens(base, T, 3 * C, D)  # noqa: E731
        qv, kv, vv = (tokv(tqkv.data_ptr() + i * C * es) for i in range(3))
        dqv, dkv, dvv = (tokv(tg.data_ptr() + i * C * es) for i in range(3))
        ov = ops.HeadView.tokens(to.data_ptr(), T, C, D)
        dov = ops.HeadView.tokens(tdo.data_ptr(), T, C, D)

        def get_g(i):
            return tg[:, i * C:(i + 1) * C].float().cpu().numpy().reshape(B, T, NH, D).transpose(0, 2, 1, 3)
    lse = torch.empty((B, NH, T), dtype=torch.float32, device="cuda")
    scale = 1.0 / math.sqrt(D)
    ops.attention_forward(qv, kv, vv, ov, lse, B, NH, T, D, scale, code)
    ops.attention_backward(qv, kv, vv, ov, dov, lse, dqv, dkv, dvv, B, NH, T, D, scale, code)
    torch.cuda.synchronize()
    if layout == "heads":
        res = (get(to), lse.cpu().numpy(), get(tdq), get(tdk), get(tdv))
    else:
        o = to.float().cpu().numpy().reshape(B, T, NH, D).transpose(0, 2, 1, 3)
        res = (o, lse.cpu().numpy(), get_g(0), get_g(1), get_g(2))
    return [np.asarray(r, dtype=np.float64) for r in res]


def _oracle(q, k, v, do):
    D = q.shape[-1]
    scale = 1.0 / math.sqrt(D)
    o, lse, p = O.causal_attention_forward(q, k, v, scale)
    dq, dk, dv, _ = O.causal_attention_backward(p, q, k, v, do, scale, apply_scale=True)
    return o, lse, dq, dk, dv


def _inputs(B, NH, T, D, seed):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((B, NH, T, D)).astype(np.float32) for _ in range(4)]


@pytest.mark.parametrize("B,NH,T,D", [(1, 3, 17, 8), (2, 2, 5, 4), (2, 4, 128, 16), (1, 2, 130, 32),
                                      (1, 2, 200, 64), (1, 1, 97, 128), (2, 8, 128, 32)])
@pytest.mark.parametrize("layout", ["heads", "tokens"])
def test_attention_f32_matches_oracle(pkg, cuda_dev, B, NH, T, D, layout):
    q, k, v, do = _inputs(B, NH, T, D, seed=B * 1000 + T * 10 + D)
    got = _run_attention(pkg, q, k, v, do, "f32", layout)
    ref = _oracle(q, k, v, do)
    for name, g, r in zip(("o", "lse", "dq", "dk", "dv"), got, ref):
        assert O.rel_err(g, r) < F32_TOL, (name, O.rel_err(g, r))


@pytest.mark.parametrize("B,NH,T,D", [(1, 2, 256, 64), (2, 2, 200, 64), (1, 2, 384, 64), (1, 2, 77, 32),
                                      (2, 3, 130, 16), (1, 2, 1024, 64), (1, 1, 129, 128),
                                      # head_dim < 64 on the tensor-core kernels (TMA zero-pads to 64)
                                      (2, 4, 128, 8), (1, 3, 257, 24), (2, 2, 190, 48), (8, 8, 128, 32),
                                      # more heads than SMs: the persistent kernels loop over items
                                      (40, 4, 200, 64), (100, 4, 130, 64)])
@pytest.mark.parametrize("layout", ["heads", "tokens"])
def test_attention_bf16_matches_oracle(pkg, cuda_dev, B, NH, T, D, layout):
    q, k, v, do = (_bf16_round(a) for a in _inputs(B, NH, T, D, seed=7 + T + D))
    got = _run_attention(pkg, q, k, v, do, "bf16", layout)
    ref = _oracle(q, k, v, do)
    for name, g, r in zip(("o", "lse", "dq", "dk", "dv"), got, ref):
        assert O.rel_err(g, r) < BF16_TOL, (name, O.rel_err(g, r))


@pytest.mark.parametrize("B,NH,T,D", [(1, 2, 128, 32), (2, 2, 200, 32), (1, 2, 384, 32), (2, 3, 130, 16),
                                      (2, 4, 128, 8), (1, 3, 257, 16), (1, 2, 77, 4), (2, 2, 1024, 32),
                                      (40, 4, 200, 32), (256, 8, 128, 32)])
@pytest.mark.parametrize("layout", ["heads", "tokens"])
def test_attention_tf32_matches_oracle(pkg, cuda_dev, B, NH, T, D, layout):
    """float32 inputs with the forward on the tf32 tensor cores (head_dim <= 32; the backward runs
    the float32 CUDA-core kernels on the tf32 forward's O and lse), against the oracle on the same
    float32 inputs at 2e-2."""
    q, k, v, do = _inputs(B, NH, T, D, seed=11 + T + D)
    got = _run_attention(pkg, q, k, v, do, "tf32", layout)
    ref = _oracle(q, k, v, do)
    for name, g, r in zip(("o", "lse", "dq", "dk", "dv"), got, ref):
        assert O.rel_err(g, r) < BF16_TOL, (name, O.rel_err(g, r))
    assert pkg.lib.attn_device_error(1) == 0


@pytest.mark.parametrize("dtype,D", [("bf16", 64), ("bf16", 32), ("f32", 64), ("tf32", 32)])
def test_attention_long_rows(pkg, cuda_dev, dtype, D):
    """T = 2048 (16 key tiles per row) with large scores whose row maximum keeps growing along the
    keys: the forward's lazy rescaling (the running max moves only when it grows by more than 2^8)
    and the backward over many key tiles, against the oracle."""
    B, NH, T = 1, 2, 2048
    rng = np.random.default_rng(2048 + D)
    q, k, v, do = (2.5 * rng.standard_normal((B, NH, T, D)) for _ in range(4))
    u = rng.standard_normal(D)
    u /= np.linalg.norm(u)
    q += 2.0 * u
    k += (4.0 * np.arange(T) / T)[None, None, :, None] * u  # later keys score higher
    q, k, v, do = (a.astype(np.float32) for a in (q, k, v, do))
    if dtype == "bf16":
        q, k, v, do = (_bf16_round(a) for a in (q, k, v, do))
    got = _run_attention(pkg, q, k, v, do, dtype, "tokens")
    ref = _oracle(q, k, v, do)
    tol = F32_TOL if dtype == "f32" else BF16_TOL
    for name, g, r in zip(("o", "lse", "dq", "dk", "dv"), got, ref):
        assert O.rel_err(g, r) < tol, (name, O.rel_err(g, r))
    assert pkg.lib.attn_device_error(1) == 0


def test_kernel_golden_fixture(pkg, cuda_dev):
    """The reference's Layer-1 golden case (seed 1337, H=3, M=17, D=8) through the fp32 kernels."""
    torch = _torch()
    g = np.load(os.path.join(GOLDEN, "kernel_h3_m17_d8.npz"))
    H, M, D = int(g["H"]), int(g["M"]), int(g["D"])
    scale = float(g["scale"])
    q, k, v, do = (g[n][None] for n in ("Q", "K", "V", "dOut"))
    o, lse, dq, dk, dv = _run_attention(pkg, q, k, v, do, "f32", "heads")
    tol = dict(rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(o[0], g["out"], **tol)
    # golden dQ/dK leave the scale out of dS (test_mha_golden_model.py:75-91); the kernels apply it
    np.testing.assert_allclose(dq[0] / scale, g["dQ"], **tol)
    np.testing.assert_allclose(dk[0] / scale, g["dK"], **tol)
    np.testing.assert_allclose(dv[0], g["dV"], **tol)
    # probabilities rebuilt from lse match the reference's cache_attn_weights semantics
    ops = pkg.mha_ops
    tq = _dev(g["Q"]).contiguous()
    tk = _dev(g["K"]).contiguous()
    tl = _dev(lse.astype(np.float32)).contiguous()
    p = ops.attention_probs(ops.HeadView.heads(tq.data_ptr(), H, M, D),
                            ops.HeadView.heads(tk.data_ptr(), H, M, D), tl, 1, H, M, D, scale,
                            torch.float32)
    np.testing.assert_allclose(p.cpu().numpy()[0], g["probs"], **tol)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("B,NH,L,D", [(2, 3, 37, 16), (4, 8, 2048, 64), (1, 2, 300, 128), (3, 2, 1, 32)])
def test_decode_matches_oracle(pkg, cuda_dev, dtype, B, NH, L, D):
    torch = _torch()
    if dtype == "bf16" and D < 8:
        pytest.skip("bf16 decode needs head_dim % 8 == 0")
    rng = np.random.default_rng(L + D)
    q = rng.standard_normal((B, NH, D)).astype(np.float32)
    kc = rng.standard_normal((B, L, NH, D)).astype(np.float32)
    vc = rng.standard_normal((B, L, NH, D)).astype(np.float32)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    if dtype == "bf16":
        q, kc, vc = _bf16_round(q), _bf16_round(kc), _bf16_round(vc)
    tq, tk, tv = _dev(q, tdt), _dev(kc, tdt), _dev(vc, tdt)
    lse = torch.empty((B, NH), dtype=torch.float32, device="cuda")
    out = pkg.mha_ops.decode(tq, tk, tv, lse=lse)
    torch.cuda.synchronize()
    ref_o, ref_l = O.decode_attention(q, kc.transpose(0, 2, 1, 3), vc.transpose(0, 2, 1, 3), 1.0 / math.sqrt(D))
    tol = F32_TOL if dtype == "f32" else BF16_TOL
    assert O.rel_err(out.float().cpu().numpy(), ref_o) < tol
    assert O.rel_err(lse.cpu().numpy(), ref_l) < tol


def test_tf32_operands_drop_their_low_mantissa_bits(pkg, cuda_dev):
    """The tf32 tensor cores read a float32 operand's upper 19 bits (the low 13 mantissa bits are
    dropped, not rounded): A = 1 + 0.75 * 2^-10 (between the tf32 values 1 and 1 + 2^-10) times the
    identity gives exactly 1.  The CUDA-core backward after a tf32 forward relies on this: it
    recomputes the scores from q and k truncated the same way."""
    torch = _torch()
    n = 256
    a = torch.full((n, n), 1.0 + 0.75 * 2.0 ** -10, dtype=torch.float32, device="cuda")
    eye = torch.eye(n, dtype=torch.float32, device="cuda")
    c = torch.empty((n, n), dtype=torch.float32, device="cuda")
    for at, bt in ((False, False), (True, True)):  # K-major and MN-major operands
        pkg.mha_ops.gemm(a.data_ptr(), n, at, eye.data_ptr(), n, bt, "tf32", c.data_ptr(), n, torch.float32, n, n, n)
        torch.cuda.synchronize()
        assert torch.equal(c, torch.ones_like(c)), (at, bt, c[0, :4].tolist())


@pytest.mark.parametrize("dtype", ["f32", "tf32", "bf16"])
@pytest.mark.parametrize("M,N,K,at,bt", [(100, 72, 40, 0, 0), (256, 768, 256, 0, 0), (64, 96, 300, 1, 0),
                                         (130, 64, 96, 0, 1), (384, 256, 128, 1, 1), (1024, 2304, 768, 0, 0),
                                         (768, 2304, 4096, 1, 0), (4096, 768, 2304, 0, 1), (512, 512, 8192, 1, 0),
                                         (300, 520, 200, 0, 0), (1000, 300, 136, 1, 1), (777, 2304, 768, 0, 1)])
def test_gemm_matches_numpy(pkg, cuda_dev, dtype, M, N, K, at, bt):
    torch = _torch()
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((K, M) if at else (M, K)).astype(np.float32)
    Bm = rng.standard_normal((N, K) if bt else (K, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32  # storage
    code = "tf32" if dtype == "tf32" else tdt                    # operand type of the call
    if dtype == "bf16":
        A, Bm = _bf16_round(A), _bf16_round(Bm)
    tA, tB, tbias = _dev(A, tdt), _dev(Bm, tdt), _dev(bias)
    ref = (A.T if at else A).astype(np.float64) @ (Bm.T if bt else Bm).astype(np.float64)
    # bf16 operands are exact (fp32 accumulation); tf32 keeps 10 mantissa bits of each operand
    tol = dict(f32=F32_TOL, bf16=1e-3, tf32=5e-3)[dtype]
    for acc in (False, True):
        tC = _dev(C0.copy())
        pkg.mha_ops.gemm(tA.data_ptr(), A.shape[1], at, tB.data_ptr(), Bm.shape[1], bt, code,
                         tC.data_ptr(), N, torch.float32, M, N, K, bias=tbias.data_ptr(), accumulate=acc)
        torch.cuda.synchronize()
        want = ref + bias + (C0 if acc else 0)
        assert O.rel_err(tC.cpu().numpy(), want) < tol, (acc, O.rel_err(tC.cpu().numpy(), want))
    # bf16 output
    tCb = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    pkg.mha_ops.gemm(tA.data_ptr(), A.shape[1], at, tB.data_ptr(), Bm.shape[1], bt, code, tCb.data_ptr(), N,
                     torch.bfloat16, M, N, K)
    torch.cuda.synchronize()
    assert O.rel_err(tCb.float().cpu().numpy(), ref) < 1e-2
    assert pkg.lib.attn_device_error(1) == 0  # no bounded wait inside a kernel gave up


@pytest.mark.parametrize("M,N", [(1, 5), (1000, 33), (262144, 96), (4097, 2304)])
def test_colsum_and_cast(pkg, cuda_dev, M, N):
    torch = _torch()
    rng = np.random.default_rng(M + N)
    X = rng.standard_normal((M, N)).astype(np.float32)
    tX = _dev(X)
    out = torch.full((N,), 3.0, dtype=torch.float32, device="cuda")
    pkg.mha_ops.colsum(tX.data_ptr(), torch.float32, N, M, N, out, accumulate=True)
    torch.cuda.synchronize()
    assert O.rel_err(out.cpu().numpy(), X.astype(np.float64).sum(0) + 3.0) < 1e-5
    xb = pkg.mha_ops.cast_bf16(tX)
    torch.cuda.synchronize()
    assert torch.equal(xb, tX.to(torch.bfloat16))
    pkg.mha_ops.colsum(xb.data_ptr(), torch.bfloat16, N, M, N, out, accumulate=False)
    torch.cuda.synchronize()
    ref = _bf16_round(X).astype(np.float64).sum(0)
    assert O.rel_err(out.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("M,N", [(5, 16), (1000, 768), (333, 20)])
def test_cast_rows_ones_and_fused_bias_gradient(pkg, cuda_dev, M, N):
    """bf16(X) | 1 | 0..: the weight-gradient GEMM over N + 1 rows yields X^T G and, as its last
    row, the column sums of G (the bias gradient), exactly as a separate column-sum pass would."""
    torch = _torch()
    rng = np.random.default_rng(M * 7 + N)
    X = rng.standard_normal((M, N)).astype(np.float32)
    G = rng.standard_normal((M, 3 * N)).astype(np.float32)
    xa = pkg.mha_ops.cast_rows_ones(_dev(X))
    torch.cuda.synchronize()
    L = xa.shape[1]
    assert xa.shape[0] == M and L % 8 == 0 and N < L <= N + 8
    assert torch.equal(xa[:, :N], _dev(X).to(torch.bfloat16))
    assert torch.all(xa[:, N] == 1) and torch.all(xa[:, N + 1:] == 0)
    tg = _dev(G, torch.bfloat16)
    out = torch.empty((N + 1, 3 * N), dtype=torch.float32, device="cuda")
    pkg.mha_ops.gemm(xa.data_ptr(), L, True, tg.data_ptr(), 3 * N, False, torch.bfloat16, out.data_ptr(),
                     3 * N, torch.float32, N + 1, 3 * N, M)
    torch.cuda.synchronize()
    Xb, Gb = _bf16_round(X).astype(np.float64), _bf16_round(G).astype(np.float64)
    got = out.cpu().numpy()
    assert O.rel_err(got[:N], Xb.T @ Gb) < 1e-5
    assert O.rel_err(got[N], Gb.sum(0)) < 1e-5


def test_split_merge_heads_reference_semantics(pkg, cuda_dev):
    torch = _torch()
    B, T, NH, HD = 2, 7, 3, 4
    C = NH * HD
    qkv = np.random.default_rng(0).standard_normal((B * T, 3 * C)).astype(np.float32)
    tq = _dev(qkv)
    q, k, v = (torch.empty(B * NH * T * HD, device="cuda") for _ in range(3))
    pkg.mha_ops.split_heads(tq.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), B, T, NH, HD)
    rq, rk, rv = O.split_heads(qkv, B, T, NH, HD)
    torch.cuda.synchronize()
    assert np.array_equal(q.cpu().numpy(), rq.reshape(-1))
    assert np.array_equal(k.cpu().numpy(), rk.reshape(-1))
    assert np.array_equal(v.cpu().numpy(), rv.reshape(-1))
    ctx = torch.empty(B * T * C, device="cuda")
    pkg.mha_ops.merge_heads(q.data_ptr(), ctx.data_ptr(), B, T, NH, HD)
    torch.cuda.synchronize()
    assert np.array_equal(ctx.cpu().numpy(), O.merge_heads(rq, B, T, NH, HD).reshape(-1))
    # the same adapters by the reference's kernel names (get_shared_mha_module().get_function)
    mod = pkg.get_shared_mha_module()
    ctx2 = torch.empty_like(ctx)
    mod.get_function("merge_heads_kernel")(q, ctx2, np.int32(B), np.int32(T), np.int32(NH), np.int32(HD),
                                           block=(256, 1, 1), grid=(1, 1))
    torch.cuda.synchronize()
    assert torch.equal(ctx, ctx2)


@pytest.mark.parametrize("M,N", [(4096, 768), (1000, 33), (262144, 64)])
def test_cast_colsum_fused(pkg, cuda_dev, M, N):
    """bf16 copy plus column sums of a float32 matrix in one pass (the dY cast fused with dbo)."""
    torch = _torch()
    rng = np.random.default_rng(M + N + 1)
    X = rng.standard_normal((M, N)).astype(np.float32)
    tX = _dev(X)
    sums = torch.full((N,), 2.0, dtype=torch.float32, device="cuda")
    y = pkg.mha_ops.cast_colsum(tX, sums, accumulate=True)
    torch.cuda.synchronize()
    assert torch.equal(y, tX.to(torch.bfloat16))
    assert O.rel_err(sums.cpu().numpy(), X.astype(np.float64).sum(0) + 2.0) < 1e-5


@pytest.mark.parametrize("M,N,K,at,bt,pad", [(512, 256, 128, 0, 0, 1), (256, 256, 8192, 1, 0, 3),
                                             (384, 520, 256, 0, 1, 5)])
def test_gemm_tc_unaligned_output_pitch(pkg, cuda_dev, M, N, K, at, bt, pad):
    """Tensor-core GEMM whose output rows are not 16-byte aligned: the per-row store epilogue."""
    torch = _torch()
    rng = np.random.default_rng(M * 7 + K)
    A = _bf16_round(rng.standard_normal((K, M) if at else (M, K)).astype(np.float32))
    Bm = _bf16_round(rng.standard_normal((N, K) if bt else (K, N)).astype(np.float32))
    C0 = rng.standard_normal((M, N + pad)).astype(np.float32)
    tA, tB = _dev(A, torch.bfloat16), _dev(Bm, torch.bfloat16)
    ref = (A.T if at else A).astype(np.float64) @ (Bm.T if bt else Bm).astype(np.float64)
    for acc in (False, True):
        tC = _dev(C0.copy())
        pkg.mha_ops.gemm(tA.data_ptr(), A.shape[1], at, tB.data_ptr(), Bm.shape[1], bt, torch.bfloat16,
                         tC.data_ptr(), N + pad, torch.float32, M, N, K, accumulate=acc)
        torch.cuda.synchronize()
        got = tC.cpu().numpy()
        assert O.rel_err(got[:, :N], ref + (C0[:, :N] if acc else 0)) < 1e-3
        np.testing.assert_array_equal(got[:, N:], C0[:, N:])  # padding columns untouched
    assert pkg.lib.attn_device_error(1) == 0


@pytest.mark.parametrize("max_ctas", [1, 7, 116])
def test_gemm_on_capped_sms(pkg, cuda_dev, max_ctas):
    """attn_gemm_ex on at most max_ctas SMs (the dX GEMM beside the gradient all-reduce): the
    persistent CTAs take more tiles each.  A bf16 output has no K splits, so the result is bit for
    bit that of the uncapped launch; an fp32 weight-gradient shape (K splits chosen for the capped
    grid: none on one SM, so one fp32 accumulator over 8,192 products, about 1e-5 relative) matches
    float64 within 1e-4."""
    torch = _torch()
    rng = np.random.default_rng(max_ctas)
    M, N, K = 1024, 768, 2304
    A = _bf16_round(rng.standard_normal((M, K)).astype(np.float32))
    Bm = _bf16_round(rng.standard_normal((N, K)).astype(np.float32))
    tA, tB = _dev(A, torch.bfloat16), _dev(Bm, torch.bfloat16)
    full = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    capped = torch.empty_like(full)
    ops = pkg.mha_ops
    ops.gemm(tA.data_ptr(), K, False, tB.data_ptr(), K, True, torch.bfloat16, full.data_ptr(), N, torch.bfloat16,
             M, N, K)
    ops.gemm(tA.data_ptr(), K, False, tB.data_ptr(), K, True, torch.bfloat16, capped.data_ptr(), N,
             torch.bfloat16, M, N, K, max_ctas=max_ctas)
    torch.cuda.synchronize()
    assert torch.equal(full, capped)
    # weight gradient: C[768, 768] = A^T B over K = 8192 tokens, fp32 output with K splits
    Kt = 8192
    X = _bf16_round(rng.standard_normal((Kt, 768)).astype(np.float32))
    G = _bf16_round(rng.standard_normal((Kt, 768)).astype(np.float32))
    tX, tG = _dev(X, torch.bfloat16), _dev(G, torch.bfloat16)
    dW = torch.empty((768, 768), dtype=torch.float32, device="cuda")
    ops.gemm(tX.data_ptr(), 768, True, tG.data_ptr(), 768, False, torch.bfloat16, dW.data_ptr(), 768,
             torch.float32, 768, 768, Kt, max_ctas=max_ctas)
    torch.cuda.synchronize()
    want = X.astype(np.float64).T @ G.astype(np.float64)
    assert O.rel_err(dW.cpu().numpy(), want) < 1e-4
    assert pkg.lib.attn_device_error(1) == 0


@pytest.mark.parametrize("dtype,M,N,K,at,bt,pad", [
    ("bf16", 300, 3072, 768, False, False, 0),   # FFN c_fc shape: tensor cores, 12 column tiles
    ("bf16", 1000, 200, 64, False, True, 0),     # ragged N: partial 64-column chunks
    ("bf16", 130, 1024, 256, True, False, 0),    # MN-major A
    ("bf16", 256, 512, 128, False, False, 1),    # unaligned output pitch: CUDA-core epilogue
    ("f32", 77, 96, 40, False, False, 0),
    ("f32", 64, 256, 128, False, True, 0),
])
def test_gemm_act_gelu_matches_oracle(pkg, cuda_dev, dtype, M, N, K, at, bt, pad):
    """The feed-forward epilogues of attn_gemm_act: ATTN_ACT_GELU (activation plus the cached
    pre-activation, with and without the cache) and ATTN_ACT_GELU_BWD, against the oracle's
    tanh-GELU (activation_kernel / gelu_backward_kernel, core/kernels.py:237-250, :424-447)."""
    torch = _torch()
    ops = pkg.mha_ops
    rng = np.random.default_rng(M * 3 + N + K)
    A = rng.standard_normal((K, M) if at else (M, K)).astype(np.float32) / np.sqrt(K) * 2
    Bm = rng.standard_normal((N, K) if bt else (K, N)).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    if dtype == "bf16":
        A, Bm = _bf16_round(A), _bf16_round(Bm)
    tA, tB, tbias = _dev(A, tdt), _dev(Bm, tdt), _dev(bias)
    acc = (A.T if at else A).astype(np.float64) @ (Bm.T if bt else Bm).astype(np.float64)
    tol = F32_TOL if dtype == "f32" else 1e-2
    ld = N + pad
    for c_dt in ((tdt, torch.float32) if dtype == "bf16" else (tdt,)):
        # forward: act = gelu(acc + bias), pre = acc + bias
        act = torch.full((M, ld), 7.0, dtype=c_dt, device="cuda")
        pre = torch.full((M, ld), 7.0, dtype=c_dt, device="cuda")
        ops.gemm_act(tA.data_ptr(), A.shape[1], at, tB.data_ptr(), Bm.shape[1], bt, tdt, act.data_ptr(), ld, c_dt,
                     M, N, K, ops.ATTN_ACT_GELU, aux=pre.data_ptr(), ldaux=ld, aux_dtype=c_dt, bias=tbias.data_ptr())
        torch.cuda.synchronize()
        want_pre = acc + bias
        assert O.rel_err(pre.float().cpu().numpy()[:, :N], want_pre) < tol
        assert O.rel_err(act.float().cpu().numpy()[:, :N], O.gelu(want_pre)) < tol
        if pad:
            assert (act.float().cpu().numpy()[:, N:] == 7.0).all() and (pre.float().cpu().numpy()[:, N:] == 7.0).all()
        act2 = torch.empty((M, ld), dtype=c_dt, device="cuda")  # inference: no pre-activation cache
        ops.gemm_act(tA.data_ptr(), A.shape[1], at, tB.data_ptr(), Bm.shape[1], bt, tdt, act2.data_ptr(), ld, c_dt,
                     M, N, K, ops.ATTN_ACT_GELU, bias=tbias.data_ptr())
        torch.cuda.synchronize()
        assert torch.equal(act2[:, :N], act[:, :N])
        # backward: d = acc * gelu'(aux), aux a cached pre-activation in either dtype
        for aux_dt in (torch.float32, tdt):
            aux = (rng.standard_normal((M, ld)) * 1.5).astype(np.float32)
            if aux_dt == torch.bfloat16:
                aux = _bf16_round(aux)
            taux = _dev(aux, aux_dt)
            d = torch.full((M, ld), 7.0, dtype=c_dt, device="cuda")
            ops.gemm_act(tA.data_ptr(), A.shape[1], at, tB.data_ptr(), Bm.shape[1], bt, tdt, d.data_ptr(), ld, c_dt,
                         M, N, K, ops.ATTN_ACT_GELU_BWD, aux=taux.data_ptr(), ldaux=ld, aux_dtype=aux_dt)
            torch.cuda.synchronize()
            assert O.rel_err(d.float().cpu().numpy()[:, :N], acc * O.gelu_grad(aux[:, :N])) < tol, (c_dt, aux_dt)
    assert pkg.lib.attn_device_error(1) == 0


def test_gemm_act_rejects_bad_arguments(pkg, cuda_dev):
    torch = _torch()
    ops = pkg.mha_ops
    a = torch.zeros((64, 64), dtype=torch.bfloat16, device="cuda")
    c = torch.zeros((64, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(pkg.AttnError):  # GELU_BWD without its pre-activation
        ops.gemm_act(a.data_ptr(), 64, False, a.data_ptr(), 64, False, torch.bfloat16, c.data_ptr(), 64,
                     torch.bfloat16, 64, 64, 64, ops.ATTN_ACT_GELU_BWD)
    with pytest.raises(pkg.AttnError):  # unknown activation
        ops.gemm_act(a.data_ptr(), 64, False, a.data_ptr(), 64, False, torch.bfloat16, c.data_ptr(), 64,
                     torch.bfloat16, 64, 64, 64, 9)
    with pytest.raises(pkg.AttnError):  # aux aliasing the output
        ops.gemm_act(a.data_ptr(), 64, False, a.data_ptr(), 64, False, torch.bfloat16, c.data_ptr(), 64,
                     torch.bfloat16, 64, 64, 64, ops.ATTN_ACT_GELU, aux=c.data_ptr(), ldaux=64,
                     aux_dtype=torch.bfloat16)
