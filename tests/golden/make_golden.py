"""Regenerate the golden fixtures in this folder by running the reference trainer's own Python.

Usage (needs the reference checkout, which only the build container has):

    python tests/golden/make_golden.py <reference checkout>      (or LLM_GPU5_REFERENCE=<checkout>)
    python tests/golden/make_golden.py <reference checkout> --only=checkpoint   (that archive alone)

The reference is PyCUDA code for a Kepler GPU.  Its attention *math* is plain NumPy and host
Python, so this script installs a host-memory stand-in for ``pycuda.driver`` /
``pycuda.compiler`` / ``pycuda.autoinit`` and then imports the reference unchanged:

* ``test_mha_golden_model.numpy_causal_attention_forward/backward`` (test_mha_golden_model.py:60-91)
  produce the kernel-level fixture, with the exact inputs of its Layer 1 (seed 1337, H=3, M=17,
  D=8; test_mha_golden_model.py:41-45, 98-101, 513-518);
* ``model.gpt.MultiHeadAttention`` runs its real ``forward`` (model/gpt.py:531-631) and its real
  NumPy ``backward`` (model/gpt.py:633-698).
* ``model.gpt.FeedForward`` runs its real ``forward`` (model/gpt.py:327-365) and its NumPy
  ``backward`` (``use_cpu_backward = True``, model/gpt.py:381-426), with ``activation_kernel``
  (core/kernels.py:237-250) emulated in float32 on the host; the scenario of
  test_ffn_gpu_backward.py:35-56 (seed 1337, C=16, M=6, dOut = output) and a wider one.  The four kernels ``forward`` launches are emulated on
  the host: ``matmul_2d_kernel`` (core/kernels.py:119-140), ``split_heads_kernel``
  (core/mha_kernels.py:534-558), ``merge_heads_kernel`` (core/mha_kernels.py:567-584) by their
  index arithmetic, and ``fused_attention_forward_kernel`` by the reference's own golden forward
  ``numpy_causal_attention_forward``.  The capture scenario of capture_mha_oracle.py:23-73
  (seed 4242, B=2, T=5, C=8, NH=2), whose ``.npz`` the reference does not ship, is rebuilt this way.
* ``model.gpt.GPTModel.save_checkpoint`` (model/gpt.py:1103-1176) writes ``ckpt_gpt_c16_nh2_l2.npz``
  for a small seeded model (2 layers, C=16, 2 heads, non-zero attention biases): the reference's
  own checkpoint archive, which the drop-in modules must read and write back unchanged.

Nothing here is imported by the tests; they only read the ``.npz`` files it writes.
"""

from __future__ import annotations

import os
import sys
import tempfile
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


# --------------------------------------------------------------------------------------------
# host-memory stand-in for the three pycuda modules the reference imports
# --------------------------------------------------------------------------------------------
class _HostAlloc:
    """A 'device' allocation that is a host byte array."""

    def __init__(self, nbytes):
        self.buf = np.zeros(int(nbytes), dtype=np.uint8)

    def free(self):
        self.buf = None

    def view(self, dtype, count=None):
        v = self.buf.view(dtype)
        return v if count is None else v[:count]


def _as_bytes(arr):
    return np.ascontiguousarray(arr).view(np.uint8).reshape(-1)


def _install_fake_pycuda(kernels):
    drv = types.ModuleType("pycuda.driver")
    drv.mem_alloc = _HostAlloc
    drv.DeviceAllocation = _HostAlloc

    def memcpy_htod(dst, src):
        b = _as_bytes(src)
        dst.buf[: b.size] = b

    def memcpy_dtoh(dst, src):
        out = dst.view(np.uint8).reshape(-1)
        out[:] = src.buf[: out.size]

    def memcpy_dtod(dst, src, n):
        dst.buf[: int(n)] = src.buf[: int(n)]

    def memset_d8(dst, val, n):
        dst.buf[: int(n)] = val

    drv.memcpy_htod = memcpy_htod
    drv.memcpy_dtoh = memcpy_dtoh
    drv.memcpy_dtod = memcpy_dtod
    drv.memset_d8 = memset_d8

    class Event:  # GpuProfiler-style zones are not used on this path
        def record(self, *a, **k):
            pass

        def synchronize(self):
            pass

        def time_till(self, other):
            return 0.0

    drv.Event = Event

    comp = types.ModuleType("pycuda.compiler")

    class _Module:
        def get_function(self, name):
            if name in kernels:
                return kernels[name]

            def _missing(*a, **k):
                raise RuntimeError(f"kernel {name} is not emulated on the host")

            return _missing

    comp.SourceModule = lambda src, options=None, **kw: _Module()

    pkg = types.ModuleType("pycuda")
    pkg.driver = drv
    pkg.compiler = comp
    pkg.autoinit = types.ModuleType("pycuda.autoinit")
    sys.modules["pycuda"] = pkg
    sys.modules["pycuda.driver"] = drv
    sys.modules["pycuda.compiler"] = comp
    sys.modules["pycuda.autoinit"] = pkg.autoinit


def _make_kernels(golden_mod_getter):
    """Host emulations of the four kernels MultiHeadAttention.forward launches."""

    def matmul_2d_kernel(A, Bm, bias, Cm, M, N, K, **launch):
        M, N, K = int(M), int(N), int(K)
        a = A.view(np.float32, M * K).reshape(M, K)
        b = Bm.view(np.float32, K * N).reshape(K, N)
        c = (a @ b).astype(np.float32) + bias.view(np.float32, N)
        Cm.view(np.float32, M * N)[:] = c.reshape(-1)

    def split_heads_kernel(QKV, Q, K, V, B, T, NH, HD, **launch):
        B, T, NH, HD = int(B), int(T), int(NH), int(HD)
        C = NH * HD
        idx = np.arange(B * T * NH * HD)
        hd = idx % HD
        nh = (idx // HD) % NH
        t = (idx // (HD * NH)) % T
        b = idx // (HD * NH * T)
        row = b * T + t
        col = nh * HD + hd
        out_idx = (b * NH + nh) * T * HD + t * HD + hd
        src = QKV.view(np.float32, B * T * 3 * C)
        Q.view(np.float32, idx.size)[out_idx] = src[row * 3 * C + col]
        K.view(np.float32, idx.size)[out_idx] = src[row * 3 * C + C + col]
        V.view(np.float32, idx.size)[out_idx] = src[row * 3 * C + 2 * C + col]

    def merge_heads_kernel(CH, Ctx, B, T, NH, HD, **launch):
        B, T, NH, HD = int(B), int(T), int(NH), int(HD)
        idx = np.arange(B * T * NH * HD)
        hd = idx % HD
        nh = (idx // HD) % NH
        t = (idx // (HD * NH)) % T
        b = idx // (HD * NH * T)
        in_idx = (b * NH + nh) * T * HD + t * HD + hd
        out_idx = (b * T + t) * (NH * HD) + nh * HD + hd
        Ctx.view(np.float32, idx.size)[out_idx] = CH.view(np.float32, idx.size)[in_idx]

    def fused_attention_forward_kernel(Q, K, V, Scores, Out, row_max, row_sum, H, M, D, scale,
                                       **launch):
        H, M, D = int(H), int(M), int(D)
        g = golden_mod_getter()
        g.M = M  # the golden functions read the sequence length from this module global
        q = Q.view(np.float32, H * M * D).reshape(H, M, D)
        k = K.view(np.float32, H * M * D).reshape(H, M, D)
        v = V.view(np.float32, H * M * D).reshape(H, M, D)
        scores, probs, out = g.numpy_causal_attention_forward(q, k, v, float(scale))
        Scores.view(np.float32, H * M * M)[:] = probs.reshape(-1)
        Out.view(np.float32, H * M * D)[:] = out.reshape(-1)
        mask = np.tril(np.ones((M, M), dtype=bool))
        masked = np.where(mask, scores, -np.inf)
        mx = masked.max(axis=-1)
        row_max.view(np.float32, H * M)[:] = mx.reshape(-1)
        row_sum.view(np.float32, H * M)[:] = np.where(mask, np.exp(masked - mx[..., None]), 0.0) \
            .sum(-1).astype(np.float32).reshape(-1)

    def activation_kernel(D, n, **launch):
        x = D.view(np.float32, int(n))
        inner = np.float32(0.7978845608) * (x + np.float32(0.044715) * (x * x * x))
        x[:] = np.float32(0.5) * x * (np.float32(1.0) + np.tanh(inner))

    return dict(matmul_2d_kernel=matmul_2d_kernel, activation_kernel=activation_kernel,
                split_heads_kernel=split_heads_kernel,
                merge_heads_kernel=merge_heads_kernel,
                fused_attention_forward_kernel=fused_attention_forward_kernel)


# --------------------------------------------------------------------------------------------
# fixture scenarios
# --------------------------------------------------------------------------------------------
def _kernel_level(golden):
    """Layer 1 of test_mha_golden_model.py: same seed, same draw order, same shapes."""
    H, M, D = golden.H, golden.M, golden.D
    np.random.seed(golden.SEED)
    Din = 6
    np.random.normal(0.0, 1.0, size=(H, M, Din)).astype(np.float32)          # X   (main, :513)
    np.random.normal(0.0, 1.0 / np.sqrt(Din), size=(Din, 3 * D)).astype(np.float32)  # W_qkv
    Q = np.random.normal(0.0, 1.0, size=(H, M, D)).astype(np.float32)        # :98-101
    K = np.random.normal(0.0, 1.0, size=(H, M, D)).astype(np.float32)
    V = np.random.normal(0.0, 1.0, size=(H, M, D)).astype(np.float32)
    dOut = np.random.normal(0.0, 1.0, size=(H, M, D)).astype(np.float32)
    golden.M = M
    scores, probs, out = golden.numpy_causal_attention_forward(Q, K, V, golden.SCALE)
    dV, dS, dQ, dK = golden.numpy_causal_attention_backward(probs, Q, K, V, dOut)
    np.savez(os.path.join(HERE, "kernel_h3_m17_d8.npz"), Q=Q, K=K, V=V, dOut=dOut,
             scores=scores, probs=probs, out=out, dV=dV, dScores_pre=dS, dQ=dQ, dK=dK,
             H=H, M=M, D=D, scale=np.float32(golden.SCALE))


def _run_reference_mha(gpt, cuda, B, T, C, NH, param_seed, data_seed, x=None, dout=None):
    """capture_mha_oracle.py:28-71 generalised to any shape."""
    np.random.seed(param_seed)
    config = gpt.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T)
    attn = gpt.MultiHeadAttention(config)
    rng = np.random.RandomState(data_seed)
    if x is None:
        x = rng.normal(0.0, 1.0, size=(B * T, C)).astype(np.float32)
    gx = cuda.mem_alloc(x.nbytes)
    cuda.memcpy_htod(gx, x)
    gout = attn.forward(gx, B, T)
    out = np.empty((B * T, C), np.float32)
    cuda.memcpy_dtoh(out, gout)
    if dout is None:
        dout = rng.normal(0.0, 1.0, size=(B * T, C)).astype(np.float32)
    gd = cuda.mem_alloc(dout.nbytes)
    cuda.memcpy_htod(gd, dout)
    gdin = attn.backward(gd, B, T)
    din = np.empty((B * T, C), np.float32)
    cuda.memcpy_dtoh(din, gdin)

    def dl(p):
        h = np.empty(p.shape, np.float32)
        cuda.memcpy_dtoh(h, p.gpu_grads)
        return h

    def wl(p):
        h = np.empty(p.shape, np.float32)
        cuda.memcpy_dtoh(h, p.gpu_weights)
        return h

    return dict(x=x, dy=dout, out=out, din=din,
                w_qkv=wl(attn.c_attn_w), b_qkv=wl(attn.c_attn_b),
                w_o=wl(attn.c_proj_w), b_o=wl(attn.c_proj_b),
                cache_q=attn.cache_q, cache_k=attn.cache_k, cache_v=attn.cache_v,
                cache_attn_weights=attn.cache_attn_weights, cache_context=attn.cache_context,
                d_attn_w=dl(attn.c_attn_w), d_attn_b=dl(attn.c_attn_b),
                d_proj_w=dl(attn.c_proj_w), d_proj_b=dl(attn.c_proj_b),
                B=B, T=T, C=C, NH=NH)


def _run_reference_ffn(gpt, cuda, C, M, seed, dout_seed=None, bias_scale=0.0):
    """FeedForward forward + NumPy backward.  dout_seed None: dOut = output, the synthetic loss
    0.5 * sum(out^2) of test_ffn_gpu_backward.py:51-53; otherwise dOut ~ N(0, 1)."""
    np.random.seed(seed)
    config = gpt.GPTConfig(vocab_size=64, embedding_dim=C, num_heads=2, max_len=8)
    ffn = gpt.FeedForward(config)
    if bias_scale:  # the reference initialises both biases to zero; give them values
        brng = np.random.RandomState(seed + 1)
        for p in (ffn.c_fc_b, ffn.c_proj_b):
            cuda.memcpy_htod(p.gpu_weights, brng.normal(0.0, bias_scale, size=p.shape).astype(np.float32))
    x = np.random.normal(0.0, 1.0, size=(M, C)).astype(np.float32)
    gx = cuda.mem_alloc(x.nbytes)
    cuda.memcpy_htod(gx, x)
    gout = ffn.forward(gx, 1, M)
    out = np.empty((M, C), np.float32)
    cuda.memcpy_dtoh(out, gout)
    pre = np.empty((M, 4 * C), np.float32)
    cuda.memcpy_dtoh(pre, ffn.cache_pre_act)
    act = np.empty((M, 4 * C), np.float32)
    cuda.memcpy_dtoh(act, ffn.cache_activated)
    dout = out.copy() if dout_seed is None else \
        np.random.RandomState(dout_seed).normal(0.0, 1.0, size=(M, C)).astype(np.float32)
    gd = cuda.mem_alloc(dout.nbytes)
    cuda.memcpy_htod(gd, dout)
    ffn.use_cpu_backward = True
    gdin = ffn.backward(gd, 1, M, accumulate=False)
    din = np.empty((M, C), np.float32)
    cuda.memcpy_dtoh(din, gdin)

    def dl(p, which):
        h = np.empty(p.shape, np.float32)
        cuda.memcpy_dtoh(h, getattr(p, which))
        return h

    return dict(x=x, dy=dout, out=out, pre=pre, act=act, din=din,
                w_fc=dl(ffn.c_fc_w, "gpu_weights"), b_fc=dl(ffn.c_fc_b, "gpu_weights"),
                w_proj=dl(ffn.c_proj_w, "gpu_weights"), b_proj=dl(ffn.c_proj_b, "gpu_weights"),
                d_fc_w=dl(ffn.c_fc_w, "gpu_grads"), d_fc_b=dl(ffn.c_fc_b, "gpu_grads"),
                d_proj_w=dl(ffn.c_proj_w, "gpu_grads"), d_proj_b=dl(ffn.c_proj_b, "gpu_grads"), C=C, M=M)


def _run_reference_checkpoint(gpt, cuda, path, seed):
    """The reference's own GPTModel.save_checkpoint (model/gpt.py:1103-1176) on a small seeded
    model (vocab 20, max_len 8, C=16, 2 heads, 2 layers) whose attention biases are set to
    non-zero draws first (the reference initialises them to 0), so every attention key of the
    archive carries values.  The archive it writes is the checkpoint format the drop-in modules
    must read and write back unchanged."""
    np.random.seed(seed)
    cfg = gpt.GPTConfig(vocab_size=20, max_len=8, embedding_dim=16, num_heads=2, num_layers=2)
    model = gpt.GPTModel(cfg)
    rng = np.random.default_rng(seed + 1)
    for block in model.blocks:
        for p in (block.attn.c_attn_b, block.attn.c_proj_b):
            cuda.memcpy_htod(p.gpu_weights, (0.1 * rng.standard_normal(p.shape)).astype(np.float32))
    model.save_checkpoint(path)


def main(ref_root, only=None):
    ref_root = os.path.abspath(ref_root)
    state = {}
    _install_fake_pycuda(_make_kernels(lambda: state["golden"]))
    sys.path.insert(0, ref_root)
    cwd = os.getcwd()
    work = tempfile.mkdtemp(prefix="golden_")
    os.chdir(work)  # the reference's logging_config writes output/logs relative to the CWD
    try:
        import test_mha_golden_model as golden  # noqa: E402
        import pycuda.driver as cuda  # noqa: E402  (the stand-in)
        from model import gpt  # noqa: E402
        state["golden"] = golden
        if only == "checkpoint":
            _run_reference_checkpoint(gpt, cuda, os.path.join(HERE, "ckpt_gpt_c16_nh2_l2.npz"), 2026)
            return
        saved_M = golden.M
        _kernel_level(golden)
        golden.M = saved_M

        # capture_mha_oracle.py scenario: seed 4242 params, RandomState(4243) data
        res = _run_reference_mha(gpt, cuda, 2, 5, 8, 2, 4242, 4243)
        np.savez(os.path.join(HERE, "mha_b2_t5_c8_nh2.npz"), **res)

        # wider shapes through the same reference path: odd T, head_dim 8/16/32/64
        for (B, T, C, NH, s) in [(2, 33, 64, 4, 11), (1, 70, 64, 2, 12), (1, 130, 128, 2, 13),
                                 (2, 17, 32, 4, 14)]:
            res = _run_reference_mha(gpt, cuda, B, T, C, NH, 5000 + s, 6000 + s)
            res.pop("cache_attn_weights")  # T×T; the oracle rebuilds it, keep fixtures small
            np.savez_compressed(os.path.join(HERE, f"mha_b{B}_t{T}_c{C}_nh{NH}.npz"), **res)

        # FeedForward: test_ffn_gpu_backward.py's scenario, then a wider one with biases
        np.savez(os.path.join(HERE, "ffn_c16_m6.npz"), **_run_reference_ffn(gpt, cuda, 16, 6, 1337))
        np.savez_compressed(os.path.join(HERE, "ffn_c64_m40.npz"),
                            **_run_reference_ffn(gpt, cuda, 64, 40, 2024, dout_seed=2025, bias_scale=0.5))

        # a checkpoint archive written by the reference's GPTModel.save_checkpoint
        _run_reference_checkpoint(gpt, cuda, os.path.join(HERE, "ckpt_gpt_c16_nh2_l2.npz"), 2026)
    finally:
        os.chdir(cwd)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--only=")]
    only = next((a.split("=", 1)[1] for a in sys.argv[1:] if a.startswith("--only=")), None)
    ref = args[0] if args else os.environ.get("LLM_GPU5_REFERENCE")
    if not ref:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout> [--only=checkpoint]  "
                 "(or set LLM_GPU5_REFERENCE)")
    main(ref, only)
