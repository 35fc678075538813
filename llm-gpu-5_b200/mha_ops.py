"""Launch wrappers over the C ABI, in the role core/mha_ops.py plays for the reference.

Each wrapper takes torch CUDA tensors (or raw device addresses), checks shapes on the host,
and launches on the current torch stream.  All compute is in libattn_b200.so.

The reference's launch constants (core/mha_ops.py:22-23) are kept for callers that read them;
the kernels here choose their own tiling.
"""

from __future__ import annotations

import math

import torch

from ._lib import ATTN_ACT_GELU, ATTN_ACT_GELU_BWD, ATTN_ACT_NONE, ATTN_BF16, ATTN_F32, ATTN_TF32, call, lib  # noqa: F401

THREADS_PER_BLOCK = 256
SOFTMAX_BLOCK_THREADS = 64

_DT = {torch.float32: ATTN_F32, torch.bfloat16: ATTN_BF16}


def dtype_code(t) -> int:
    """Library code of an operand type: torch.float32, torch.bfloat16, or "tf32" (float32 storage
    multiplied on the tensor cores as tf32)."""
    if isinstance(t, str) and t == "tf32":
        return ATTN_TF32
    try:
        return _DT[t]
    except KeyError:
        raise TypeError(f"unsupported dtype {t}; expected float32, bfloat16 or 'tf32'") from None


def _stream():
    return torch.cuda.current_stream().cuda_stream


def ptr(x) -> int:
    """Device address of a torch tensor, a DeviceBuffer, a pycuda DeviceAllocation or an int."""
    if isinstance(x, torch.Tensor):
        if not x.is_cuda:
            raise TypeError("expected a CUDA tensor")
        return x.data_ptr()
    if hasattr(x, "data_ptr"):
        return int(x.data_ptr())
    return int(x)


class HeadView:
    """Element strides of an attention operand: element (b, t, h, d) at base[b*sb + t*st + h*sh + d]."""

    __slots__ = ("base", "sb", "st", "sh")

    def __init__(self, base: int, sb: int, st: int, sh: int):
        self.base, self.sb, self.st, self.sh = int(base), int(sb), int(st), int(sh)

    @staticmethod
    def tokens(base: int, T: int, ld: int, D: int) -> "HeadView":
        """Token layout [B*T, ld] with head h at column offset h*D (the fused projection layout)."""
        return HeadView(base, T * ld, ld, D)

    @staticmethod
    def heads(base: int, NH: int, T: int, D: int) -> "HeadView":
        """The reference's split layout [B*NH, T, D] (split_heads_kernel output)."""
        return HeadView(base, NH * T * D, D, T * D)


def attention_forward(q: HeadView, k: HeadView, v: HeadView, o: HeadView, lse: torch.Tensor,
                      B: int, NH: int, T: int, D: int, scale: float, dtype: torch.dtype):
    """Causal attention forward; q/k/v share strides.  lse: float32 [B, NH, T]."""
    assert (k.sb, k.st, k.sh) == (q.sb, q.st, q.sh) == (v.sb, v.st, v.sh)
    assert lse.dtype == torch.float32 and lse.numel() >= B * NH * T
    call("attn_fwd", q.base, k.base, v.base, o.base, lse.data_ptr(), B, NH, T, D,
         q.sb, q.st, q.sh, o.sb, o.st, o.sh, float(scale), dtype_code(dtype), _stream())


def attention_backward(q: HeadView, k: HeadView, v: HeadView, o: HeadView, do: HeadView,
                       lse: torch.Tensor, dq: HeadView, dk: HeadView, dv: HeadView,
                       B: int, NH: int, T: int, D: int, scale: float, dtype: torch.dtype,
                       workspace: torch.Tensor | None = None):
    """Causal attention backward.  dq/dk/dv use q's strides, do uses o's."""
    assert (dq.sb, dq.st, dq.sh) == (q.sb, q.st, q.sh) == (dk.sb, dk.st, dk.sh) == (dv.sb, dv.st, dv.sh)
    assert (do.sb, do.st, do.sh) == (o.sb, o.st, o.sh)
    code = dtype_code(dtype)
    need = lib.attn_bwd_workspace_size(B, NH, T, D, code)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device="cuda")
    call("attn_bwd", q.base, k.base, v.base, o.base, do.base, lse.data_ptr(), dq.base, dk.base,
         dv.base, workspace.data_ptr(), workspace.numel() * workspace.element_size(), B, NH, T, D,
         q.sb, q.st, q.sh, o.sb, o.st, o.sh, float(scale), code, _stream())


def attention_probs(q: HeadView, k: HeadView, lse: torch.Tensor, B, NH, T, D, scale, dtype):
    """Rebuild the [B, NH, T, T] probabilities from lse (debug/test accessor)."""
    out = torch.empty((B, NH, T, T), dtype=torch.float32, device="cuda")
    call("attn_probs", q.base, k.base, lse.data_ptr(), out.data_ptr(), B, NH, T, D, q.sb, q.st, q.sh,
         float(scale), dtype_code(dtype), _stream())
    return out


def decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, scale: float | None = None,
           out: torch.Tensor | None = None, lse: torch.Tensor | None = None,
           workspace: torch.Tensor | None = None):
    """Single-query decode: q [B, NH, D], caches [B, L, NH, D] (token layout) -> out [B, NH, D]."""
    B, NH, D = q.shape
    L = k_cache.shape[1]
    assert k_cache.shape == v_cache.shape == (B, L, NH, D)
    assert q.dtype == k_cache.dtype == v_cache.dtype
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    # q and out are addressed with the same (b, h) strides
    assert out.shape == q.shape and out.dtype == q.dtype and out.stride() == q.stride(), \
        "decode: q and out must have the same shape, dtype and strides"
    need = lib.attn_decode_workspace_size(B, NH, L, D)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    qs = q.stride()
    ks = k_cache.stride()
    assert k_cache.stride() == v_cache.stride() and ks[3] == 1 and qs[2] == 1
    call("attn_decode", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(),
         lse.data_ptr() if lse is not None else None, B, NH, L, D, qs[0], qs[1], ks[0], ks[1], ks[2],
         float(scale), dtype_code(q.dtype), workspace.data_ptr(),
         workspace.numel() * workspace.element_size(), _stream())
    return out


def gemm(A: int, lda: int, a_trans: bool, B: int, ldb: int, b_trans: bool, ab_dtype: torch.dtype,
         C: int, ldc: int, c_dtype: torch.dtype, M: int, N: int, K: int, bias: int | None = None,
         accumulate: bool = False, max_ctas: int = 0):
    """C[M,N] (=|+=) op(A) op(B) (+bias) on raw device addresses (see include/attn_b200.h); on at
    most ``max_ctas`` SMs when it is positive (attn_gemm_ex)."""
    if max_ctas:
        call("attn_gemm_ex", A, lda, int(a_trans), B, ldb, int(b_trans), dtype_code(ab_dtype), C, ldc,
             dtype_code(c_dtype), bias, M, N, K, int(accumulate), int(max_ctas), _stream())
        return
    call("attn_gemm", A, lda, int(a_trans), B, ldb, int(b_trans), dtype_code(ab_dtype), C, ldc,
         dtype_code(c_dtype), bias, M, N, K, int(accumulate), _stream())


def gemm_act(A: int, lda: int, a_trans: bool, B: int, ldb: int, b_trans: bool, ab_dtype: torch.dtype,
             C: int, ldc: int, c_dtype: torch.dtype, M: int, N: int, K: int, act: int, aux: int | None = None,
             ldaux: int = 0, aux_dtype: torch.dtype = torch.float32, bias: int | None = None):
    """GEMM with the feed-forward activation in its epilogue (attn_gemm_act): ATTN_ACT_GELU writes
    gelu(op(A) op(B) + bias) to C and the pre-activation to aux; ATTN_ACT_GELU_BWD writes
    op(A) op(B) * gelu'(aux)."""
    call("attn_gemm_act", A, lda, int(a_trans), B, ldb, int(b_trans), dtype_code(ab_dtype), C, ldc,
         dtype_code(c_dtype), bias, M, N, K, int(act), aux, ldaux, dtype_code(aux_dtype), _stream())


def colsum(X: int, x_dtype: torch.dtype, ldx: int, M: int, N: int, out: torch.Tensor,
           accumulate: bool = False, workspace: torch.Tensor | None = None):
    need = lib.attn_colsum_workspace_size(M, N)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device="cuda")
    call("attn_colsum", X, dtype_code(x_dtype), ldx, M, N, out.data_ptr(), int(accumulate),
         workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream())


def cast_colsum(x: torch.Tensor, colsum_out: torch.Tensor, accumulate: bool = False,
                out: torch.Tensor | None = None, workspace: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 copy of a float32 [M, N] matrix plus its column sums (into/onto colsum_out), one pass."""
    assert x.dtype == torch.float32 and x.is_contiguous() and x.dim() == 2
    M, N = x.shape
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    need = lib.attn_colsum_workspace_size(M, N)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    call("attn_cast_colsum_f32", x.data_ptr(), N, M, N, out.data_ptr(), N, colsum_out.data_ptr(),
         int(accumulate), workspace.data_ptr(), workspace.numel() * workspace.element_size(), _stream())
    return out


def cast_bf16(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    assert x.dtype == torch.float32 and x.is_contiguous()
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    call("attn_cast_f32_to_bf16", x.data_ptr(), out.data_ptr(), x.numel(), _stream())
    return out


def cast_rows_ones(x: torch.Tensor) -> torch.Tensor:
    """float32 [M, N] -> bf16 [M, L] with L = N + 1 rounded up to a multiple of 8 (16-byte rows):
    bf16(x), then a column of ones, then zeros.  Used as the QKV projection's input so the
    weight-gradient GEMM also yields the bias gradient."""
    assert x.dtype == torch.float32 and x.is_contiguous() and x.dim() == 2
    M, N = x.shape
    L = (N + 1 + 7) // 8 * 8
    out = torch.empty((M, L), dtype=torch.bfloat16, device=x.device)
    call("attn_cast_rows_ones_bf16", x.data_ptr(), N, M, N, out.data_ptr(), L, _stream())
    return out


def layernorm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
              out_dtype: torch.dtype = torch.float32, ones_col: bool = False) -> torch.Tensor:
    """Row LayerNorm of float32 x [M, C] (layernorm_kernel, core/kernels.py:75-110) -> [M, C] in
    out_dtype, or, with ones_col (bf16), [M, L] = LN(x) | 1 | 0.. like cast_rows_ones."""
    assert x.dtype == torch.float32 and x.is_contiguous() and x.dim() == 2
    M, C = x.shape
    L = (C + 1 + 7) // 8 * 8 if ones_col else C
    out = torch.empty((M, L), dtype=out_dtype, device=x.device)
    call("attn_layernorm", x.data_ptr(), C, gamma.data_ptr(), beta.data_ptr(), M, C, float(eps), out.data_ptr(),
         L, dtype_code(out_dtype), int(ones_col), _stream())
    return out


def layernorm_backward(dy: torch.Tensor, x: torch.Tensor, gamma: torch.Tensor, dx: torch.Tensor,
                       dgamma: torch.Tensor, dbeta: torch.Tensor, eps: float = 1e-5, accumulate_dx: bool = False,
                       accumulate_params: bool = False):
    """LayerNorm backward of layernorm_backward_kernel (core/kernels.py:361-416) on float32 [M, C]
    rows: dx (=|+=) dLN/dx, dgamma/dbeta (=|+=) the parameter gradients."""
    assert dy.dtype == x.dtype == dx.dtype == torch.float32 and dy.shape == x.shape == dx.shape
    M, C = x.shape
    call("attn_layernorm_bwd", dy.data_ptr(), x.data_ptr(), gamma.data_ptr(), M, C, float(eps), dx.data_ptr(),
         int(accumulate_dx), dgamma.data_ptr(), dbeta.data_ptr(), int(accumulate_params), _stream())


def split_heads(qkv: int, q: int, k: int, v: int, B: int, T: int, NH: int, HD: int):
    """split_heads_kernel (core/mha_kernels.py:534-558) on float32 device buffers."""
    call("attn_split_heads", qkv, q, k, v, B, T, NH, HD, _stream())


def merge_heads(ctx_heads: int, ctx: int, B: int, T: int, NH: int, HD: int):
    """merge_heads_kernel (core/mha_kernels.py:567-584) on float32 device buffers."""
    call("attn_merge_heads", ctx_heads, ctx, B, T, NH, HD, _stream())


class _Kernel:
    """A named kernel handle shaped like the reference's PyCUDA functions (positional args)."""

    def __init__(self, name, fn):
        self.__name__ = name
        self._fn = fn

    def __call__(self, *args, block=None, grid=None, shared=None, stream=None):
        return self._fn(*[ptr(a) if not isinstance(a, (int, float)) else a for a in args])


class _SharedModule:
    """Stand-in for the compiled PyCUDA module of get_shared_mha_module (core/mha_ops.py:39-48):
    the layout adapters are exposed by the reference's kernel names."""

    def get_function(self, name):
        if name == "split_heads_kernel":
            return _Kernel(name, lambda qkv, q, k, v, B, T, NH, HD: split_heads(
                qkv, q, k, v, int(B), int(T), int(NH), int(HD)))
        if name == "merge_heads_kernel":
            return _Kernel(name, lambda ch, c, B, T, NH, HD: merge_heads(
                ch, c, int(B), int(T), int(NH), int(HD)))
        raise KeyError(f"{name}: the B200 library replaces this kernel; use MultiHeadAttention or "
                       "the attention_* wrappers")


_SHARED = _SharedModule()


def get_shared_mha_module():
    return _SHARED


class MHAController:
    """The reference's sandbox attention controller (core/mha_ops.py:55-138) on this library.

    ``forward(X[H, M, Din], W_qkv[Din, 3D])`` runs the fused-QKV causal attention pass on host
    float32 arrays and returns ``(out[H, M, D], probs[H, M, M])`` as the reference's does: the
    fused projection ``X W_qkv`` (matmul_qkv_fused, core/mha_kernels.py:689-720) is one float32
    GEMM; the reference's split into contiguous Q/K/V (split_qkv_kernel, :722-) is folded into the
    attention's strides (it reads Q, K and V straight out of the fused [H*M, 3D] buffer); the causal
    attention (fused_attention_forward_kernel) runs on the float32 kernels and writes the row
    log-sum-exp, from which ``probs`` is rebuilt on the device.  Inputs are copied to the device
    and the results back, as in the reference.  ``H, M, D`` fix the attention shape; ``module`` is
    accepted for signature compatibility.
    """

    def __init__(self, H: int, M: int, D: int, module=None):
        self.H, self.M, self.D = int(H), int(M), int(D)
        self.scale = 1.0 / math.sqrt(D)
        self.module = module if module is not None else get_shared_mha_module()

    def _fused(self, gX, gW, Din: int) -> torch.Tensor:
        H, M, D = self.H, self.M, self.D
        fused = torch.empty((H * M, 3 * D), dtype=torch.float32, device="cuda")
        gemm(gX.data_ptr(), Din, False, gW.data_ptr(), 3 * D, False, torch.float32, fused.data_ptr(), 3 * D,
             torch.float32, H * M, 3 * D, Din)
        return fused

    def matmul_qkv_fused(self, gpu_X, gpu_W, gpu_fused, Din: int, block=None, grid=None):
        """Fused[H, M, 3D] = X[H, M, Din] @ W_qkv[Din, 3D] on device buffers (the launch
        configuration arguments of the reference are accepted and unused)."""
        H, M, D = self.H, self.M, self.D
        gemm(ptr(gpu_X), Din, False, ptr(gpu_W), 3 * D, False, torch.float32, ptr(gpu_fused), 3 * D,
             torch.float32, H * M, 3 * D, int(Din))

    def forward(self, X, W_qkv):
        import numpy as np
        H, M, D = self.H, self.M, self.D
        X = np.ascontiguousarray(X, dtype=np.float32)
        W_qkv = np.ascontiguousarray(W_qkv, dtype=np.float32)
        if X.shape[:2] != (H, M) or W_qkv.shape != (X.shape[-1], 3 * D):
            raise ValueError(f"MHAController({H}, {M}, {D}): X {X.shape} / W_qkv {W_qkv.shape} do not match")
        Din = X.shape[-1]
        gX = torch.from_numpy(X).cuda().view(H * M, Din)
        gW = torch.from_numpy(W_qkv).cuda()
        fused = self._fused(gX, gW, Din)
        base, es = fused.data_ptr(), fused.element_size()
        # heads as batch entries of one head each: element (h, m, d) of Q/K/V at h*M*3D + m*3D + d
        qv, kv, vv = (HeadView(base + i * D * es, M * 3 * D, 3 * D, D) for i in range(3))
        out = torch.empty((H, M, D), dtype=torch.float32, device="cuda")
        lse = torch.empty((H, 1, M), dtype=torch.float32, device="cuda")
        attention_forward(qv, kv, vv, HeadView(out.data_ptr(), M * D, D, D), lse, H, 1, M, D, self.scale,
                          torch.float32)
        probs = attention_probs(qv, kv, lse, H, 1, M, D, self.scale, torch.float32)
        return out.cpu().numpy(), probs.view(H, M, M).cpu().numpy()
