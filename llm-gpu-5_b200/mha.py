"""Drop-in ``MultiHeadAttention`` for llm-gpu-5 (model/gpt.py:478-707), running on B200 kernels.

Same constructor, same ``forward(gpu_input, B, T)`` / ``backward(gpu_dOut, B, T, accumulate)`` /
``free_forward_caches()`` contract, same ``c_attn_w[C,3C]``, ``c_attn_b[3C]``, ``c_proj_w[C,C]``,
``c_proj_b[C]`` parameters with ``gpu_weights``/``gpu_grads``/``gpu_m``/``gpu_v`` buffers, so
TransformerBlock (model/gpt.py:742, :779, :825), GPTModel checkpoints (model/gpt.py:1136-1143) and
the training loops keep working.  What changes is where the work runs:

* forward: QKV projection, causal flash attention (row log-sum-exp instead of the T x T
  probabilities), output projection: three library calls, no host round trip.  The reference's
  split_heads/merge_heads copies are folded into the attention kernels' addressing (they read
  Q/K/V straight out of the fused [B*T, 3C] projection and write the context in [B*T, C]).
* backward: the whole of model/gpt.py:652-698 on the GPU (projection gradients, softmax VJP,
  dQ/dK/dV, dX), gradients set or accumulated in place on the device.

Precision: ``"fp32"`` reproduces the reference's float32 arithmetic on CUDA cores (the golden
tolerance, 1e-5 relative); ``"bf16"`` runs the projections and attention on tcgen05 tensor cores
with bf16 operands and fp32 accumulation/softmax statistics (2e-2 relative).

Device memory comes from PyTorch's caching allocator; launches go to the current torch stream.
Buffers returned by ``forward``/``backward`` are ``DeviceBuffer`` objects the caller frees, as in
the reference (model/gpt.py:780-783, :819, :836-837).
"""

from __future__ import annotations

import functools
import math

import numpy as np
import torch

from . import dp
from . import mha_ops as ops
from ._lib import check_device_error, watch_device_error
from .mha_ops import HeadView, ptr


def device_checked(fn):
    """Wrap a module entry point: raise DeviceWaitError first if a kernel of an earlier call gave
    up a bounded wait, and after the call enqueue the copy of the device status word that the next
    call reads.  Costs one 4-byte device-to-host copy per call and no synchronisation."""

    @functools.wraps(fn)
    def wrapper(*args, **kwargs):
        check_device_error()
        out = fn(*args, **kwargs)
        watch_device_error()
        return out
    return wrapper


def start_grad_sync(mod, bucket=None):
    """Start the all-reduce (SUM over ``mod.grad_sync_group``) of floats [lo, hi) = ``bucket`` of a
    module's flat gradient buffer (all of it by default) once they are final, ahead of the work that
    follows in backward: through NCCL on its own stream (``wait_grad_sync`` waits for it), or, with a
    MulticastGradReducer attached, the library's NVSwitch multicast all-reduce, either on a side
    stream beside the next kernels (``reducer.overlap``, its small blocks sharing the SMs with them)
    or on the current stream when ``finish_grad_sync`` is called.  Returns what ``finish_grad_sync``
    completes before backward returns, or None."""
    if mod.grad_sync_group is None:
        return None
    lo, hi = bucket if bucket is not None else (0, mod.flat_grads.numel())
    red = mod.grad_reducer
    if red is None:
        mod._grad_sync_works.append(
            dp.allreduce_grads(mod.flat_grads[lo:hi], mod.grad_sync_group, async_op=True))
        return None
    if not red.overlap:
        def serial():
            with mod._rng("grad_allreduce"):
                red.allreduce(lo, hi)
        return serial
    mod._grad_stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(mod._grad_stream):
        with mod._rng("grad_allreduce"):
            red.allreduce(lo, hi)
        joined = torch.cuda.Event()
        joined.record(mod._grad_stream)
    return lambda: torch.cuda.current_stream().wait_event(joined)


def grad_sync_gemm_ctas(mod) -> int:
    """max_ctas for the GEMM that follows start_grad_sync: fewer than every SM when the module's
    multicast reducer runs beside it and asks for SMs of its own (reducer.reserve_sms)."""
    if mod.grad_sync_group is None or mod.grad_reducer is None:
        return 0
    return mod.grad_reducer.gemm_ctas()


def grad_sync_buckets(mod, layout, first_names):
    """The module's all-reduce buckets: one for the whole buffer, or, with ``mod.grad_buckets``,
    the parameters in ``first_names`` (final earlier in backward) and the rest (dp.grad_buckets)."""
    if not mod.grad_buckets:
        return [None]
    return dp.grad_buckets(layout, first_names)


def finish_grad_sync(*pending):
    """Complete what start_grad_sync began (the current stream waits for the side stream's
    all-reduces, or launches them), so the summed gradients are in place, in stream order, when
    backward returns."""
    for p in pending:
        if p is not None:
            p()


def attach_grad_reducer(mod, reducer, layout):
    """Move a module's flat gradient buffer into ``reducer.buffer`` (copying the current values) and
    point its Parameters' gradients at their places in it (``layout`` as dp.grad_layout)."""
    if reducer.numel != mod.flat_grads.numel():
        raise ValueError(f"use_grad_reducer: the buffer holds {reducer.numel} floats, "
                         f"{mod.flat_grads.numel()} needed")
    reducer.buffer.copy_(mod.flat_grads)
    mod.flat_grads = reducer.buffer
    for name, off, shape in layout:
        getattr(mod, name).grads = mod.flat_grads[off:off + int(np.prod(shape))].view(shape)
    mod.grad_reducer = reducer
    mod._grad_stream = torch.cuda.Stream()


class GPTConfig:
    """The fields of llm-gpu-5's GPTConfig (model/gpt.py:53-87) that the attention path and its
    callers read, under the same argument names, plus ``attention_precision``: "fp32" (the
    reference's float32 arithmetic), "tf32" (float32 storage, tf32 tensor-core products) or "bf16".

    ``attention_impl`` is only carried for the checkpoint metadata (model/gpt.py:1114, :1196-1199);
    the reference's older spellings of it (``attention_mode``, ``use_flash_attention`` /
    ``flash_attention``) are accepted.  Other keyword arguments are ignored, as there."""

    def __init__(self, vocab_size: int, max_len: int = 8, embedding_dim: int = 16, num_heads: int = 2,
                 num_layers: int = 1, dropout_prob: float = 0.1, max_seq_len: int = None,
                 attention_impl: str = None, use_flash_attention: bool = None,
                 attention_precision: str = "fp32", **kwargs):
        if embedding_dim % num_heads:
            raise ValueError("embedding_dim must be divisible by num_heads")
        if attention_precision not in ("fp32", "tf32", "bf16"):
            raise ValueError(f"attention_precision must be 'fp32', 'tf32' or 'bf16', got {attention_precision!r}")
        self.vocab_size = vocab_size
        self.max_len = max_seq_len if max_seq_len is not None else max_len
        self.embedding_dim = embedding_dim
        self.num_heads = num_heads
        self.head_dim = embedding_dim // num_heads
        self.num_layers = num_layers
        self.dropout_prob = dropout_prob
        self.attention_precision = attention_precision
        impl = attention_impl if attention_impl is not None else kwargs.get("attention_mode")
        if impl is None:
            flash = use_flash_attention if use_flash_attention is not None else kwargs.get("flash_attention")
            impl = "strided" if flash else "identity"
        self.attention_impl = str(impl).strip().lower()
        if self.attention_impl not in ("identity", "strided"):
            raise ValueError(f"Unsupported attention_impl: {impl}")
        self.use_flash_attention = self.attention_impl == "strided"


class DeviceBuffer:
    """A device allocation handed to the caller: ``int(buf)`` is its address, ``free()`` releases
    it (the PyCUDA ``DeviceAllocation`` surface the reference's callers use)."""

    __slots__ = ("tensor",)

    def __init__(self, tensor: torch.Tensor):
        self.tensor = tensor

    def __int__(self):
        return self.tensor.data_ptr()

    def data_ptr(self):
        return self.tensor.data_ptr()

    @property
    def nbytes(self):
        return self.tensor.numel() * self.tensor.element_size()

    def free(self):
        self.tensor = None

    def get(self):
        return self.tensor.detach().cpu().numpy()


def _as_tensor(x, numel: int, dtype=torch.float32) -> torch.Tensor:
    """View any device pointer-like object as a flat CUDA tensor of ``numel`` elements."""
    if isinstance(x, torch.Tensor):
        assert x.is_cuda and x.dtype == dtype and x.is_contiguous() and x.numel() >= numel
        return x.reshape(-1)[:numel]
    if isinstance(x, DeviceBuffer):
        return _as_tensor(x.tensor, numel, dtype)
    addr = int(x)

    class _Iface:  # expose a raw address to torch without copying
        __cuda_array_interface__ = {
            "shape": (numel,), "typestr": "<f4" if dtype == torch.float32 else "<u2",
            "data": (addr, False), "version": 3}
    return torch.as_tensor(_Iface(), device="cuda")


class Parameter:
    """Weights plus gradient and AdamW moment buffers in device memory (model/gpt.py:101-154).

    Initialised exactly as the reference: ``np.random.normal(0, init_scale, shape)`` from NumPy's
    global generator, so seeded runs reproduce the reference's weights.  ``grad_storage`` lets a
    module place the gradient inside one flat buffer (for a single all-reduce).
    """

    def __init__(self, shape: tuple = None, init_scale: float = 0.02, dtype=None, grad_storage=None):
        self.shape = tuple(shape)
        self.dtype = dtype if dtype is not None else np.float32
        self.total_elements = int(np.prod(shape))
        self.bytes_size = self.total_elements * 4
        host_w = np.random.normal(0.0, init_scale, size=shape).astype(np.float32)
        self.weights = torch.from_numpy(host_w).to("cuda")
        self.grads = grad_storage if grad_storage is not None else torch.zeros(
            self.shape, dtype=torch.float32, device="cuda")
        self.grads.zero_()
        self.m = torch.zeros(self.shape, dtype=torch.float32, device="cuda")
        self.v = torch.zeros(self.shape, dtype=torch.float32, device="cuda")
        self._handed_out = 0  # times gpu_weights gave the weights' address to a caller
        self._bf16 = None     # (key, bf16 copy of the weights)

    # PyCUDA-style handles (``int()`` gives the device address)
    @property
    def gpu_weights(self):
        # whoever takes the address may write the weights behind torch's back (the reference's
        # optimizer kernels do, core/ops.py:545-570): the bf16 copy is made again after this
        self._handed_out += 1
        return DeviceBuffer(self.weights)

    def bf16_weights(self) -> torch.Tensor:
        """The weights rounded to bf16 for the tensor-core path, kept between calls while the
        weights are unchanged: while the tensor is the same, torch's version counter of it has not
        moved (no in-place torch op) and ``gpu_weights`` has not handed its address out.  While a
        CUDA graph is being captured the cast is always recorded, so every replay casts the weights
        as they are then."""
        key = (self.weights.data_ptr(), self.weights._version, self._handed_out)
        if torch.cuda.is_current_stream_capturing():
            return ops.cast_bf16(self.weights)
        if self._bf16 is None or self._bf16[0] != key:
            self._bf16 = (key, ops.cast_bf16(self.weights))
        return self._bf16[1]

    @property
    def gpu_grads(self):
        return DeviceBuffer(self.grads)

    @property
    def gpu_m(self):
        return DeviceBuffer(self.m)

    @property
    def gpu_v(self):
        return DeviceBuffer(self.v)

    def free(self):
        self.weights = self.grads = self.m = self.v = None

    def set_or_accumulate_grads(self, host_grads, accumulate=False):
        g = torch.from_numpy(np.ascontiguousarray(host_grads, dtype=np.float32)).to("cuda").view(self.shape)
        if accumulate:
            self.grads.add_(g)
        else:
            self.grads.copy_(g)

    def set_or_accumulate_grads_from_gpu(self, gpu_grads_ptr, accumulate=False):
        g = _as_tensor(gpu_grads_ptr, self.total_elements).view(self.shape)
        if accumulate:
            self.grads.add_(g)
        else:
            self.grads.copy_(g)


class _NullRange:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NULL = _NullRange()


class MultiHeadAttention:
    """Multi-head causal self-attention with the reference's API (model/gpt.py:478-707)."""

    def __init__(self, config_or_embedding_dim=None, num_heads: int = None, precision: str = None):
        if isinstance(config_or_embedding_dim, GPTConfig):
            config = config_or_embedding_dim
        elif config_or_embedding_dim is not None:
            config = GPTConfig(vocab_size=50, embedding_dim=config_or_embedding_dim,
                               num_heads=num_heads or 2, max_len=8)
        else:
            raise ValueError("MultiHeadAttention requires either GPTConfig or embedding_dim parameter")
        self.config = config
        C = config.embedding_dim
        self.precision = precision or getattr(config, "attention_precision", "fp32")
        if self.precision not in ("fp32", "tf32", "bf16"):
            raise ValueError(f"precision must be 'fp32', 'tf32' or 'bf16', got {self.precision!r}")

        # one flat fp32 gradient buffer [dWqkv | dbqkv | dWo | dbo] so data-parallel training
        # all-reduces the four gradients with a single collective
        self.flat_grads = torch.zeros(dp.flat_grad_size(C), dtype=torch.float32, device="cuda")
        views = {name: self.flat_grads[off:off + int(np.prod(shape))].view(shape)
                 for name, off, shape in dp.grad_layout(C)}
        # same parameter order and init as model/gpt.py:507-510
        self.c_attn_w = Parameter((C, C * 3), grad_storage=views["c_attn_w"])
        self.c_attn_b = Parameter((C * 3,), init_scale=0.0, grad_storage=views["c_attn_b"])
        self.c_proj_w = Parameter((C, C), grad_storage=views["c_proj_w"])
        self.c_proj_b = Parameter((C,), init_scale=0.0, grad_storage=views["c_proj_b"])

        self.profiler = None  # optional: object with .range(name) -> context manager (CUDA events)
        self.grad_sync_group = None  # a torch.distributed group: backward all-reduces (SUM) into it
        self.grad_reducer = None     # a dp.MulticastGradReducer holding flat_grads (use_grad_reducer)
        # True: all-reduce dWo/dbo as soon as they are final, then dWqkv/dbqkv.  Off by default: the
        # early all-reduce holds SMs that the attention backward's persistent CTAs need whole
        # (0.890 vs 0.877 ms per step on 8 GPUs at 64 sequences per GPU)
        self.grad_buckets = False
        self._grad_sync_works = []
        self.training = True
        self._cache = None

    # ---------------------------------------------------------------- helpers
    def _rng(self, name):
        return self.profiler.range(name) if self.profiler is not None else _NULL

    @property
    def _dt(self):
        return torch.bfloat16 if self.precision == "bf16" else torch.float32

    @property
    def _mm(self):
        """Operand type of the module's GEMM and attention calls: the storage dtype, or "tf32"
        (float32 storage multiplied on the tensor cores as tf32)."""
        return "tf32" if self.precision == "tf32" else self._dt

    def _shape(self):
        C = self.config.embedding_dim
        NH = self.config.num_heads
        return C, NH, C // NH

    # ---------------------------------------------------------------- forward
    @device_checked
    def forward(self, gpu_input, B: int, T: int, kv_cache: "KVCache | None" = None):
        """x [B*T, C] float32 (device) -> DeviceBuffer [B*T, C] float32 (caller frees).

        With ``kv_cache`` (from ``new_kv_cache``) the prompt's keys and values are also stored in
        it, so that ``forward_decode`` can continue the sequences one token at a time."""
        C, NH, D = self._shape()
        M = B * T
        dt = self._dt
        self._cache = None
        x = _as_tensor(gpu_input, M * C)
        if dt == torch.bfloat16:
            with self._rng("cast"):
                # bf16 x with a ones column (16-byte row pitch): the backward's weight-gradient
                # GEMM over C + 1 rows then also produces the bias gradient
                x_op = ops.cast_rows_ones(x.view(M, C))
        else:
            x_op = x.clone().view(M, C)  # the caller may overwrite its input (residual adds are in place)
        out = torch.empty((M, C), dtype=torch.float32, device="cuda")
        self._forward_core(x_op, B, T, out, accumulate=False, kv_cache=kv_cache)
        return DeviceBuffer(out)

    @device_checked
    def forward_residual(self, gpu_x, B: int, T: int, ln_gamma, ln_beta, eps: float = 1e-5):
        """x += attn(LayerNorm(x)) in place on the residual stream x [B*T, C] float32.

        Fuses the pre-attention part of TransformerBlock.forward (model/gpt.py:778-783):
        ``ln1 = ln_op(x, gamma, beta)``, ``out = attn.forward(ln1)``, ``add_op(x, out)``.  One
        LayerNorm kernel writes the QKV projection's operand directly (bf16 with the ones column on
        the bf16 path), and the output projection adds ctx Wo + bo into x in its epilogue, so
        neither the float32 LayerNorm output nor the attention output is written to memory.
        ``backward`` afterwards is unchanged: its upstream gradient is dL/dx after the add."""
        C, NH, D = self._shape()
        M = B * T
        dt = self._dt
        self._cache = None
        x = _as_tensor(gpu_x, M * C).view(M, C)
        g, b = _as_tensor(ln_gamma, C), _as_tensor(ln_beta, C)
        with self._rng("layernorm"):
            x_op = ops.layernorm(x, g, b, eps, out_dtype=dt, ones_col=dt == torch.bfloat16)
        # the LayerNorm input, for backward_residual (TransformerBlock keeps the same copy,
        # cache_input_ln1, model/gpt.py:773-775)
        ln_input = x.clone() if getattr(self, "training", True) else None
        self._forward_core(x_op, B, T, x, accumulate=True)
        if self._cache is not None:
            self._cache.update(ln_input=ln_input, ln_eps=eps)

    @device_checked
    def backward_residual(self, gpu_dx, B: int, T: int, ln_gamma, ln_dgamma, ln_dbeta, accumulate=False):
        """Backward of forward_residual, in place: dx (dL/dx after the residual add) becomes
        dL/dx before it, dx + LN_bwd(attn.backward(dx)), and the four attention gradients and the
        LayerNorm's dgamma/dbeta are set (or accumulated).  Replaces the attention half of
        TransformerBlock.backward (model/gpt.py:825-838): attn.backward, ln_bwd_op, a copy of dX1 and
        the residual add, with the LayerNorm backward adding into dx directly."""
        c = self._cache
        if c is None or c.get("ln_input") is None:
            raise RuntimeError("MultiHeadAttention.backward_residual() called without forward_residual caches")
        C, NH, D = self._shape()
        M = B * T
        dx = _as_tensor(gpu_dx, M * C).view(M, C)
        dln = self.backward(dx, B, T, accumulate=accumulate)
        with self._rng("layernorm_bwd"):
            ops.layernorm_backward(dln.tensor.view(M, C), c["ln_input"], _as_tensor(ln_gamma, C), dx,
                                   _as_tensor(ln_dgamma, C), _as_tensor(ln_dbeta, C), c["ln_eps"],
                                   accumulate_dx=True, accumulate_params=accumulate)
        dln.free()

    def _forward_core(self, x_op, B, T, out, accumulate, kv_cache=None):
        """QKV projection of the prepared operand x_op [M, >= C], attention, output projection
        into out [M, C] float32 (added to it when accumulate)."""
        C, NH, D = self._shape()
        M = B * T
        dt = self._dt
        mm = self._mm
        if dt == torch.bfloat16:
            with self._rng("cast"):
                w_qkv = self.c_attn_w.bf16_weights()
                w_o = self.c_proj_w.bf16_weights()
        else:
            w_qkv, w_o = self.c_attn_w.weights, self.c_proj_w.weights
        ldx = x_op.shape[1]
        qkv = torch.empty((M, 3 * C), dtype=dt, device="cuda")
        with self._rng("gemm_qkv"):
            ops.gemm(x_op.data_ptr(), ldx, False, w_qkv.data_ptr(), 3 * C, False, mm, qkv.data_ptr(),
                     3 * C, dt, M, 3 * C, C, bias=self.c_attn_b.weights.data_ptr())
        if kv_cache is not None:
            kv_cache.store(qkv.view(B, T, 3 * C), 0)
        ctx = torch.empty((M, C), dtype=dt, device="cuda")
        lse = torch.empty((B, NH, T), dtype=torch.float32, device="cuda")
        es = qkv.element_size()
        base = qkv.data_ptr()
        qv = HeadView.tokens(base, T, 3 * C, D)
        kv = HeadView.tokens(base + C * es, T, 3 * C, D)
        vv = HeadView.tokens(base + 2 * C * es, T, 3 * C, D)
        ov = HeadView.tokens(ctx.data_ptr(), T, C, D)
        scale = 1.0 / math.sqrt(D)
        with self._rng("attn_fwd"):
            ops.attention_forward(qv, kv, vv, ov, lse, B, NH, T, D, scale, mm)
        with self._rng("gemm_out"):
            ops.gemm(ctx.data_ptr(), C, False, w_o.data_ptr(), C, False, mm, out.data_ptr(), C,
                     torch.float32, M, C, C, bias=self.c_proj_b.weights.data_ptr(), accumulate=accumulate)
        if getattr(self, "training", True):
            self._cache = dict(B=B, T=T, x=x_op, qkv=qkv, ctx=ctx, lse=lse, w_qkv=w_qkv, w_o=w_o)

    # ---------------------------------------------------------------- backward
    @device_checked
    def backward(self, gpu_dOut, B: int, T: int, accumulate=False):
        """dY [B*T, C] float32 -> dX DeviceBuffer [B*T, C]; parameter grads set or accumulated."""
        c = self._cache
        if c is None or c["B"] != B or c["T"] != T:
            raise RuntimeError("MultiHeadAttention.backward() called without forward caches")
        C, NH, D = self._shape()
        M = B * T
        dt = self._dt
        mm = self._mm
        dy = _as_tensor(gpu_dOut, M * C)
        # output projection: dbo = sum(dY), dWo = ctx^T dY, dCtx = dY Wo^T   (gpt.py:666-670)
        if dt == torch.bfloat16:
            with self._rng("cast_colsum"):  # one pass over dY: bf16 copy + bias gradient
                dy_op = ops.cast_colsum(dy.view(M, C), self.c_proj_b.grads, accumulate=accumulate)
        else:
            dy_op = dy
            with self._rng("colsum"):
                ops.colsum(dy.data_ptr(), torch.float32, C, M, C, self.c_proj_b.grads, accumulate=accumulate)
        with self._rng("gemm_dwo"):
            ops.gemm(c["ctx"].data_ptr(), C, True, dy_op.data_ptr(), C, False, mm,
                     self.c_proj_w.grads.data_ptr(), C, torch.float32, C, C, M, accumulate=accumulate)
        buckets = grad_sync_buckets(self, dp.grad_layout(C), ("c_proj_w", "c_proj_b"))
        # dWo and dbo are final: with buckets, their all-reduce overlaps dCtx and the attention backward
        pending_o = start_grad_sync(self, buckets[0]) if len(buckets) == 2 else None
        dctx = torch.empty((M, C), dtype=dt, device="cuda")
        with self._rng("gemm_dctx"):
            ops.gemm(dy_op.data_ptr(), C, False, c["w_o"].data_ptr(), C, True, mm, dctx.data_ptr(), C,
                     dt, M, C, C)
        # attention: softmax VJP + dQ/dK/dV written straight into the [B*T, 3C] layout (gpt.py:672-685)
        dqkv = torch.empty((M, 3 * C), dtype=dt, device="cuda")
        es = dqkv.element_size()
        qb, gb = c["qkv"].data_ptr(), dqkv.data_ptr()
        tv = lambda base: HeadView.tokens(base, T, 3 * C, D)  # noqa: E731
        ov = HeadView.tokens(c["ctx"].data_ptr(), T, C, D)
        dov = HeadView.tokens(dctx.data_ptr(), T, C, D)
        with self._rng("attn_bwd"):
            ops.attention_backward(tv(qb), tv(qb + C * es), tv(qb + 2 * C * es), ov, dov, c["lse"],
                                   tv(gb), tv(gb + C * es), tv(gb + 2 * C * es), B, NH, T, D,
                                   1.0 / math.sqrt(D), mm)
        # input projection: dWqkv = x^T dQKV, dbqkv = sum(dQKV), dX = dQKV Wqkv^T  (gpt.py:687-689)
        x_op = c["x"]
        if x_op.shape[1] > C:
            # x carries a ones column: the C + 1 output rows are [dWqkv; dbqkv], and dbqkv follows
            # dWqkv in the flat gradient buffer, so one GEMM writes both
            with self._rng("gemm_dwqkv"):
                ops.gemm(x_op.data_ptr(), x_op.shape[1], True, gb, 3 * C, False, mm,
                         self.c_attn_w.grads.data_ptr(), 3 * C, torch.float32, C + 1, 3 * C, M,
                         accumulate=accumulate)
        else:
            with self._rng("gemm_dwqkv"):
                ops.gemm(x_op.data_ptr(), C, True, gb, 3 * C, False, mm, self.c_attn_w.grads.data_ptr(),
                         3 * C, torch.float32, C, 3 * C, M, accumulate=accumulate)
            with self._rng("colsum"):
                ops.colsum(gb, dt, 3 * C, M, 3 * C, self.c_attn_b.grads, accumulate=accumulate)
        # the remaining gradients are final: their all-reduce overlaps the dX GEMM below
        pending = start_grad_sync(self, buckets[-1])
        dx = torch.empty((M, C), dtype=torch.float32, device="cuda")
        with self._rng("gemm_dx"):
            ops.gemm(gb, 3 * C, False, c["w_qkv"].data_ptr(), 3 * C, True, mm, dx.data_ptr(), C,
                     torch.float32, M, C, 3 * C, max_ctas=grad_sync_gemm_ctas(self))
        finish_grad_sync(pending_o, pending)
        return DeviceBuffer(dx)

    def use_grad_reducer(self, reducer):
        """Keep the four gradients in ``reducer``'s buffer (a dp.MulticastGradReducer of
        dp.flat_grad_size(C) floats), so that backward sums them over the ranks with the library's
        NVSwitch multicast all-reduce instead of NCCL (when ``grad_sync_group`` is set, as for
        NCCL: on the last micro-step of an accumulation).  The current gradients are copied over."""
        attach_grad_reducer(self, reducer, dp.grad_layout(self.config.embedding_dim))

    def wait_grad_sync(self):
        """Wait for the gradient all-reduce launched by the last backward (if any), and raise
        DeviceWaitError if a kernel of a finished call gave up a bounded wait."""
        for work in self._grad_sync_works:
            work.wait()
        self._grad_sync_works = []
        check_device_error()

    def free_forward_caches(self):
        """Release the forward caches (model/gpt.py:700-707)."""
        self._cache = None

    # ---------------------------------------------------------------- reference cache views
    # The reference keeps host copies of its caches (model/gpt.py:603-619) and its parity test
    # reads them (test_mha_integration_parity.py:88-93).  Here the caches stay on the device;
    # these properties download them in the reference's shapes on demand (debug/test only).
    def _qkv_heads(self, which):
        c = self._cache
        if c is None:
            return None
        C, NH, D = self._shape()
        B, T = c["B"], c["T"]
        t = c["qkv"].view(B, T, 3, NH, D)[:, :, which].permute(0, 2, 1, 3)
        return t.float().contiguous().cpu().numpy()

    @property
    def cache_q(self):
        return self._qkv_heads(0)

    @property
    def cache_k(self):
        return self._qkv_heads(1)

    @property
    def cache_v(self):
        return self._qkv_heads(2)

    # ---------------------------------------------------------------- incremental decoding
    def new_kv_cache(self, B: int, max_len: int) -> "KVCache":
        """A key/value cache for ``B`` sequences of up to ``max_len`` tokens, in this module's
        compute precision."""
        C, NH, D = self._shape()
        return KVCache(B, max_len, NH, D, self._dt)

    @device_checked
    def forward_decode(self, gpu_input, B: int, kv_cache: "KVCache"):
        """One new token per sequence: x [B, C] float32 -> DeviceBuffer [B, C] float32.

        Equals the last rows of ``forward`` over the whole sequence (causal attention, the new
        token sees every cached one), which is what GenerationSession.generate recomputes for
        every token (generate.py:611-628).  Here the token's key and value are appended to the
        cache and one ``attn_decode`` call attends over it: O(L) per token instead of O(L^2).
        No backward (inference only; the training caches are left untouched)."""
        C, NH, D = self._shape()
        dt = self._dt
        mm = self._mm
        L = kv_cache.length
        if kv_cache.B != B or L >= kv_cache.max_len:
            raise RuntimeError(f"forward_decode: cache holds {kv_cache.B} sequences, {L} of "
                               f"{kv_cache.max_len} positions used")
        x = _as_tensor(gpu_input, B * C).view(B, C)
        if dt == torch.bfloat16:
            x_op = ops.cast_bf16(x)
            w_qkv = self.c_attn_w.bf16_weights()
            w_o = self.c_proj_w.bf16_weights()
        else:
            x_op, w_qkv, w_o = x, self.c_attn_w.weights, self.c_proj_w.weights
        qkv = torch.empty((B, 3 * C), dtype=dt, device="cuda")
        ops.gemm(x_op.data_ptr(), C, False, w_qkv.data_ptr(), 3 * C, False, mm, qkv.data_ptr(), 3 * C, dt,
                 B, 3 * C, C, bias=self.c_attn_b.weights.data_ptr())
        kv_cache.store(qkv.view(B, 1, 3 * C), L)
        q = qkv[:, :C].contiguous().view(B, NH, D)  # q and the output share one layout
        ctx = ops.decode(q, kv_cache.k[:, :L + 1], kv_cache.v[:, :L + 1], 1.0 / math.sqrt(D))
        out = torch.empty((B, C), dtype=torch.float32, device="cuda")
        ops.gemm(ctx.data_ptr(), C, False, w_o.data_ptr(), C, False, mm, out.data_ptr(), C, torch.float32,
                 B, C, C, bias=self.c_proj_b.weights.data_ptr())
        return DeviceBuffer(out)

    @property
    def cache_context(self):
        c = self._cache
        return None if c is None else c["ctx"].float().cpu().numpy()

    @property
    def cache_input(self):
        c = self._cache
        if c is None:
            return None
        C = self.c_proj_w.weights.shape[0]
        return c["x"][:, :C].float().cpu().numpy()  # without the bf16 path's ones column

    @property
    def cache_lse(self):
        c = self._cache
        return None if c is None else c["lse"].cpu().numpy()

    @property
    def cache_attn_weights(self):
        """[B, NH, T, T] probabilities rebuilt on the GPU from lse (never stored by forward)."""
        c = self._cache
        if c is None:
            return None
        C, NH, D = self._shape()
        B, T = c["B"], c["T"]
        es = c["qkv"].element_size()
        base = c["qkv"].data_ptr()
        p = ops.attention_probs(HeadView.tokens(base, T, 3 * C, D),
                                HeadView.tokens(base + C * es, T, 3 * C, D), c["lse"], B, NH, T, D,
                                1.0 / math.sqrt(D), self._mm)
        return p.cpu().numpy()


class KVCache:
    """Keys and values of B sequences in token layout [B, max_len, NH, D] (the layout the
    projection writes and ``attn_decode`` reads), plus the number of positions filled."""

    def __init__(self, B: int, max_len: int, NH: int, D: int, dtype: torch.dtype):
        self.B, self.max_len, self.NH, self.D = B, max_len, NH, D
        self.k = torch.empty((B, max_len, NH, D), dtype=dtype, device="cuda")
        self.v = torch.empty((B, max_len, NH, D), dtype=dtype, device="cuda")
        self.length = 0

    def store(self, qkv: torch.Tensor, pos: int):
        """Copy K and V of qkv [B, T, 3C] (the fused projection's output) to positions
        pos .. pos+T-1 and extend the filled length to pos+T."""
        B, T, C3 = qkv.shape
        C = C3 // 3
        if pos + T > self.max_len:
            raise RuntimeError(f"KVCache: {pos + T} positions exceed max_len {self.max_len}")
        self.k[:, pos:pos + T].copy_(qkv[:, :, C:2 * C].view(B, T, self.NH, self.D))
        self.v[:, pos:pos + T].copy_(qkv[:, :, 2 * C:].view(B, T, self.NH, self.D))
        self.length = max(self.length, pos + T)
