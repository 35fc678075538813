"""Drop-in ``FeedForward`` for llm-gpu-5 (model/gpt.py:282-470), running on the library's GEMMs.

Same constructor, same ``forward(gpu_input, B, T)`` / ``backward(gpu_dOut, B, T, accumulate)`` /
``free_forward_caches()`` contract and the same ``c_fc_w[C,4C]``, ``c_fc_b[4C]``, ``c_proj_w[4C,C]``,
``c_proj_b[C]`` parameters, so TransformerBlock (model/gpt.py:785-795, :806-821) and the checkpoint
code keep working.  The reference runs five kernels forward (two matmul_2d_kernel, a device copy of
the pre-activation, the in-place activation_kernel) and nine backward (matmul_backward_weights x2,
reduce_sum_axis0 x2, matmul_backward_input x2, gelu_backward, plus gradient copies).  Here:

* forward: two GEMM launches.  The first applies bias + GELU in its epilogue and writes both the
  activation (the second GEMM's operand) and the pre-activation (for backward); the second adds
  its bias in its epilogue (or adds the whole FFN output into the residual stream in place, see
  ``forward_residual``).
* backward: four GEMM launches and one pass over dOut.  dOut is cast once with its column sums
  (dProjB) in the same pass; dProjW = act^T dOut; dPre = (dOut W_proj^T) * gelu'(pre) with the GELU
  derivative in the GEMM epilogue; [dFcW; dFcB] = [x | 1]^T dPre as one GEMM (the input carries a
  ones column on the bf16 path); dIn = dPre W_fc^T.

Precision follows ``MultiHeadAttention``: ``"fp32"`` on CUDA cores (1e-5 relative to the
reference's float32 math), ``"bf16"`` on tcgen05 tensor cores with bf16 operands and cached
activations, fp32 accumulation (2e-2 relative).
"""

from __future__ import annotations

import numpy as np
import torch

from . import dp
from . import mha_ops as ops
from ._lib import check_device_error
from .mha import (DeviceBuffer, GPTConfig, Parameter, _as_tensor, _NULL, attach_grad_reducer, device_checked,
                  finish_grad_sync, grad_sync_buckets, grad_sync_gemm_ctas, start_grad_sync)


class FeedForward:
    """Position-wise MLP, C -> 4C -> C with tanh-GELU (model/gpt.py:282-470)."""

    def __init__(self, config_or_embedding_dim=None, hidden_dim: int = None, precision: str = None):
        if isinstance(config_or_embedding_dim, GPTConfig):
            config = config_or_embedding_dim
        elif config_or_embedding_dim is not None:
            config = GPTConfig(vocab_size=50, embedding_dim=config_or_embedding_dim, max_len=8)
        else:
            raise ValueError('FeedForward requires either GPTConfig or embedding_dim parameter')
        self.config = config
        C = config.embedding_dim
        self.hidden = C * 4  # the reference fixes the expansion at 4C whatever hidden_dim says
        self.precision = precision or getattr(config, "attention_precision", "fp32")
        if self.precision not in ("fp32", "tf32", "bf16"):
            raise ValueError(f"precision must be 'fp32', 'tf32' or 'bf16', got {self.precision!r}")
        self.flat_grads = torch.zeros(dp.layout_size(dp.ffn_grad_layout(C)), dtype=torch.float32, device="cuda")
        views = {name: self.flat_grads[off:off + int(np.prod(shape))].view(shape)
                 for name, off, shape in dp.ffn_grad_layout(C)}
        # same parameter order and init as model/gpt.py:305-308
        self.c_fc_w = Parameter((C, self.hidden), grad_storage=views["c_fc_w"])
        self.c_fc_b = Parameter((self.hidden,), init_scale=0.0, grad_storage=views["c_fc_b"])
        self.c_proj_w = Parameter((self.hidden, C), grad_storage=views["c_proj_w"])
        self.c_proj_b = Parameter((C,), init_scale=0.0, grad_storage=views["c_proj_b"])
        self.training = True
        # The reference's switch to its host NumPy backward (model/gpt.py:325, :381-426).  That
        # backward is this library's test oracle, not a product path: setting it raises in backward.
        self.use_cpu_backward = False
        self.profiler = None
        self.grad_sync_group = None
        self.grad_reducer = None  # a dp.MulticastGradReducer holding flat_grads (use_grad_reducer)
        self.grad_buckets = False  # True: all-reduce dWproj/dbproj as soon as they are final, then dWfc/dbfc
        self._grad_sync_works = []
        self._cache = None

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

    # ---------------------------------------------------------------- forward
    @device_checked
    def forward(self, gpu_input, B: int, T: int):
        """x [B*T, C] float32 (device) -> DeviceBuffer [B*T, C] float32 (caller frees)."""
        C = self.config.embedding_dim
        M = B * T
        x = _as_tensor(gpu_input, M * C).view(M, C)
        self._cache = None
        if self._dt == torch.bfloat16:
            with self._rng("cast"):  # bf16 x | 1 | 0..: the dFcW GEMM also yields dFcB
                x_op = ops.cast_rows_ones(x)
        else:
            x_op = x.clone()
        out = torch.empty((M, C), dtype=torch.float32, device="cuda")
        self._forward_core(x_op, B, T, out, accumulate=False)
        return DeviceBuffer(out)

    @device_checked
    def forward_residual(self, gpu_x, B: int, T: int, ln_gamma, ln_beta, eps: float = 1e-5):
        """x += FFN(LayerNorm(x)) in place on the residual stream x [B*T, C] float32: the second
        half of TransformerBlock.forward (model/gpt.py:785-795: ln_2, mlp.forward, the residual add).
        The LayerNorm writes the first GEMM's operand directly and the second GEMM adds its output
        (with its bias) into x in its epilogue."""
        C = self.config.embedding_dim
        M = B * T
        x = _as_tensor(gpu_x, M * C).view(M, C)
        g, b = _as_tensor(ln_gamma, C), _as_tensor(ln_beta, C)
        dt = self._dt
        self._cache = None
        with self._rng("layernorm"):
            x_op = ops.layernorm(x, g, b, eps, out_dtype=dt, ones_col=dt == torch.bfloat16)
        ln_input = x.clone() if getattr(self, "training", True) else None
        self._forward_core(x_op, B, T, x, accumulate=True)
        if self._cache is not None:
            self._cache.update(ln_input=ln_input, ln_eps=eps)

    def _forward_core(self, x_op, B, T, out, accumulate):
        C, H = self.config.embedding_dim, self.hidden
        M = B * T
        dt = self._dt
        mm = self._mm
        if dt == torch.bfloat16:
            with self._rng("cast"):
                w_fc = self.c_fc_w.bf16_weights()
                w_proj = self.c_proj_w.bf16_weights()
        else:
            w_fc, w_proj = self.c_fc_w.weights, self.c_proj_w.weights
        training = getattr(self, "training", True)
        act = torch.empty((M, H), dtype=dt, device="cuda")
        pre = torch.empty((M, H), dtype=dt, device="cuda") if training else None
        with self._rng("gemm_fc_gelu"):
            ops.gemm_act(x_op.data_ptr(), x_op.shape[1], False, w_fc.data_ptr(), H, False, mm, act.data_ptr(), H, dt,
                         M, H, C, ops.ATTN_ACT_GELU, aux=pre.data_ptr() if pre is not None else None, ldaux=H,
                         aux_dtype=dt, bias=self.c_fc_b.weights.data_ptr())
        with self._rng("gemm_proj"):
            ops.gemm(act.data_ptr(), H, False, w_proj.data_ptr(), C, False, mm, out.data_ptr(), C, torch.float32,
                     M, C, H, bias=self.c_proj_b.weights.data_ptr(), accumulate=accumulate)
        if training:
            self._cache = dict(B=B, T=T, x=x_op, pre=pre, act=act, w_fc=w_fc, w_proj=w_proj)

    # ---------------------------------------------------------------- backward
    @device_checked
    def backward(self, gpu_dOut, B: int, T: int, accumulate=False):
        """dOut [B*T, C] float32 -> dIn DeviceBuffer [B*T, C]; the four gradients set or accumulated
        in place (model/gpt.py:367-456, the GPU-resident path :428-456)."""
        c = self._cache
        if c is None or c["B"] != B or c["T"] != T:
            raise RuntimeError("FeedForward.backward() called without forward caches")
        if getattr(self, "use_cpu_backward", False):
            raise RuntimeError("FeedForward.use_cpu_backward: the host NumPy backward is the test oracle "
                               "(oracle.mha_oracle.ffn_backward), not part of the library")
        C, H = self.config.embedding_dim, self.hidden
        M = B * T
        dt = self._dt
        mm = self._mm
        dy = _as_tensor(gpu_dOut, M * C).view(M, C)
        # c_proj: dProjB = sum(dOut), dProjW = act^T dOut   (model/gpt.py:431-432)
        if dt == torch.bfloat16:
            with self._rng("cast_colsum"):
                dy_op = ops.cast_colsum(dy, self.c_proj_b.grads, accumulate=accumulate)
        else:
            dy_op = dy
            with self._rng("colsum"):
                ops.colsum(dy.data_ptr(), torch.float32, C, M, C, self.c_proj_b.grads, accumulate=accumulate)
        with self._rng("gemm_dwproj"):
            ops.gemm(c["act"].data_ptr(), H, True, dy_op.data_ptr(), C, False, mm, self.c_proj_w.grads.data_ptr(), C,
                     torch.float32, H, C, M, accumulate=accumulate)
        buckets = grad_sync_buckets(self, dp.ffn_grad_layout(C), ("c_proj_w", "c_proj_b"))
        # dWproj and dbproj are final: with buckets, their all-reduce overlaps the GEMMs that follow
        pending_p = start_grad_sync(self, buckets[0]) if len(buckets) == 2 else None
        # dPre = (dOut W_proj^T) * gelu'(pre)   (model/gpt.py:433-436)
        dpre = torch.empty((M, H), dtype=dt, device="cuda")
        with self._rng("gemm_dhidden_gelu"):
            ops.gemm_act(dy_op.data_ptr(), C, False, c["w_proj"].data_ptr(), C, True, mm, dpre.data_ptr(), H, dt,
                         M, H, C, ops.ATTN_ACT_GELU_BWD, aux=c["pre"].data_ptr(), ldaux=H, aux_dtype=dt)
        # c_fc: dFcW = x^T dPre, dFcB = sum(dPre)   (model/gpt.py:441-442)
        x_op = c["x"]
        if x_op.shape[1] > C:  # ones column: the C + 1 output rows are [dFcW; dFcB], adjacent in flat_grads
            with self._rng("gemm_dwfc"):
                ops.gemm(x_op.data_ptr(), x_op.shape[1], True, dpre.data_ptr(), H, False, mm,
                         self.c_fc_w.grads.data_ptr(), H, torch.float32, C + 1, H, M, accumulate=accumulate)
        else:
            with self._rng("gemm_dwfc"):
                ops.gemm(x_op.data_ptr(), C, True, dpre.data_ptr(), H, False, mm, self.c_fc_w.grads.data_ptr(), H,
                         torch.float32, C, H, M, accumulate=accumulate)
            with self._rng("colsum"):
                ops.colsum(dpre.data_ptr(), dt, H, M, H, self.c_fc_b.grads, accumulate=accumulate)
        pending = start_grad_sync(self, buckets[-1])  # the rest are final: their all-reduce overlaps dIn
        # dIn = dPre W_fc^T   (model/gpt.py:443)
        dx = torch.empty((M, C), dtype=torch.float32, device="cuda")
        with self._rng("gemm_dx"):
            ops.gemm(dpre.data_ptr(), H, False, c["w_fc"].data_ptr(), H, True, mm, dx.data_ptr(), C, torch.float32,
                     M, C, H, max_ctas=grad_sync_gemm_ctas(self))
        finish_grad_sync(pending_p, pending)
        return DeviceBuffer(dx)

    def use_grad_reducer(self, reducer):
        """Keep the four gradients in ``reducer``'s buffer (a dp.MulticastGradReducer of
        dp.layout_size(dp.ffn_grad_layout(C)) floats): backward then sums them over the ranks with the
        library's NVSwitch multicast all-reduce instead of NCCL (when ``grad_sync_group`` is set)."""
        attach_grad_reducer(self, reducer, dp.ffn_grad_layout(self.config.embedding_dim))

    @device_checked
    def backward_residual(self, gpu_dx, B: int, T: int, ln_gamma, ln_dgamma, ln_dbeta, accumulate=False):
        """Backward of forward_residual, in place: dx (dL/dx after the residual add) becomes
        dx + LN_bwd(ffn.backward(dx)), and the FFN's and the LayerNorm's gradients are set (or
        accumulated); the FFN half of TransformerBlock.backward (model/gpt.py:806-821)."""
        c = self._cache
        if c is None or c.get("ln_input") is None:
            raise RuntimeError("FeedForward.backward_residual() called without forward_residual caches")
        C = self.config.embedding_dim
        M = B * T
        dx = _as_tensor(gpu_dx, M * C).view(M, C)
        dln = self.backward(dx, B, T, accumulate=accumulate)
        with self._rng("layernorm_bwd"):
            ops.layernorm_backward(dln.tensor.view(M, C), c["ln_input"], _as_tensor(ln_gamma, C), dx,
                                   _as_tensor(ln_dgamma, C), _as_tensor(ln_dbeta, C), c["ln_eps"],
                                   accumulate_dx=True, accumulate_params=accumulate)
        dln.free()

    def wait_grad_sync(self):
        """Wait for the gradient all-reduce launched by the last backward (if any), and raise
        DeviceWaitError if a kernel of a finished call gave up a bounded wait."""
        for work in self._grad_sync_works:
            work.wait()
        self._grad_sync_works = []
        check_device_error()

    def free_forward_caches(self):
        """Release the forward caches (model/gpt.py:458-470)."""
        self._cache = None

    # the reference's cache attributes (device allocations there): the cached tensors, in the
    # module's precision, or None
    def _cached(self, key):
        c = self._cache
        return None if c is None or c.get(key) is None else DeviceBuffer(c[key])

    @property
    def cache_input(self):
        c = self._cache
        return None if c is None else DeviceBuffer(c["x"][:, :self.config.embedding_dim].contiguous())

    @property
    def cache_pre_act(self):
        return self._cached("pre")

    @property
    def cache_activated(self):
        return self._cached("act")
