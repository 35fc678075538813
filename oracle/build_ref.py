"""Build ``oracle/_ref/libref_kernels.so`` from the reference's own CUDA kernel sources (checker only).

    python oracle/build_ref.py <reference checkout>      (or LLM_GPU5_REFERENCE=<checkout>)

The reference's GPU kernels live as CUDA source in Python strings, compiled at run time by
PyCUDA's ``SourceModule`` with ``-O3 --use_fast_math`` (core/ops.py:27-34, core/mha_ops.py:26-33).
This script reads two of those files as text (``ast``, nothing of the reference is imported or
executed), takes

* ``LAYERNORM_KERNEL`` (core/kernels.py:73-110): ``layernorm_kernel``, one thread per row;
* ``LAYERNORM_BACKWARD_KERNEL`` (core/kernels.py:359-420): ``layernorm_backward_kernel``;
* the FeedForward kernels (core/kernels.py): ``MATMUL_2D_KERNEL`` (:117-140), ``ACTIVATION_KERNEL``
  (:233-250), ``MATMUL_BACKWARD_WEIGHTS_KERNEL`` (:333-356), ``GELU_BACKWARD_KERNEL`` (:422-447),
  ``REDUCE_SUM_AXIS0_KERNEL`` (:449-470), ``MATMUL_BACKWARD_INPUT_KERNEL`` (:472-497);
* ``MHA_KERNELS_STRING`` (core/mha_kernels.py:53-...): among others
  ``fused_attention_forward_kernel`` (core/mha_kernels.py:404-521), the gradient kernels the
  reference's GPU golden test chains (``matmul_score_kernel``, ``softmax_fused_backward``,
  ``matmul_grad_q_kernel``, ``matmul_grad_k_kernel``, ``matmul_grad_v``) and the layout adapters
  ``split_heads_kernel`` / ``merge_heads_kernel`` (core/mha_kernels.py:534-584),

wraps the MHA string in ``extern "C"`` as SourceModule does, appends host launchers of our own that
use the reference's launch configurations (256 threads per block and ceil(rows / 256) blocks for the
LayerNorm, core/ops.py:128-132; 64 threads, grid (B*NH, T) and (D + T + 64) * 4 bytes of shared
memory for the fused forward, model/gpt.py:563, :587-592), and compiles the result for sm_100a into
``oracle/_ref/`` (git-ignored, so the reference's sources never enter the repository; the built
library still travels with the working tree).  ``tests/test_gpu_reference_kernels.py`` runs these
kernels next to the library's on the same inputs; nothing in the product loads them.
"""

from __future__ import annotations

import ast
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT, "libref_kernels.so")

LAUNCHERS = r'''
// ---- host launchers (this repository's code): the reference's launch configurations ----
#include <cuda_runtime.h>
extern "C" int ref_layernorm(const float* x, float* y, const float* gamma, const float* beta, int rows,
                             int channels) {
  const int threads = 256;  // core/ops.py:128-132
  const int blocks = (rows + threads - 1) / threads;
  layernorm_kernel<<<blocks, threads>>>(x, y, gamma, beta, rows, channels);
  return (int)cudaDeviceSynchronize();
}

extern "C" int ref_fused_attention_forward(const float* q, const float* k, const float* v, float* scores,
                                           float* out, float* row_max, float* row_sum, int H, int M, int D,
                                           float scale) {
  const int threads = 64;  // MHA_SOFTMAX_BLOCK_THREADS, model/gpt.py:563
  const size_t smem = (size_t)(D + M + threads) * 4;  // model/gpt.py:587
  fused_attention_forward_kernel<<<dim3(H, M), threads, smem>>>(q, k, v, scores, out, row_max, row_sum, H, M,
                                                                D, scale);
  return (int)cudaDeviceSynchronize();
}

// LayerNormBackward.__call__ (core/ops.py:410-437): zeroed dGamma/dBeta, 256 threads per block.
extern "C" int ref_layernorm_backward(const float* dy, const float* x, const float* gamma, float* dx, float* dgamma,
                                      float* dbeta, int rows, int channels) {
  if (cudaMemset(dgamma, 0, (size_t)channels * 4) != cudaSuccess ||
      cudaMemset(dbeta, 0, (size_t)channels * 4) != cudaSuccess)
    return -1;
  const int threads = 256;
  layernorm_backward_kernel<<<(rows + threads - 1) / threads, threads>>>(dy, x, gamma, dx, dgamma, dbeta, rows,
                                                                        channels);
  return (int)cudaDeviceSynchronize();
}

// The kernel-level backward chain of the reference's GPU golden test (test_mha_golden_model.py:136-156):
// dP = dOut V^T with matmul_score_kernel (scale 1), the softmax VJP softmax_fused_backward (no softmax
// scale, as that test), then matmul_grad_q_kernel / matmul_grad_k_kernel / matmul_grad_v.  probs is
// the Scores output of the fused forward.  Scratch is allocated here (checker code only).
extern "C" int ref_attention_backward(const float* q, const float* k, const float* v, const float* dout,
                                      const float* probs, float* dq, float* dk, float* dv, int H, int M, int D) {
  float *dprobs = 0, *dscores = 0, *rsum = 0;
  const size_t mm = (size_t)H * M * M * sizeof(float);
  if (cudaMalloc(&dprobs, mm) != cudaSuccess || cudaMalloc(&dscores, mm) != cudaSuccess ||
      cudaMalloc(&rsum, (size_t)H * M * sizeof(float)) != cudaSuccess)
    return -1;
  const int threads = 256, softmax_threads = 64;  // test_mha_golden_model.py:118-122
  const int score_blocks = (H * M * M + threads - 1) / threads, proj_blocks = (H * M * D + threads - 1) / threads;
  matmul_score_kernel<<<score_blocks, threads>>>(dout, v, dprobs, H, M, D, 1.0f);
  softmax_fused_backward<<<dim3(H, M), softmax_threads, softmax_threads * 4>>>(dprobs, probs, rsum, dscores, H, M);
  matmul_grad_q_kernel<<<proj_blocks, threads>>>(dscores, k, dq, H, M, D);
  matmul_grad_k_kernel<<<proj_blocks, threads>>>(dscores, q, dk, H, M, D);
  matmul_grad_v<<<proj_blocks, threads>>>(probs, dout, dv, H, M, D);
  const int rc = (int)cudaDeviceSynchronize();
  cudaFree(dprobs);
  cudaFree(dscores);
  cudaFree(rsum);
  return rc;
}

// FeedForward.forward's kernel sequence (model/gpt.py:345-363) with the launch geometry of core/ops.py:
// matmul_2d_kernel on 16x16 blocks (:163-168), the pre-activation copy, activation_kernel on 256
// threads (:255-258), matmul_2d_kernel again.  pre/act/out [M, 4C] / [M, 4C] / [M, C].
extern "C" int ref_ffn_forward(const float* x, const float* w_fc, const float* b_fc, const float* w_proj,
                               const float* b_proj, float* pre, float* act, float* out, int M, int C) {
  const int H = 4 * C;
  const dim3 blk(16, 16);
  matmul_2d_kernel<<<dim3((H + 15) / 16, (M + 15) / 16), blk>>>(x, w_fc, b_fc, pre, M, H, C);
  if (cudaMemcpy(act, pre, (size_t)M * H * 4, cudaMemcpyDeviceToDevice) != cudaSuccess) return -1;
  activation_kernel<<<(M * H + 255) / 256, 256>>>(act, M * H);
  matmul_2d_kernel<<<dim3((C + 15) / 16, (M + 15) / 16), blk>>>(act, w_proj, b_proj, out, M, C, H);
  return (int)cudaDeviceSynchronize();
}

// FeedForward.backward's GPU-resident path (model/gpt.py:428-443): matmul_backward_weights (16x16,
// core/ops.py:388-394), reduce_sum_axis0 into zeroed sums (256 threads over rows, :491-498),
// matmul_backward_input (16x16, :526-531), gelu_backward (256 threads, :462-466).  Scratch is
// allocated here (checker code only).
extern "C" int ref_ffn_backward(const float* dout, const float* x, const float* pre, const float* act,
                                const float* w_fc, const float* w_proj, float* din, float* d_fc_w, float* d_fc_b,
                                float* d_proj_w, float* d_proj_b, int M, int C) {
  const int H = 4 * C;
  const dim3 blk(16, 16);
  float *dhidden = 0, *dpre = 0;
  if (cudaMalloc(&dhidden, (size_t)M * H * 4) != cudaSuccess || cudaMalloc(&dpre, (size_t)M * H * 4) != cudaSuccess)
    return -1;
  if (cudaMemset(d_proj_b, 0, (size_t)C * 4) != cudaSuccess || cudaMemset(d_fc_b, 0, (size_t)H * 4) != cudaSuccess)
    return -1;
  matmul_backward_weights_kernel<<<dim3((C + 15) / 16, (H + 15) / 16), blk>>>(act, dout, d_proj_w, M, C, H);
  reduce_sum_axis0_kernel<<<(M + 255) / 256, 256>>>(dout, d_proj_b, M, C, C);
  matmul_backward_input_kernel<<<dim3((H + 15) / 16, (M + 15) / 16), blk>>>(dout, w_proj, dhidden, M, C, H);
  gelu_backward_kernel<<<(M * H + 255) / 256, 256>>>(dhidden, pre, dpre, M * H);
  matmul_backward_weights_kernel<<<dim3((H + 15) / 16, (C + 15) / 16), blk>>>(x, dpre, d_fc_w, M, H, C);
  reduce_sum_axis0_kernel<<<(M + 255) / 256, 256>>>(dpre, d_fc_b, M, H, H);
  matmul_backward_input_kernel<<<dim3((C + 15) / 16, (M + 15) / 16), blk>>>(dpre, w_fc, din, M, H, C);
  const int rc = (int)cudaDeviceSynchronize();
  cudaFree(dhidden);
  cudaFree(dpre);
  return rc;
}

// The layout adapters, 256 threads per block over B*T*NH*HD elements (model/gpt.py:569-598).
extern "C" int ref_split_heads(const float* qkv, float* q, float* k, float* v, int B, int T, int NH, int HD) {
  const int total = B * T * NH * HD, threads = 256;
  split_heads_kernel<<<(total + threads - 1) / threads, threads>>>(qkv, q, k, v, B, T, NH, HD);
  return (int)cudaDeviceSynchronize();
}

extern "C" int ref_merge_heads(const float* heads, float* ctx, int B, int T, int NH, int HD) {
  const int total = B * T * NH * HD, threads = 256;
  merge_heads_kernel<<<(total + threads - 1) / threads, threads>>>(heads, ctx, B, T, NH, HD);
  return (int)cudaDeviceSynchronize();
}
'''


def _string_constant(path: str, name: str) -> str:
    """The value of the module-level string assignment ``name = "..."`` in ``path``."""
    with open(path) as f:
        tree = ast.parse(f.read(), filename=path)
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(isinstance(t, ast.Name) and t.id == name for t in node.targets):
            if isinstance(node.value, ast.Constant) and isinstance(node.value.value, str):
                return node.value.value
    raise KeyError(f"{name} not found in {path}")


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(reference_root: str) -> str:
    ln = _string_constant(os.path.join(reference_root, "core", "kernels.py"), "LAYERNORM_KERNEL")
    ln_bwd = _string_constant(os.path.join(reference_root, "core", "kernels.py"), "LAYERNORM_BACKWARD_KERNEL")
    mha = _string_constant(os.path.join(reference_root, "core", "mha_kernels.py"), "MHA_KERNELS_STRING")
    ffn = [_string_constant(os.path.join(reference_root, "core", "kernels.py"), name)
           for name in ("MATMUL_2D_KERNEL", "ACTIVATION_KERNEL", "MATMUL_BACKWARD_WEIGHTS_KERNEL",
                        "GELU_BACKWARD_KERNEL", "REDUCE_SUM_AXIS0_KERNEL", "MATMUL_BACKWARD_INPUT_KERNEL")]
    os.makedirs(OUT, exist_ok=True)
    src = os.path.join(OUT, "ref_kernels.cu")
    with open(src, "w") as f:
        f.write("// Generated by oracle/build_ref.py from the reference's kernel strings; not part of the repo.\n")
        f.write(ln)
        f.write(ln_bwd)
        for k in ffn:
            f.write(k)
        f.write('\nextern "C" {\n')
        f.write(mha)
        f.write("\n}\n")
        f.write(LAUNCHERS)
    cmd = [_nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math", "-Xcompiler",
           "-fPIC", "-shared", "-w", "-o", LIB, src, "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building the reference kernels failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def reference_root(argv=None):
    """The reference checkout: the first argument, else $LLM_GPU5_REFERENCE; None if neither names
    a directory holding the reference's ``core/`` sources."""
    root = (argv[0] if argv else None) or os.environ.get("LLM_GPU5_REFERENCE")
    if root and os.path.isdir(os.path.join(root, "core")):
        return root
    return None


if __name__ == "__main__":
    root = reference_root(sys.argv[1:])
    if root is None:
        sys.exit("usage: python oracle/build_ref.py <reference checkout>  (or set LLM_GPU5_REFERENCE)")
    print(build(root))
