"""Checkpoint-format compatibility of the drop-in attention parameters (model/gpt.py:1103-1243).

GPTModel.save_checkpoint / load_checkpoint walk every block's ``attn`` sub-layer over the
attribute names c_attn_w, c_attn_b, c_proj_w, c_proj_b (c_fc_w/c_fc_b are absent on attention),
copy ``p_obj.shape`` float32 values between host arrays and ``p_obj.gpu_weights`` with
pycuda's memcpy_dtoh / memcpy_htod, and store them under ``block_{idx}_attn_{attr}`` in an .npz
(model/gpt.py:1136-1143 and :1220-1227).  These tests run that loop, restated with a stand-in
for the two pycuda copies (cuda-python's cudaMemcpy on ``int(ptr)``), against the module: the
archive gets the reference's keys, shapes and dtypes, and a module loaded from it computes the
same forward output.
"""
import os

import numpy as np
import pytest

from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu
ATTRS = ["c_attn_w", "c_attn_b", "c_proj_w", "c_proj_b", "c_fc_w", "c_fc_b"]


def _memcpy(dst, src, nbytes, kind):
    from cuda.bindings import runtime as rt
    err, = rt.cudaMemcpy(dst, src, nbytes, kind)
    assert err == rt.cudaError_t.cudaSuccess, err


def memcpy_dtoh(host_arr, dev_ptr):
    from cuda.bindings import runtime as rt
    _memcpy(host_arr.ctypes.data, int(dev_ptr), host_arr.nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)


def memcpy_htod(dev_ptr, host_arr):
    from cuda.bindings import runtime as rt
    host_arr = np.ascontiguousarray(host_arr)
    _memcpy(int(dev_ptr), host_arr.ctypes.data, host_arr.nbytes, rt.cudaMemcpyKind.cudaMemcpyHostToDevice)


def _save_attn(blocks, path):
    """The attention part of GPTModel.save_checkpoint (model/gpt.py:1136-1143)."""
    d = {}
    for idx, attn in enumerate(blocks):
        for attr in ATTRS:
            if hasattr(attn, attr):
                p_obj = getattr(attn, attr)
                host_arr = np.empty(p_obj.shape, dtype=np.float32)
                memcpy_dtoh(host_arr, p_obj.gpu_weights)
                d[f"block_{idx}_attn_{attr}"] = host_arr
    np.savez_compressed(path, **d)
    return d


def _load_attn(blocks, path):
    """The attention part of GPTModel.load_checkpoint (model/gpt.py:1220-1227)."""
    with np.load(path, allow_pickle=False) as data:
        for idx, attn in enumerate(blocks):
            for attr in ATTRS:
                if hasattr(attn, attr):
                    p_obj = getattr(attn, attr)
                    arr = data[f"block_{idx}_attn_{attr}"].astype(np.float32)
                    assert arr.shape == tuple(p_obj.shape)
                    memcpy_htod(p_obj.gpu_weights, arr)


@pytest.mark.parametrize("prec", ["fp32", "bf16"])
def test_checkpoint_round_trip(pkg, cuda_dev, tmp_path, prec):
    import torch
    C, NH, B, T = 64, 4, 2, 33
    cfg = pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T, attention_precision=prec)
    np.random.seed(11)
    saved = [pkg.MultiHeadAttention(cfg) for _ in range(2)]
    for attn in saved:  # non-zero biases so every parameter is visible in the round trip
        attn.c_attn_b.weights.copy_(torch.randn(3 * C) * 0.1)
        attn.c_proj_b.weights.copy_(torch.randn(C) * 0.1)
    path = os.path.join(tmp_path, "gpt_model_latest.npz")
    d = _save_attn(saved, path)
    assert sorted(d) == sorted(f"block_{i}_attn_{a}" for i in range(2) for a in ATTRS[:4])
    shapes = {"c_attn_w": (C, 3 * C), "c_attn_b": (3 * C,), "c_proj_w": (C, C), "c_proj_b": (C,)}
    for k, v in d.items():
        assert v.dtype == np.float32 and v.shape == shapes[k.split("_attn_", 1)[1]], k
    np.random.seed(12)
    loaded = [pkg.MultiHeadAttention(cfg) for _ in range(2)]
    _load_attn(loaded, path)
    x = torch.from_numpy(O.make_config_inputs(1, B, T, C, NH)["x"]).cuda()
    for a, b in zip(saved, loaded):
        for attr in ATTRS[:4]:
            assert torch.equal(getattr(a, attr).weights, getattr(b, attr).weights), attr
        ya, yb = a.forward(x, B, T), b.forward(x, B, T)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ya.get(), yb.get())
        ya.free()
        yb.free()
