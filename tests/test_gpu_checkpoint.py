"""Checkpoint-format compatibility of the drop-in attention parameters (model/gpt.py:1103-1243).

``tests/golden/ckpt_gpt_c16_nh2_l2.npz`` was written by the reference's own
GPTModel.save_checkpoint (run by tests/golden/make_golden.py on a small seeded model).  Its
load_checkpoint walks every block's ``attn`` over the attribute names c_attn_w, c_attn_b,
c_proj_w, c_proj_b (c_fc_w / c_fc_b are absent on attention), checks each array's shape against
``p_obj.shape`` and copies it with pycuda's memcpy_htod into ``p_obj.gpu_weights``
(model/gpt.py:1220-1227); save_checkpoint copies back with memcpy_dtoh into
``np.empty(p_obj.shape, float32)`` under ``block_{idx}_attn_{attr}`` (model/gpt.py:1136-1143), and
both check the archive's attention_impl and num_heads against the model config
(model/gpt.py:1196-1205).  These tests drive the drop-in modules through exactly that surface
(``shape``, ``gpu_weights`` as a raw device address, host<->device copies with cuda-python standing
in for pycuda's): the modules loaded from the reference's archive compute what the oracle computes
with its weights, and written back they reproduce the archive's attention arrays bit for bit.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import mha_oracle as O

pytestmark = pytest.mark.gpu
ATTRS = ["c_attn_w", "c_attn_b", "c_proj_w", "c_proj_b", "c_fc_w", "c_fc_b"]
ARCHIVE = os.path.join(GOLDEN, "ckpt_gpt_c16_nh2_l2.npz")


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


def _modules(pkg, data, prec):
    cfg = pkg.GPTConfig(vocab_size=int(data["__meta_vocab_size"]), max_len=int(data["__meta_max_len"]),
                        embedding_dim=int(data["__meta_embedding_dim"]), num_heads=int(data["__meta_num_heads"]),
                        num_layers=int(data["__meta_num_layers"]), attention_precision=prec)
    # the checks load_checkpoint makes against the model config
    assert str(np.asarray(data["__meta_attention_impl"]).item()) == cfg.attention_impl
    assert int(data["__meta_num_heads"]) == cfg.num_heads
    return cfg, [pkg.MultiHeadAttention(cfg) for _ in range(cfg.num_layers)]


def _load(blocks, data):
    for idx, attn in enumerate(blocks):
        for attr in ATTRS:
            if hasattr(attn, attr):
                p_obj = getattr(attn, attr)
                arr = data[f"block_{idx}_attn_{attr}"].astype(np.float32)
                assert arr.shape == tuple(p_obj.shape), (idx, attr)
                memcpy_htod(p_obj.gpu_weights, arr)


def _save(blocks):
    d = {}
    for idx, attn in enumerate(blocks):
        for attr in ATTRS:
            if hasattr(attn, attr):
                p_obj = getattr(attn, attr)
                host_arr = np.empty(p_obj.shape, dtype=np.float32)
                memcpy_dtoh(host_arr, p_obj.gpu_weights)
                d[f"block_{idx}_attn_{attr}"] = host_arr
    return d


@pytest.mark.parametrize("prec,tol", [("fp32", 1e-5), ("bf16", 2e-2)])
def test_reference_checkpoint_loads_computes_and_saves_back(pkg, cuda_dev, tmp_path, prec, tol):
    import torch
    with np.load(ARCHIVE, allow_pickle=False) as f:
        data = {k: f[k] for k in f.files}
    cfg, blocks = _modules(pkg, data, prec)
    _load(blocks, data)
    # written back: the reference's attention arrays, keys, shapes and dtypes, bit for bit
    saved = _save(blocks)
    want = {k: v for k, v in data.items() if "_attn_" in k}
    assert sorted(saved) == sorted(want)
    for k, v in saved.items():
        assert v.dtype == want[k].dtype == np.float32 and v.shape == want[k].shape, k
        np.testing.assert_array_equal(v, want[k], err_msg=k)
    np.savez_compressed(os.path.join(tmp_path, "attn_part.npz"), **saved)  # the archive format round-trips
    # the loaded modules compute the attention of the archive's weights
    B, T, C, NH = 3, cfg.max_len, cfg.embedding_dim, cfg.num_heads
    x = np.random.default_rng(5).standard_normal((B * T, C)).astype(np.float32)
    for idx, attn in enumerate(blocks):
        g = lambda a: data[f"block_{idx}_attn_{a}"]  # noqa: E731
        out = attn.forward(torch.from_numpy(x).cuda(), B, T)
        torch.cuda.synchronize()
        ref, _ = O.mha_forward(x, g("c_attn_w"), g("c_attn_b"), g("c_proj_w"), g("c_proj_b"), B, T, NH)
        assert O.rel_err(out.get(), ref) < tol, (idx, O.rel_err(out.get(), ref))
        out.free()


def test_drop_in_checkpoint_round_trip(pkg, cuda_dev, tmp_path):
    """Modules saved through the reference's loop and loaded into fresh modules compute the same
    output bit for bit."""
    import torch
    with np.load(ARCHIVE, allow_pickle=False) as f:
        data = {k: f[k] for k in f.files}
    cfg, saved = _modules(pkg, data, "bf16")
    np.random.seed(11)
    for attn in saved:  # fresh, different weights
        attn.c_attn_b.weights.copy_(torch.randn(3 * cfg.embedding_dim) * 0.1)
    path = os.path.join(tmp_path, "gpt_model_latest.npz")
    np.savez_compressed(path, **_save(saved))
    np.random.seed(12)
    _, loaded = _modules(pkg, data, "bf16")
    with np.load(path, allow_pickle=False) as f:
        _load(loaded, f)
    B, T, C = 2, cfg.max_len, cfg.embedding_dim
    x = torch.from_numpy(O.make_config_inputs(1, B, T, C, cfg.num_heads)["x"]).cuda()
    for a, b in zip(saved, loaded):
        for attr in ATTRS[:4]:
            assert torch.equal(getattr(a, attr).weights, getattr(b, attr).weights), attr
        ya, yb = a.forward(x, B, T), b.forward(x, B, T)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(ya.get(), yb.get())
        ya.free()
        yb.free()
