"""C-ABI checks that need no GPU: the library loads, exports every declared symbol, and rejects
bad arguments before launching anything (the error path the reference's API raises on,
model/gpt.py:649-650, here as status codes)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT, load_pkg

HEADER = os.path.join(ROOT, "include", "attn_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(attn_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("attn_fwd", "attn_bwd", "attn_decode", "attn_gemm", "attn_colsum", "attn_probs",
              "attn_bwd_workspace_size", "attn_last_error_string", "attn_split_heads",
              "attn_merge_heads", "attn_cast_f32_to_bf16"):
        assert n in names


def test_library_exports_every_declared_symbol():
    pkg = load_pkg()
    raw = ctypes.CDLL(pkg.LIB_PATH)
    for name in declared_functions():
        assert hasattr(raw, name), f"{name} declared in attn_b200.h but not exported"
    # and the Python binding types every one of them
    from importlib import import_module
    lib_mod = import_module("llm-gpu-5_b200._lib")
    assert set(declared_functions()) <= set(lib_mod.SIGNATURES)


def test_bad_arguments_rejected_without_launch():
    pkg = load_pkg()
    L = pkg.lib
    before = pkg.launch_count()
    # null pointers
    rc = L.attn_fwd(None, None, None, None, None, 1, 1, 16, 16, 256, 16, 256, 256, 16, 256, 0.25, 0, None)
    assert rc == -1 and "null" in L.attn_last_error_string().decode()
    fake = 1 << 20  # never dereferenced: validation fails first
    # head_dim not a multiple of 4
    rc = L.attn_fwd(fake, fake, fake, fake, fake, 1, 1, 16, 6, 96, 6, 96, 96, 6, 96, 0.25, 0, None)
    assert rc == -1 and "multiple of 4" in L.attn_last_error_string().decode()
    # bad dtype
    rc = L.attn_fwd(fake, fake, fake, fake, fake, 1, 1, 16, 16, 256, 16, 256, 256, 16, 256, 0.25, 7, None)
    assert rc == -1
    # non-positive sizes
    rc = L.attn_fwd(fake, fake, fake, fake, fake, 0, 1, 16, 16, 256, 16, 256, 256, 16, 256, 0.25, 0, None)
    assert rc == -1
    # backward with a short workspace
    need = L.attn_bwd_workspace_size(2, 2, 64, 16, 0)
    assert need >= 2 * 2 * 64 * 4
    rc = L.attn_bwd(fake, fake, fake, fake, fake, fake, fake, fake, fake, fake, need - 4,
                    2, 2, 64, 16, 2048, 32, 16, 2048, 32, 16, 0.25, 0, None)
    assert rc == -4 and "workspace" in L.attn_last_error_string().decode()
    # gemm: accumulate into a bf16 C is refused
    rc = L.attn_gemm(fake, 64, 0, fake, 64, 0, 1, fake, 64, 1, None, 64, 64, 64, 1, None)
    assert rc == -1
    # gemm: leading dimension too small
    rc = L.attn_gemm(fake, 32, 0, fake, 64, 0, 0, fake, 64, 0, None, 64, 64, 64, 0, None)
    assert rc == -1
    # gemm on a capped number of SMs: a negative cap is refused
    rc = L.attn_gemm_ex(fake, 64, 0, fake, 64, 0, 1, fake, 64, 0, None, 64, 64, 64, 0, -1, None)
    assert rc == -1 and "max_ctas" in L.attn_last_error_string().decode()
    # decode with a head_dim the vector width does not divide
    rc = L.attn_decode(fake, fake, fake, fake, None, 1, 1, 8, 12, 12, 12, 96, 12, 12, 0.3, 1, fake,
                       1 << 20, None)
    assert rc == -1
    # the bounded-wait self-test takes limits of 1 us .. 1 s only
    for limit in (0, -5, 1000001):
        rc = L.attn_wait_selftest(limit, None)
        assert rc == -1 and "limit_us" in L.attn_last_error_string().decode()
    assert pkg.launch_count() == before


def test_workspace_sizes_are_consistent():
    L = load_pkg().lib
    assert L.attn_decode_workspace_size(64, 8, 2048, 64) == 64 * 8 * 8 * 66 * 4
    assert L.attn_colsum_workspace_size(262144, 768) % (768 * 4) == 0
    assert L.attn_bwd_workspace_size(0, 1, 1, 1, 0) == 0


def test_import_fails_loudly_without_library(tmp_path, monkeypatch):
    """The product path has no fallback: a missing .so is an ImportError, not a slow path."""
    import importlib.util
    import sys
    src = os.path.join(ROOT, "llm-gpu-5_b200", "_lib.py")
    spec = importlib.util.spec_from_file_location("_lib_probe", src)
    mod = importlib.util.module_from_spec(spec)
    monkeypatch.setattr(os.path, "exists", lambda p: False if p.endswith("libattn_b200.so") else True)
    with pytest.raises(ImportError, match="no non-CUDA fallback"):
        spec.loader.exec_module(mod)
    sys.modules.pop("_lib_probe", None)


def test_bad_arguments_of_the_block_entry_points():
    """The FFN GEMM, LayerNorm and LayerNorm-backward entry points validate before launching."""
    pkg = load_pkg()
    L = pkg.lib
    before = pkg.launch_count()
    fake = 1 << 20  # never dereferenced: validation fails first
    # unknown activation
    rc = L.attn_gemm_act(fake, 64, 0, fake, 64, 0, 1, fake, 64, 1, None, 64, 64, 64, 9, None, 0, 1, None)
    assert rc == -1 and "activation" in L.attn_last_error_string().decode()
    # GELU backward without the cached pre-activation
    rc = L.attn_gemm_act(fake, 64, 0, fake, 64, 0, 1, fake, 64, 1, None, 64, 64, 64, 2, None, 0, 1, None)
    assert rc == -1 and "aux" in L.attn_last_error_string().decode()
    # the pre-activation output aliasing C
    rc = L.attn_gemm_act(fake, 64, 0, fake, 64, 0, 1, fake, 64, 1, None, 64, 64, 64, 1, fake, 64, 1, None)
    assert rc == -1 and "alias" in L.attn_last_error_string().decode()
    # aux pitch below N
    rc = L.attn_gemm_act(fake, 64, 0, fake, 64, 0, 1, fake, 64, 1, None, 64, 64, 64, 1, fake + 4096, 32, 1, None)
    assert rc == -1 and "ldaux" in L.attn_last_error_string().decode()
    # LayerNorm: eps must be positive, output must not alias the input, ones column needs room
    rc = L.attn_layernorm(fake, 64, fake, fake, 8, 64, 0.0, fake + 8192, 64, 0, 0, None)
    assert rc == -1 and "eps" in L.attn_last_error_string().decode()
    rc = L.attn_layernorm(fake, 64, fake, fake, 8, 64, 1e-5, fake, 64, 0, 0, None)
    assert rc == -1 and "alias" in L.attn_last_error_string().decode()
    rc = L.attn_layernorm(fake, 64, fake, fake, 8, 64, 1e-5, fake + 8192, 64, 1, 1, None)
    assert rc == -1 and "ldy" in L.attn_last_error_string().decode()
    # LayerNorm backward: null pointers, dx aliasing x or dy
    rc = L.attn_layernorm_bwd(None, fake, fake, 8, 64, 1e-5, fake, 0, fake, fake, 0, None)
    assert rc == -1 and "null" in L.attn_last_error_string().decode()
    rc = L.attn_layernorm_bwd(fake, fake + 4096, fake, 8, 64, 1e-5, fake + 4096, 0, fake, fake, 0, None)
    assert rc == -1 and "alias" in L.attn_last_error_string().decode()
    assert pkg.launch_count() == before


def test_decode_rejects_more_than_65535_sequence_heads_without_launch():
    """B*NH is the decode kernel's grid.y: both decode entry points refuse B*NH > 65535 with a
    message before launching (bf16, D = 8, L = 256 would fit the no-allocation array)."""
    pkg = load_pkg()
    L = pkg.lib
    before = pkg.launch_count()
    fake = 1 << 20
    B, NH, Lk, D = 7000, 10, 256, 8
    ws_bytes = L.attn_decode_workspace_size(B, NH, Lk, D)
    assert ws_bytes <= 4 * (1 << 20)
    rc = L.attn_decode(fake, fake, fake, fake, None, B, NH, Lk, D, NH * D, D, Lk * NH * D, NH * D, D,
                       ctypes.c_float(0.35), 1, fake, ws_bytes, None)
    assert rc == -2 and "65535" in L.attn_last_error_string().decode()
    rc = L.attn_decode_noalloc(fake, fake, fake, fake, None, B, NH, Lk, D, NH * D, D, Lk * NH * D, NH * D, D,
                               ctypes.c_float(0.35), 1, None)
    assert rc == -2 and "65535" in L.attn_last_error_string().decode()
    assert pkg.launch_count() == before


def test_backward_beyond_the_tensor_core_row_limit_sizes_the_cuda_core_workspace():
    """Rows longer than the tensor-core backward's limit (2,097,024) go to the CUDA-core backward;
    its workspace (one float per row: delta) is what attn_bwd_workspace_size reports for them."""
    L = load_pkg().lib
    t_max = 2097024
    B, NH, D = 1, 1, 64
    assert L.attn_bwd_workspace_size(B, NH, t_max + 1, D, 1) == B * NH * (t_max + 1) * 4
    assert L.attn_bwd_workspace_size(B, NH, t_max, D, 1) > B * NH * t_max * 4  # the tensor-core layout
