"""ctypes binding of libattn_b200.so (the C ABI declared in include/attn_b200.h).

The library is the only compute path: if it is missing or fails to load, importing this module
raises.  There is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libattn_b200.so")

ATTN_OK = 0
ATTN_ERR_ARG = -1
ATTN_ERR_UNSUPPORTED = -2
ATTN_ERR_CUDA = -3
ATTN_ERR_WORKSPACE = -4
ATTN_F32 = 0
ATTN_BF16 = 1
ATTN_TF32 = 2
ATTN_ACT_NONE = 0
ATTN_ACT_GELU = 1
ATTN_ACT_GELU_BWD = 2
ATTN_SELFTEST_SITE = 900

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); every function include/attn_b200.h declares
SIGNATURES = {
    "attn_version": (_i, []),
    "attn_last_error_string": (ctypes.c_char_p, []),
    "attn_launch_count": (ctypes.c_uint64, []),
    "attn_device_error": (_i, [_i]),
    "attn_device_error_async": (_i, [_p, _p]),
    "attn_wait_selftest": (_i, [_i, _p]),
    "attn_fwd": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i64, _i64, _i64, _i64, _i64, _i64, _f, _i, _p]),
    "attn_bwd_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "attn_bwd": (_i, [_p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _sz, _i, _i, _i, _i,
                      _i64, _i64, _i64, _i64, _i64, _i64, _f, _i, _p]),
    "attn_decode_workspace_size": (_sz, [_i, _i, _i, _i]),
    "attn_decode": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i64, _i64, _i64, _i64, _i64, _f, _i,
                         _p, _sz, _p]),
    "attn_decode_noalloc": (_i, [_p, _p, _p, _p, _p, _i, _i, _i, _i, _i64, _i64, _i64, _i64, _i64, _f,
                                 _i, _p]),
    "attn_probs": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i64, _i64, _i64, _f, _i, _p]),
    "attn_gemm": (_i, [_p, _i64, _i, _p, _i64, _i, _i, _p, _i64, _i, _p, _i, _i, _i, _i, _p]),
    "attn_gemm_ex": (_i, [_p, _i64, _i, _p, _i64, _i, _i, _p, _i64, _i, _p, _i, _i, _i, _i, _i, _p]),
    "attn_gemm_act": (_i, [_p, _i64, _i, _p, _i64, _i, _i, _p, _i64, _i, _p, _i, _i, _i, _i, _p, _i64, _i, _p]),
    "attn_colsum_workspace_size": (_sz, [_i, _i]),
    "attn_colsum": (_i, [_p, _i, _i64, _i, _i, _p, _i, _p, _sz, _p]),
    "attn_cast_f32_to_bf16": (_i, [_p, _p, _i64, _p]),
    "attn_cast_rows_ones_bf16": (_i, [_p, _i64, _i, _i, _p, _i64, _p]),
    "attn_layernorm": (_i, [_p, _i64, _p, _p, _i, _i, _f, _p, _i64, _i, _i, _p]),
    "attn_layernorm_bwd": (_i, [_p, _p, _p, _i, _i, _f, _p, _i, _p, _p, _i, _p]),
    "attn_cast_colsum_f32": (_i, [_p, _i64, _i, _i, _p, _i64, _p, _i, _p, _sz, _p]),
    "attn_split_heads": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "attn_merge_heads": (_i, [_p, _p, _i, _i, _i, _i, _p]),
    "attn_grad_allreduce_signal_bytes": (_sz, [_i64, _i]),
    "attn_grad_allreduce": (_i, [_p, _p, _i, _i, _i64, _sz, _i, _p]),
}


class AttnError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, fn, code, msg):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `python llm-gpu-5_b200/build.py` "
                          "(or __graft_entry__.build()); there is no non-CUDA fallback")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    s = lib.attn_last_error_string()
    return s.decode() if s else ""


def call(name, *args):
    """Call a status-returning entry point and raise AttnError on failure."""
    rc = getattr(lib, name)(*args)
    if rc != ATTN_OK:
        raise AttnError(name, rc, last_error())
    return rc


def launch_count() -> int:
    return int(lib.attn_launch_count())


# ---------------------------------------------------------------- device status word
# A bounded wait inside a tensor-core kernel that gives up leaves a site code in the library's
# device status word (attn_device_error) and that launch's outputs incomplete.  The modules watch
# the word without synchronising: after each call they enqueue a copy of it into pinned host
# memory (attn_device_error_async), and at the start of the next call they read that memory and
# raise DeviceWaitError if it is set.  The word keeps its code until clear_device_error().
_watch = {}  # device index -> pinned int32 host tensor holding the last copy of the word


class DeviceWaitError(AttnError):
    """A bounded wait inside one of the library's kernels gave up: some call's outputs are
    incomplete.  The reference raises on a failed launch (PyCUDA's LaunchError); this is its
    counterpart for a kernel that gave up instead of hanging."""

    def __init__(self, site):
        RuntimeError.__init__(self, f"a bounded wait in a tensor-core kernel gave up (site {site}); the "
                              "outputs of a recent call are incomplete.  clear_device_error() resets the status")
        self.code = ATTN_ERR_CUDA
        self.site = site


def _slot():
    import torch
    dev = torch.cuda.current_device()
    buf = _watch.get(dev)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        _watch[dev] = buf
    return buf


def watch_device_error():
    """Enqueue, on the current stream, a copy of the device status word into pinned memory."""
    import torch
    call("attn_device_error_async", _slot().data_ptr(), torch.cuda.current_stream().cuda_stream)


def check_device_error():
    """Raise DeviceWaitError if the last copy of the status word that has landed shows a code."""
    import torch
    buf = _watch.get(torch.cuda.current_device())
    if buf is not None:
        site = int(buf[0])
        if site:
            raise DeviceWaitError(site)


def clear_device_error() -> int:
    """Wait for the device, read and clear its status word; returns the code it held."""
    import torch
    torch.cuda.synchronize()
    site = lib.attn_device_error(1)
    buf = _watch.get(torch.cuda.current_device())
    if buf is not None:
        buf.zero_()
    return site
