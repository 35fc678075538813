"""Data-parallel host logic on CPU ranks (gloo, world size 2).

Each rank takes its shard of the global batch (``dp.shard``), runs the oracle's forward and
backward on it, packs the four parameter gradients into the flat layout the module all-reduces
(``dp.grad_layout``) and sums them with ``dp.allreduce_grads``, bucket by bucket (``dp.grad_buckets``).  The result must equal the
full-batch gradient of one process (the reference's single-GPU semantics, model/gpt.py:687-694),
and each rank's dX must equal its rows of the full-batch dX.  No GPU is used.
"""
import os
import socket

import numpy as np
import pytest

from conftest import load_pkg

B, T, C, NH = 4, 9, 16, 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from oracle import mha_oracle as O
    return O.make_config_inputs(5, B, T, C, NH, seed=123)


def _flat(dp, C, grads):
    out = np.zeros(dp.flat_grad_size(C))
    for (name, off, shape), g in zip(dp.grad_layout(C), grads):
        assert g.shape == shape, (name, g.shape, shape)
        out[off:off + g.size] = g.reshape(-1)
    return out


def _rank(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        from oracle import mha_oracle as O
        dp = load_pkg().dp
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        inp = _inputs()
        first, n = dp.shard(B, world, rank)
        rows = slice(first * T, (first + n) * T)
        out, cache = O.mha_forward(inp["x"][rows], inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], n, T, NH)
        d_in, *grads = O.mha_backward(cache, inp["dy"][rows], inp["w_qkv"], inp["w_o"], n, T, NH)
        flat = torch.from_numpy(_flat(dp, C, grads))
        # the module's two buckets, in the order its backward sends them: dWo/dbo, then dWqkv/dbqkv
        buckets = dp.grad_buckets(dp.grad_layout(C), ("c_proj_w", "c_proj_b"))
        assert len(buckets) == 2
        for lo, hi in buckets:
            dp.allreduce_grads(flat[lo:hi])
        q.put((rank, first, n, flat.numpy(), d_in))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(e), None, None))


@pytest.mark.timeout(300)
def test_two_rank_gradient_sum_equals_full_batch():
    import torch.multiprocessing as mp
    from oracle import mha_oracle as O
    dp = load_pkg().dp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for r in results:
        assert r[1] != "error", r
    inp = _inputs()
    out, cache = O.mha_forward(inp["x"], inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], B, T, NH)
    d_in, *grads = O.mha_backward(cache, inp["dy"], inp["w_qkv"], inp["w_o"], B, T, NH)
    full = _flat(dp, C, grads)
    for rank, first, n, flat, d_in_r in results:
        np.testing.assert_allclose(flat, full, rtol=1e-10, atol=1e-12)
        np.testing.assert_allclose(d_in_r, d_in[first * T:(first + n) * T], rtol=1e-10, atol=1e-12)


def test_shard_and_layout():
    dp = load_pkg().dp
    assert [dp.shard(512, 8, r) for r in (0, 7)] == [(0, 64), (448, 64)]
    with pytest.raises(ValueError):
        dp.shard(10, 4, 0)
    with pytest.raises(ValueError):
        dp.shard(8, 2, 2)
    lay = dp.grad_layout(768)
    assert [(n, o) for n, o, _ in lay] == [("c_attn_w", 0), ("c_attn_b", 768 * 2304),
                                          ("c_proj_w", 768 * 2304 + 2304), ("c_proj_b", 768 * 2304 + 2304 + 768 * 768)]
    assert dp.flat_grad_size(768) == 2362368  # 9.45 MB of fp32 per all-reduce at d_model 768
    # buckets: the output projection's gradients (the tail of the buffer) first, then the rest;
    # both start on 16-byte boundaries and together cover the buffer once
    tail = 768 * 2304 + 2304
    assert dp.grad_buckets(lay, ("c_proj_w", "c_proj_b")) == [(tail, 2362368), (0, tail)]
    flay = dp.ffn_grad_layout(768)
    assert dp.grad_buckets(flay, ("c_proj_w", "c_proj_b")) == [(768 * 3072 + 3072, dp.layout_size(flay)),
                                                               (0, 768 * 3072 + 3072)]
    # a first bucket that is not contiguous or not 16-byte aligned: one bucket for everything
    assert dp.grad_buckets(lay, ("c_attn_w", "c_proj_w")) == [(0, 2362368)]
    odd = dp.grad_layout(3)  # [9*3 | 9 | 3*3 | 3]: the tail starts at float 36, then 45 floats
    assert dp.grad_buckets(odd, ("c_proj_w", "c_proj_b")) == [(36, 48), (0, 36)]
    assert dp.grad_buckets(dp.grad_layout(1), ("c_proj_w", "c_proj_b")) == [(0, 8)]  # tail at float 6


def _rank_that_may_leave(rank, world, port, q):
    """Rank 1 leaves between steps (after joining, before the gradient all-reduce); rank 0 goes on
    to the all-reduce of the flat gradient buffer, which must end with an error, not wait forever."""
    import datetime
    import time
    try:
        import torch
        import torch.distributed as dist
        dp = load_pkg().dp
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        if rank == 1:
            q.put((rank, "left", 0.0))
            q.close()
            q.join_thread()  # the message is out before the process goes
            os._exit(0)  # gone, with no collective in flight
        time.sleep(1.0)  # let the other rank go first
        t0 = time.perf_counter()
        try:
            dp.allreduce_grads(torch.zeros(dp.flat_grad_size(C), dtype=torch.float64))
            q.put((rank, "completed", time.perf_counter() - t0))
        except Exception as e:  # the expected outcome: the collective fails
            q.put((rank, "error:" + type(e).__name__, time.perf_counter() - t0))
        q.close()
        q.join_thread()
        os._exit(0)  # skip destroy_process_group: its peer is gone
    except Exception as e:
        q.put((rank, "setup error " + repr(e), 0.0))


@pytest.mark.timeout(180)
def test_rank_that_leaves_ends_the_survivors_all_reduce_with_an_error():
    """Failure detection on the host: a rank that exits between steps makes the surviving rank's
    next gradient all-reduce raise within the process group's timeout instead of hanging."""
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_that_may_leave, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (what, t)) for r, what, t in (q.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results[1][0] == "left", results
    what, took = results[0]
    assert what.startswith("error:"), results
    assert took < 30.0, results  # bounded by the 10 s process-group timeout (plus slack)
