"""Data-parallel gradient sums on two GPUs, run as two spawned processes (skipped with one GPU).

* ``attn_grad_allreduce`` (the NVSwitch multicast all-reduce) against the sum computed exactly on
  the host: buffers whose values are small integers (exact in float32), three calls in a row (the
  signal pads are reused) and a call replayed from a captured CUDA graph; a buffer size that is not a
  multiple of 4 floats (the scalar tail).
  A bucket (a sub-range) is summed alone and the rest of the buffer is left as it was.
* a data-parallel step: each rank runs MultiHeadAttention forward + backward on half of the batch
  with its gradients in a MulticastGradReducer (two buckets, then one) or summed by NCCL (two
  buckets); the summed gradients match those of one module that sees the whole batch
  (model/gpt.py:687-694), fp32 within 1e-5 and bf16 within 2e-2.
The multicast cases use NCCL only for the process group and its barrier.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, result_dir):
    import datetime
    import importlib
    import sys

    import torch
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    pkg = importlib.import_module("llm-gpu-5_b200")
    from oracle import mha_oracle as O
    out = {}
    try:
        if not pkg.dp.multicast_supported(rank):
            out["skip"] = "no NVLink multicast"
            return
        # ---- the all-reduce alone
        for n in (1000003, 2362368):
            red = pkg.dp.MulticastGradReducer(n)
            g = torch.Generator(device="cuda")
            base = [torch.randint(-50, 50, (n,), generator=g.manual_seed(17 + r), device="cuda").float()
                    for r in range(world)]
            want = sum(base)
            for it in range(3):
                red.buffer.copy_(base[rank] * (it + 1))
                red.allreduce()
                torch.cuda.synchronize()
                out[f"ar{n}_{it}"] = float((red.buffer - want * (it + 1)).abs().max())
            red.buffer.copy_(base[rank])
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                red.allreduce()
            red.buffer.copy_(base[rank])
            graph.replay()
            torch.cuda.synchronize()
            out[f"ar{n}_graph"] = float((red.buffer - want).abs().max())
            graph.reset()
            # a bucket [lo, hi): only it is summed, the rest of the buffer is left alone
            lo, hi = 4 * (n // 12), n - 5
            red.buffer.copy_(base[rank])
            red.allreduce(lo, hi)
            torch.cuda.synchronize()
            expect = base[rank].clone()
            expect[lo:hi] = want[lo:hi]
            out[f"ar{n}_bucket"] = float((red.buffer - expect).abs().max())
            del red
            dist.barrier()
        # ---- a data-parallel step against the whole batch on one module: the multicast all-reduce
        # with two buckets and with one (the default), and NCCL with two buckets
        for prec, tol, mode in (("fp32", 1e-5, "mc2"), ("bf16", 2e-2, "mc2"), ("bf16", 2e-2, "mc1"),
                                ("bf16", 2e-2, "nccl2")):
            B, T, C, NH = 4, 130, 128, 2
            inp = O.make_config_inputs(9, B, T, C, NH)
            cfg = pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T, attention_precision=prec)
            mods = [pkg.MultiHeadAttention(cfg) for _ in range(2)]
            for m in mods:
                for p, k in ((m.c_attn_w, "w_qkv"), (m.c_attn_b, "b_qkv"), (m.c_proj_w, "w_o"), (m.c_proj_b, "b_o")):
                    p.weights.copy_(torch.from_numpy(inp[k]))
            dp_mod, full = mods
            red = None
            if mode != "nccl2":
                red = pkg.dp.MulticastGradReducer(dp_mod.flat_grads.numel())
                dp_mod.use_grad_reducer(red)
            dp_mod.grad_buckets = mode != "mc1"
            dp_mod.grad_sync_group = dist.group.WORLD
            b0, nb = pkg.dp.shard(B, world, rank)
            x = torch.from_numpy(inp["x"]).cuda().view(B, T, C)
            dy = torch.from_numpy(inp["dy"]).cuda().view(B, T, C)
            dp_mod.forward(x[b0:b0 + nb].reshape(-1, C).contiguous(), nb, T).free()
            dp_mod.backward(dy[b0:b0 + nb].reshape(-1, C).contiguous(), nb, T).free()
            dp_mod.wait_grad_sync()
            full.forward(x.reshape(-1, C), B, T).free()
            full.backward(dy.reshape(-1, C), B, T).free()
            torch.cuda.synchronize()
            out[f"step_{prec}_{mode}"] = O.rel_err(dp_mod.flat_grads.double().cpu().numpy(),
                                                   full.flat_grads.double().cpu().numpy())
            out[f"tol_{prec}_{mode}"] = tol
            dp_mod.grad_sync_group = None
            del red
            dist.barrier()
        out["device_error"] = pkg.lib.attn_device_error(0)
    finally:
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), out, allow_pickle=True)
        dist.barrier()
        dist.destroy_process_group()


def test_multicast_allreduce_and_data_parallel_step(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        res = np.load(os.path.join(tmp_path, f"rank{r}.npy"), allow_pickle=True).item()
        if "skip" in res:
            pytest.skip(res["skip"])
        for k, v in res.items():
            if k.startswith("ar"):
                assert v == 0.0, (r, k, v)
        steps = [k for k in res if k.startswith("step_")]
        assert len(steps) == 4, res
        for k in steps:
            assert res[k] < res["tol_" + k[5:]], (r, k, res[k])
        assert res["device_error"] == 0
