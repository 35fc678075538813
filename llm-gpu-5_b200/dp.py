"""Data-parallel plumbing of the attention path: batch sharding and the gradient all-reduce.

The reference trains on one GPU (its only scaling is gradient accumulation, auto_train.py:1591-1615).
Here the path shards by batch: every rank runs the same ``MultiHeadAttention`` (and
``FeedForward``) on its slice of the global batch with replicated weights, and after backward the
four parameter gradients, which each module keeps in one flat fp32 buffer (``[dWqkv | dbqkv | dWo |
dbo]``, ``[dWfc | dbfc | dWproj | dbproj]``), are summed over the ranks with one all-reduce.  SUM makes every rank's gradient equal the single-process full-batch gradient
the reference computes (model/gpt.py:687-694).  Nothing inside attention communicates.
"""

from __future__ import annotations


def shard(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """(first sequence, sequences) of ``rank``'s slice of the global batch.  The batch must split
    evenly: every rank then does the same work and the all-reduce sums equal-sized shards."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if global_batch % world:
        raise ValueError(f"global batch {global_batch} does not split evenly over {world} ranks")
    per = global_batch // world
    return rank * per, per


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= s
    return n


def _layout(params) -> list[tuple[str, int, tuple[int, ...]]]:
    out, off = [], 0
    for name, shape in params:
        out.append((name, off, shape))
        off += _numel(shape)
    return out


def grad_layout(C: int) -> list[tuple[str, int, tuple[int, ...]]]:
    """(parameter, element offset, shape) of each attention gradient inside the flat buffer, in the
    reference's parameter order (model/gpt.py:507-510)."""
    return _layout((("c_attn_w", (C, 3 * C)), ("c_attn_b", (3 * C,)), ("c_proj_w", (C, C)), ("c_proj_b", (C,))))


def ffn_grad_layout(C: int) -> list[tuple[str, int, tuple[int, ...]]]:
    """The same for FeedForward, ``[dWfc | dbfc | dWproj | dbproj]`` (model/gpt.py:305-308).  The
    bias gradient follows its weight gradient, so a weight-gradient GEMM over one extra operand row
    (a ones column in the input) writes both."""
    return _layout((("c_fc_w", (C, 4 * C)), ("c_fc_b", (4 * C,)), ("c_proj_w", (4 * C, C)), ("c_proj_b", (C,))))


def layout_size(layout) -> int:
    name, off, shape = layout[-1]
    return off + _numel(shape)


def flat_grad_size(C: int) -> int:
    return layout_size(grad_layout(C))


def grad_buckets(layout, first_names) -> list[tuple[int, int]]:
    """Split a flat gradient buffer (``layout`` as grad_layout) into two all-reduce buckets: the
    parameters named in ``first_names`` (final earlier in backward, sent first) and the rest, as
    [lo, hi) float ranges in the order they are sent.  Each must be one contiguous run starting on a
    16-byte boundary; otherwise the whole buffer is one bucket."""
    total = layout_size(layout)
    spans = {name: (off, off + _numel(shape)) for name, off, shape in layout}
    first = sorted(spans[n] for n in first_names)
    lo, hi = first[0][0], first[-1][1]
    contiguous = all(a[1] == b[0] for a, b in zip(first, first[1:]))
    if not contiguous or lo % 4 or (lo != 0 and hi != total) or (lo == 0 and hi % 4):
        return [(0, total)]
    rest = (hi, total) if lo == 0 else (0, lo)
    return [(lo, hi), rest]


def allreduce_grads(flat, group=None, async_op: bool = False):
    """Sum the flat gradient buffer over ``group`` in place (one collective; NCCL on GPUs)."""
    import torch.distributed as dist
    return dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=async_op)


def multicast_supported(device_index: int) -> bool:
    """Whether the GPU can bind memory to an NVLink multicast object (NVSwitch NVLS)."""
    import torch
    try:
        sm = torch._C._distributed_c10d._SymmetricMemory
        return bool(sm.has_multicast_support(torch._C._autograd.DeviceType.CUDA, device_index))
    except (AttributeError, RuntimeError):
        return False


class MulticastGradReducer:
    """A flat float32 gradient buffer summed over the ranks of a group by the library's NVSwitch
    multicast all-reduce (``attn_grad_allreduce``) instead of NCCL.

    The buffer is allocated in symmetric memory (torch's plumbing: every rank's buffer is mapped
    at one multicast address, and every rank has a signal pad the others can reach); a module puts
    its gradients in it with ``use_grad_reducer``.  ``allreduce()`` launches one kernel on the
    current stream that meets the other ranks in a cross-GPU barrier, sums the buffer in the
    NVSwitch (each rank reduces and writes back 1/world of it) and meets them again, so it can be
    captured into a CUDA graph like any other launch.  Every rank must call it at the same point.
    """

    def __init__(self, numel: int, group=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        from ._lib import lib
        self.group = group if group is not None else dist.group.WORLD
        self.numel = int(numel)
        self.buffer = symm_mem.empty(self.numel, dtype=torch.float32, device="cuda")
        self.buffer.zero_()
        self.handle = symm_mem.rendezvous(self.buffer, self.group.group_name)
        if not self.handle.multicast_ptr:
            raise RuntimeError("MulticastGradReducer: no multicast address for this group's buffers")
        self.rank, self.world = self.handle.rank, self.handle.world_size
        need = lib.attn_grad_allreduce_signal_bytes(self.numel, self.world)
        if self.handle.signal_pad_size < need:
            raise RuntimeError(f"MulticastGradReducer: signal pads of {self.handle.signal_pad_size} bytes, "
                               f"{need} needed")
        torch.cuda.synchronize()
        dist.barrier(group=self.group)  # every rank's buffer and pads exist before the first launch

    # CTAs of one launch (0: the library's default of 16), the same on every rank, and SMs that the
    # GEMM beside an overlapped reduction leaves to it.  On 8 B200s at 64 sequences per GPU: 16/16
    # 0.828 ms per step, 8/8 0.827, 32/32 0.834, and 32 CTAs sharing the GEMM's SMs 0.874.
    max_blocks = 16
    reserve_sms = 16
    overlap = True  # a module's backward runs the reduction beside its last GEMM (False: after it)

    def gemm_ctas(self) -> int:
        """max_ctas for the GEMM that runs beside this reducer's launch (0: every SM)."""
        if not self.overlap or self.reserve_sms <= 0:
            return 0
        import torch
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        return max(1, sms - int(self.reserve_sms))

    def allreduce(self, lo: int = 0, hi: int = None):
        """Sum floats [lo, hi) of the buffer (all of it by default) over the ranks, in place on every
        rank (one launch, current stream).  ``lo`` must be a multiple of 4 (16-byte aligned)."""
        import torch
        from ._lib import call
        hi = self.numel if hi is None else int(hi)
        lo = int(lo)
        if not 0 <= lo < hi <= self.numel or lo % 4:
            raise ValueError(f"MulticastGradReducer.allreduce: bad range [{lo}, {hi}) of {self.numel} floats")
        call("attn_grad_allreduce", self.handle.multicast_ptr + 4 * lo, self.handle.signal_pad_ptrs_dev,
             self.rank, self.world, hi - lo, self.handle.signal_pad_size, int(self.max_blocks),
             torch.cuda.current_stream().cuda_stream)


def make_grad_reducer(numel: int, group=None):
    """A MulticastGradReducer for ``group`` when every GPU of it supports NVLink multicast and the
    group has 2 to 8 ranks, else None (the modules then all-reduce through NCCL)."""
    import torch
    import torch.distributed as dist
    group = group if group is not None else dist.group.WORLD
    world = dist.get_world_size(group)
    ok = torch.tensor([1 if 2 <= world <= 8 and multicast_supported(torch.cuda.current_device()) else 0],
                      device="cuda")
    dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)  # all ranks take the same decision
    return MulticastGradReducer(numel, group) if int(ok.item()) else None
