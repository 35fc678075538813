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


def _layout(params) -> list[tuple[str, int, tuple[int, ...]]]:
    out, off = [], 0
    for name, shape in params:
        out.append((name, off, shape))
        n = 1
        for s in shape:
            n *= s
        off += n
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
    n = 1
    for s in shape:
        n *= s
    return off + n


def flat_grad_size(C: int) -> int:
    return layout_size(grad_layout(C))


def allreduce_grads(flat, group=None, async_op: bool = False):
    """Sum the flat gradient buffer over ``group`` in place (one collective; NCCL on GPUs)."""
    import torch.distributed as dist
    return dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group, async_op=async_op)
