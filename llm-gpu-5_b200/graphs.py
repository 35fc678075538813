"""A training or inference step captured once as a CUDA graph and replayed.

The modules' calls are host-light but not free: each enqueues a handful of library launches, a few
tensor allocations and TMA descriptor encodes.  When the GPU side of a step is short (a data-parallel
step at 64 sequences per GPU takes under a millisecond), that host work decides the step time.  A
captured step replays every launch, allocation, the gradient all-reduce and the status-word copy on
the same buffers with one host call.

The reference has no counterpart (PyCUDA launches every kernel from Python, model/gpt.py:531-698);
this is the CUDA-graph replacement for that launch path.

Rules, as for any CUDA graph: the step reads its inputs from, and writes its results to, the same
device buffers on every replay (copy new data into them between replays); the module's parameters
and gradient buffers keep their addresses; modules must have run the step once eagerly before the
capture (so that one-time set-up, such as NCCL communicator creation and the library's per-device
state, happens outside the capture).  While a capture is running the modules cast their float32
weights to bf16 inside the step, so each replay sees the weights as they are at replay time.
"""

from __future__ import annotations

import torch


class CapturedStep:
    """``fn()`` captured into a CUDA graph; ``replay()`` runs it again and returns what the capture
    returned (the same tensors, rewritten by the replay).

    ``pool`` shares one memory pool between several captures (graphs of one pool must not run
    concurrently).  ``stream`` is the stream the capture runs on (by default a side stream torch
    creates); replays go to the current stream."""

    def __init__(self, fn, pool=None, stream=None):
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool, stream=stream):
            self.result = fn()

    def replay(self):
        self.graph.replay()
        return self.result

    def pool(self):
        return self.graph.pool()

    def reset(self):
        """Release the graph (required before destroy_process_group when it holds collectives)."""
        self.graph.reset()
        self.result = None


def capturing() -> bool:
    """Whether the current stream is being captured into a graph."""
    return torch.cuda.is_current_stream_capturing()
