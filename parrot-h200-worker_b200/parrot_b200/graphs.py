"""CUDA-graph replay of ``Parrot.forward`` for a fixed input shape.

The eager forward launches a few hundred kernels from Python (the sm_100a
hot-path kernels through the C ABI plus the PyTorch attention and LM head);
at 1 x 512 tokens the GPU work is well under a millisecond, so the eager
forward is bound by host launch cost.  A captured graph replays the same
launches with no host work per kernel.

Every kernel the B200 backend launches is capturable: the C ABI never
allocates, never synchronises and takes the capturing stream from
``torch.cuda.current_stream()``; outputs come from the graph's private pool.
"""
from __future__ import annotations

import torch
from torch import Tensor


class GraphedForward:
    """``model.forward`` on ``[batch, source_len]`` ids, captured once and replayed.

    ``__call__(input_ids)`` copies the ids (host or device tensor) into the
    captured input buffer, replays the graph on the current stream and returns
    the captured ``ModelOutput``.  Its tensors are overwritten by the next call:
    copy out what must outlive it.  The model's parameters must not be
    reallocated after capture (in-place updates are seen by the next replay;
    call ``invalidate_packed_weights`` and re-capture after changing expert
    weights, because the packed expert copies are captured by address).
    """

    def __init__(self, model, batch: int, source_len: int, *, labels: bool = False,
                 warmup: int = 2, **forward_kwargs):
        if model.training:
            raise RuntimeError("capture requires model.eval()")
        device = next(model.parameters()).device
        if device.type != "cuda":
            raise RuntimeError("capture requires a CUDA model")
        self.model = model
        self.input_ids = torch.zeros((batch, source_len), dtype=torch.long, device=device)
        self.labels = self.input_ids if labels else None
        self.kwargs = forward_kwargs
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.inference_mode():
            with torch.cuda.stream(side):
                for _ in range(max(1, warmup)):
                    model(self.input_ids, self.labels, **forward_kwargs)
            torch.cuda.current_stream(device).wait_stream(side)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.output = model(self.input_ids, self.labels, **forward_kwargs)

    def __call__(self, input_ids: Tensor):
        if tuple(input_ids.shape) != tuple(self.input_ids.shape):
            raise ValueError(f"captured for ids of shape {tuple(self.input_ids.shape)}, "
                             f"got {tuple(input_ids.shape)}")
        self.input_ids.copy_(input_ids, non_blocking=True)
        self.graph.replay()
        return self.output


def capture_calls(fn, repeats: int = 1) -> torch.cuda.CUDAGraph:
    """Capture ``repeats`` calls of ``fn()`` (after one eager warm-up call) in one graph."""
    fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(repeats):
            fn()
    return graph
