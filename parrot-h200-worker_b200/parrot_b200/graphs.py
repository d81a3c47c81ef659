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
        self.stage(input_ids)
        self.graph.replay()
        return self.output

    def stage(self, input_ids: Tensor) -> None:
        """Copy the next ids into the captured input buffer on the current
        stream, without replaying: a pipelined caller can stage step i + 1's
        ids (on another stream, ordered with events) while step i computes."""
        if tuple(input_ids.shape) != tuple(self.input_ids.shape):
            raise ValueError(f"captured for ids of shape {tuple(self.input_ids.shape)}, "
                             f"got {tuple(input_ids.shape)}")
        self.input_ids.copy_(input_ids, non_blocking=True)

    def replay(self):
        """Replay on the current stream with the ids already staged."""
        self.graph.replay()
        return self.output


class GraphedDecode:
    """``model.decode_step`` on a fixed ``GenerationState``, captured once and replayed.

    The decode kernels read the position from ``state.position_device``, and
    the step ends by incrementing it, so one graph serves every position:
    ``__call__(ids)`` copies the [batch, 1] ids in, replays and advances
    ``state.position``; it returns the captured logits (or next tokens with
    ``next_token_only``), overwritten by the next call.  Decoding the same
    state eagerly in between is fine; replacing its tensors is not.
    """

    def __init__(self, model, state, next_token_only: bool = False):
        if model.training:
            raise RuntimeError("capture requires model.eval()")
        if state.position_device is None:
            raise ValueError("the state has no device position (it did not come from prefill)")
        self.model = model
        self.state = state
        self.next_token_only = next_token_only
        device = state.position_device.device
        self.input_ids = torch.zeros((state.batch_size, 1), dtype=torch.long, device=device)
        position = state.position
        side = torch.cuda.Stream(device=device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.inference_mode():
            with torch.cuda.stream(side):
                # warm-up step (allocates workspaces); its token is rewritten
                # by the first real step at the same position
                model.decode_step(self.input_ids, state, _next_token_only=next_token_only)
                state.position_device.sub_(1)
            torch.cuda.current_stream(device).wait_stream(side)
            state.position = position
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.output, _ = model.decode_step(self.input_ids, state,
                                                   _next_token_only=next_token_only)
            state.position = position  # capture ran the host code, not the kernels

    def __call__(self, input_ids: Tensor):
        state = self.state
        if tuple(input_ids.shape) != tuple(self.input_ids.shape):
            raise ValueError(f"captured for ids of shape {tuple(self.input_ids.shape)}, "
                             f"got {tuple(input_ids.shape)}")
        if state.position >= self.model.config.max_seq_len:
            raise ValueError("Generation state has reached max_seq_len")
        self.input_ids.copy_(input_ids, non_blocking=True)
        self.graph.replay()
        state.position += 1
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
