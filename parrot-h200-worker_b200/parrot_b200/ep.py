"""Expert parallelism for the MoE block.

The reference runs every expert of a layer on one device
(``parrot/model.py:521-551``).  Here ``G`` ranks (one process per GPU) each
hold their own tokens and ``n_experts / G`` experts, placed round-robin —
expert ``e`` lives on rank ``e % G`` as local expert ``e // G`` — so the
heavy head of a skewed (Zipf) routing distribution lands on different ranks.
One MoE call on a rank:

1. dispatch: router, top-2 and grouping of the local tokens; the grouped rows
   come out packed by destination rank, then local expert, then ascending
   token (``parrot_moe_ep_dispatch_bf16``);
2. all-to-all of the ``[G, E/G]`` per-(destination, local expert) row counts;
3. one host read of the counts: the split sizes of the variable all-to-all;
4. all-to-all of the token rows (the shared expert on the local tokens was
   queued before the host read, so the GPU computes it while the host waits);
5. the local experts on the received rows, one segment per (source rank,
   local expert) (``parrot_moe_expert_ffn_bf16``);
6. the reverse all-to-all of the expert outputs, back into the dispatch's
   grouped-row order;
7. combine: shared output + route-weighted outputs in ascending expert id
   (+ residual) (``parrot_moe_ep_combine_bf16``).

The result equals the single-device block bit for bit: every row meets the
same GEMM arithmetic, and the combine adds the same bf16 values in the same
order.  The exchanges go through a small communicator interface so the same
orchestration runs over NCCL (``TorchComm``) or, in tests, gloo on CPU with
the oracle's arithmetic in place of the kernels.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Protocol

import torch
from torch import Tensor

from . import _lib, bridge


def owner(expert: int, ranks: int) -> int:
    """Rank that holds ``expert`` (round-robin placement)."""
    return expert % ranks


def local_experts(rank: int, ranks: int, n_experts: int) -> list[int]:
    """Global ids of the experts on ``rank``, in local-index order."""
    if n_experts % ranks:
        raise ValueError(f"n_experts={n_experts} is not divisible by {ranks} ranks")
    return list(range(rank, n_experts, ranks))


def send_counts(counts: Tensor, ranks: int) -> Tensor:
    """Per-expert counts ``[E]`` -> ``[G, E/G]``: rows bound for (rank r, local j).

    Local expert ``j`` of rank ``r`` is global expert ``r + j * G``.
    """
    return counts.view(-1, ranks).t().contiguous()


@dataclass
class Segments:
    """Received-row segments: one per (source rank, local expert), in that order."""
    rows: list[int]
    base: list[int]
    expert: list[int]
    total: int


def receive_segments(recv: list[list[int]]) -> Segments:
    """``recv[src][j]``: rows that source ``src`` sends for local expert ``j``.

    The received buffer is ordered source-major (the all-to-all concatenates
    sources), and within a source by local expert (the dispatch's packing).
    """
    rows, base, expert = [], [], []
    at = 0
    for per_src in recv:
        for j, n in enumerate(per_src):
            rows.append(int(n))
            base.append(at)
            expert.append(j)
            at += int(n)
    return Segments(rows, base, expert, at)


class Comm(Protocol):
    rank: int
    size: int

    def all_to_all(self, out: Tensor, inp: Tensor, out_splits: list[int] | None,
                   in_splits: list[int] | None, async_op: bool = False):
        """Variable all-to-all (``torch.distributed.all_to_all_single`` semantics)."""


class TorchComm:
    """``torch.distributed`` process group (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self._dist = dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)

    def all_to_all(self, out, inp, out_splits, in_splits, async_op=False):
        return self._dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group,
                                            async_op=async_op)


class EpOps(Protocol):
    """The local compute of one rank (B200 kernels, or the oracle in tests)."""

    def dispatch(self, x: Tensor) -> tuple[Tensor, Tensor]:
        """-> (grouped rows [2T, d] packed destination-major, counts [E] int32)."""

    def shared(self, x: Tensor) -> None:
        """Shared expert on the local tokens (kept for ``combine``)."""

    def experts(self, rows: Tensor, seg: Segments) -> Tensor:
        """Local experts on received rows -> outputs [rows, d], same order."""

    def combine(self, y: Tensor, residual: Tensor | None) -> Tensor:
        """Shared + weighted expert outputs (+ residual) -> [T, d]."""


class ExpertParallelMoE:
    """Runs one MoE layer expert-parallel over ``comm``'s ranks."""

    def __init__(self, ops: EpOps, comm: Comm, n_experts: int):
        if n_experts % comm.size:
            raise ValueError(f"n_experts={n_experts} is not divisible by {comm.size} ranks")
        self.ops = ops
        self.comm = comm
        self.n_experts = n_experts
        self.last_recv_rows = 0

    def __call__(self, x: Tensor, residual: Tensor | None = None) -> Tensor:
        G = self.comm.size
        El = self.n_experts // G
        rows, counts = self.ops.dispatch(x)
        send = send_counts(counts.to(torch.int32), G).view(-1)
        recv = torch.empty_like(send)
        self.comm.all_to_all(recv, send, None, None)
        both = torch.cat([send, recv])
        self.ops.shared(x)  # the GPU computes the shared expert while the host waits below
        both = both.cpu().view(2, G, El)  # the one host sync: split sizes of the row exchange
        send_split = both[0].sum(1).tolist()
        recv_tab = both[1].tolist()
        recv_split = [sum(r) for r in recv_tab]
        seg = receive_segments(recv_tab)
        received = rows.new_empty((seg.total, rows.shape[1]))
        self.comm.all_to_all(received, rows[:sum(send_split)], recv_split, send_split)
        y_local = self.ops.experts(received, seg)
        y_back = rows.new_empty((sum(send_split), rows.shape[1]))
        self.comm.all_to_all(y_back, y_local, send_split, recv_split)
        self.last_recv_rows = seg.total
        return self.ops.combine(y_back, residual)


class B200EpOps:
    """B200 kernels for one rank: packed weights of its local experts only."""

    def __init__(self, module, rank: int, ranks: int):
        cfg = module.cfg
        self.module = module
        self.cfg = cfg
        self.ranks = ranks
        self.local = local_experts(rank, ranks, cfg.n_experts)
        router, gate_up, down, sgu, sd = bridge.pack_weights(module)
        idx = torch.tensor(self.local, device=gate_up.device)
        # packed tiles of one expert are contiguous, so selecting experts keeps the layout
        self.gate_up = gate_up.index_select(0, idx).contiguous()
        self.down = down.index_select(0, idx).contiguous()
        self.packed = (router, gate_up, down, sgu, sd)
        self.bias = bridge._router_bias(module)
        self._ws: dict[int, Tensor] = {}
        self.status = torch.zeros(4, device=gate_up.device, dtype=torch.int32)
        self._x = None
        self._dims = None

    def _workspace(self, dims) -> Tensor:
        ws = self._ws.get(dims.tokens)
        if ws is None:
            layout = bridge.workspace_layout(dims)
            ws = torch.zeros(int(layout.total), device=self.gate_up.device, dtype=torch.uint8)
            self._ws[dims.tokens] = ws
        return ws

    def dispatch(self, x: Tensor) -> tuple[Tensor, Tensor]:
        bridge._require_device(x, "MoE")
        bridge._require_inference("MoE")
        x = x.contiguous()
        T, d = x.shape
        dims = bridge.moe_dims(self.cfg, T, capacity=-1)
        ws = self._workspace(dims)
        lay = bridge.workspace_layout(dims)
        counts = torch.empty(self.cfg.n_experts, device=x.device, dtype=torch.int32)
        outputs = _lib.MoeOutputs(None, None, None, None, None, None, counts.data_ptr(), None)
        w = bridge._weights_struct(self.packed, self.bias)
        _lib.check(_lib.load().parrot_moe_ep_dispatch_bf16(
            ctypes.byref(dims), ctypes.byref(w), bridge._p(x), ctypes.byref(outputs), self.ranks,
            bridge._p(ws), ws.numel(), bridge._stream()), "parrot_moe_ep_dispatch_bf16")
        if T == 0:
            counts.zero_()
        self._x, self._dims = x, dims
        rows = ws[lay.grouped:lay.grouped + 2 * T * d * 2].view(torch.bfloat16).view(2 * T, d)
        return rows, counts

    def shared(self, x: Tensor) -> None:
        dims = self._dims
        ws = self._workspace(dims)
        w = bridge._weights_struct(self.packed, self.bias)
        _lib.check(_lib.load().parrot_moe_shared_ffn_bf16(
            ctypes.byref(dims), ctypes.byref(w), bridge._p(self._x), bridge._p(ws), ws.numel(),
            bridge._stream()), "parrot_moe_shared_ffn_bf16")

    def experts(self, rows: Tensor, seg: Segments) -> Tensor:
        cfg = self.cfg
        y = torch.empty_like(rows)
        if seg.total == 0:
            return y
        tab = torch.tensor([seg.rows, seg.base, seg.expert], dtype=torch.int32).pin_memory()
        tab = tab.to(rows.device, non_blocking=True)
        hidden = torch.empty((seg.total, cfg.expert_dim), device=rows.device, dtype=rows.dtype)
        n = len(seg.rows)
        _lib.check(_lib.load().parrot_moe_expert_ffn_bf16(
            seg.total, cfg.dim, cfg.expert_dim, len(self.local), n, bridge._p(tab[0]),
            bridge._p(tab[1]), bridge._p(tab[2]), bridge._p(self.gate_up), bridge._p(self.down),
            bridge._p(rows), bridge._p(hidden), bridge._p(y), bridge._p(self.status),
            bridge._stream()), "parrot_moe_expert_ffn_bf16")
        return y

    def combine(self, y: Tensor, residual: Tensor | None) -> Tensor:
        dims = self._dims
        ws = self._workspace(dims)
        out = torch.empty_like(self._x)
        if residual is not None:
            residual = residual.reshape(out.shape).contiguous()
        _lib.check(_lib.load().parrot_moe_ep_combine_bf16(
            ctypes.byref(dims), bridge._p(y), bridge._p(ws), ws.numel(), bridge._p(residual),
            bridge._p(out), bridge._stream()), "parrot_moe_ep_combine_bf16")
        return out
