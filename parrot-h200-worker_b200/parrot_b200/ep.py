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

On GPUs of one node the product path is ``PeerExpertParallelMoE``: the same
seven steps with the exchange done by this library's kernels through the
other ranks' memory (CUDA IPC mappings over NVLink / NVSwitch) instead of
NCCL, with the split sizes kept on the device — no host read, fixed-size
regions sized by the largest token count, so a layer can be captured in a
CUDA graph (``parrot_moe_ep_send_bf16`` … ``parrot_moe_ep_combine_peer_bf16``).
By default the two row exchanges have no copy kernel of their own: the
grouping kernel stores each dispatched row straight into its destination's
receive region, and the expert down GEMM stores each output straight into
its source's return region (``parrot_moe_ep_dispatch_send_bf16``,
``parrot_moe_ep_experts_return_bf16``), so the NVLink traffic overlaps the
grouping and the GEMM instead of following them.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Protocol

import torch
from torch import Tensor

from . import _lib, bridge

# PeerExpertParallelMoE defaults: rows stored into the peers' regions by the
# grouping kernel and the down GEMM (True) or by separate copy kernels; the
# shared expert on a side stream beside the dispatch and exchange (True) or
# on the layer's stream after the send.
FUSED_EXCHANGE = True
OVERLAP_SHARED = True


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


class ExchangeError(RuntimeError):
    """A rank received a count table that cannot be right."""


def check_count_table(table: Tensor, rank: int, max_rows: int | None) -> None:
    """``table`` [G, El + 1]: row ``s`` holds source ``s``'s row counts for this
    rank's local experts, then their total.  Raises ``ExchangeError`` for a
    negative count, a total that is not the sum of the counts, or a total
    above ``max_rows`` (what one source can send at most)."""
    counts, totals = table[:, :-1], table[:, -1]
    for s in range(table.shape[0]):
        if (counts[s] < 0).any() or int(counts[s].sum()) != int(totals[s]) or (
                max_rows is not None and int(totals[s]) > max_rows):
            raise ExchangeError(f"rank {rank}: inconsistent count table from rank {s}: "
                                f"{table[s].tolist()}")


class ExpertParallelMoE:
    """Runs one MoE layer expert-parallel over ``comm``'s ranks.

    ``max_rows_per_source`` (optional) bounds the rows one source may send to
    one rank (twice the most tokens a rank holds); a count table above it, or
    one whose total disagrees with its counts, raises ``ExchangeError`` before
    any row is exchanged.  A rank that fails or leaves makes the others'
    next exchange fail with the process group's error (its timeout)."""

    def __init__(self, ops: EpOps, comm: Comm, n_experts: int,
                 max_rows_per_source: int | None = None):
        if n_experts % comm.size:
            raise ValueError(f"n_experts={n_experts} is not divisible by {comm.size} ranks")
        self.ops = ops
        self.comm = comm
        self.n_experts = n_experts
        self.max_rows = max_rows_per_source
        self.last_recv_rows = 0

    def __call__(self, x: Tensor, residual: Tensor | None = None) -> Tensor:
        G = self.comm.size
        El = self.n_experts // G
        rows, counts = self.ops.dispatch(x)
        table = send_counts(counts.to(torch.int32), G)
        send = torch.cat([table, table.sum(1, keepdim=True)], 1).view(-1)
        recv = torch.empty_like(send)
        self.comm.all_to_all(recv, send, None, None)
        both = torch.cat([send, recv])
        self.ops.shared(x)  # the GPU computes the shared expert while the host waits below
        both = both.cpu().view(2, G, El + 1)  # the one host sync: split sizes of the row exchange
        check_count_table(both[1], self.comm.rank, self.max_rows)
        send_split = both[0, :, El].tolist()
        recv_tab = both[1, :, :El].tolist()
        recv_split = both[1, :, El].tolist()
        seg = receive_segments(recv_tab)
        received = rows.new_empty((seg.total, rows.shape[1]))
        self.comm.all_to_all(received, rows[:sum(send_split)], recv_split, send_split)
        y_local = self.ops.experts(received, seg)
        y_back = rows.new_empty((sum(send_split), rows.shape[1]))
        self.comm.all_to_all(y_back, y_local, send_split, recv_split)
        self.last_recv_rows = seg.total
        return self.ops.combine(y_back, residual)


class B200EpOps:
    """B200 kernels for one rank: packed weights of its local experts only
    (``slots``: their global ids in slot order; round-robin by default)."""

    def __init__(self, module, rank: int, ranks: int, slots: list[int] | None = None):
        cfg = module.cfg
        self.module = module
        self.cfg = cfg
        self.ranks = ranks
        self.local = list(slots) if slots is not None else local_experts(rank, ranks,
                                                                          cfg.n_experts)
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


# ---- the peer-memory exchange (one node, one process per GPU) -------------------

@dataclass(frozen=True)
class Placement:
    """Which experts each rank holds and which rank computes a source's rows.

    ``slots[q]``: the global experts rank ``q`` holds, in slot order.  An
    expert in every rank's slots is *replicated*: each source computes its own
    rows of it (data parallel); any other expert has one owner, which computes
    every source's rows of it.
    """
    ranks: int
    n_experts: int
    slots: tuple[tuple[int, ...], ...]

    def __post_init__(self):
        held = [e for q in self.slots for e in q]
        if len(self.slots) != self.ranks or sorted(set(held)) != list(range(self.n_experts)):
            raise ValueError("every expert must be held by at least one rank")
        for e in set(held):
            n = held.count(e)
            if n not in (1, self.ranks):
                raise ValueError(f"expert {e} must be held by one rank or by all of them")
        if any(len(set(q)) != len(q) for q in self.slots):
            raise ValueError("a rank holds an expert twice")

    @property
    def replicated(self) -> frozenset[int]:
        return frozenset(self.slots[0]).intersection(*map(set, self.slots[1:])) \
            if self.ranks > 1 else frozenset()

    @staticmethod
    def round_robin(ranks: int, n_experts: int) -> "Placement":
        return Placement(ranks, n_experts,
                         tuple(tuple(local_experts(r, ranks, n_experts)) for r in range(ranks)))

    @staticmethod
    def balanced(counts: list[int], ranks: int) -> "Placement":
        """For routing with counts ``counts`` [E]: an expert with more than
        1 / ranks of the assignments is replicated on every rank; the others
        go largest first to the rank with the least load so far (its share of
        the replicated experts' rows included)."""
        E = len(counts)
        total = max(1, sum(counts))
        hot = [e for e in range(E) if ranks > 1 and counts[e] * ranks > total]
        load = [sum(counts[e] for e in hot) / ranks] * ranks
        owned: list[list[int]] = [[] for _ in range(ranks)]
        for e in sorted((e for e in range(E) if e not in hot), key=lambda e: (-counts[e], e)):
            q = min(range(ranks), key=lambda r: (load[r], len(owned[r]), r))
            owned[q].append(e)
            load[q] += counts[e]
        return Placement(ranks, E, tuple(tuple(sorted(hot + owned[q])) for q in range(ranks)))

    def dest(self, source: int, expert: int) -> int:
        """The rank that computes ``source``'s rows of ``expert``."""
        if expert in self.replicated:
            return source
        return next(q for q, held in enumerate(self.slots) if expert in held)

    def plan(self, source: int) -> list[list[int]]:
        """plan[q][j]: the expert of rank q's slot j whose rows ``source``
        sends there, or -1."""
        return [[e if self.dest(source, e) == q else -1 for e in held] for q, held in
                enumerate(self.slots)]


@dataclass(frozen=True)
class EpShape:
    """Sizes of one expert-parallel set: ``max_tokens`` bounds every rank's
    tokens per call and sizes the fixed receive and return regions;
    ``placement`` (round-robin when None) says which rank holds which expert."""
    ranks: int
    max_tokens: int
    dim: int
    n_experts: int
    expert_dim: int
    wait_ns: int = 0  # limit of each device-side flag wait; 0 = 2 s
    placement: Placement | None = None

    def dims(self, rank: int) -> _lib.EpDims:
        d = _lib.EpDims(self.ranks, rank, self.max_tokens, self.dim, self.n_experts,
                        self.expert_dim, self.wait_ns)
        if self.placement is not None:
            d.slots = len(self.placement.slots[rank])
            for q, row in enumerate(self.placement.plan(rank)):
                for j, e in enumerate(row):
                    d.plan[q][j] = e
                for j in range(len(row), 32):
                    d.plan[q][j] = -1
        return d

    def slots(self, rank: int) -> list[int]:
        if self.placement is None:
            return local_experts(rank, self.ranks, self.n_experts)
        return list(self.placement.slots[rank])

    def layout(self) -> _lib.EpLayout:
        lay = _lib.EpLayout()
        _lib.check(_lib.load().parrot_ep_buffer_layout(ctypes.byref(self.dims(0)),
                                                       ctypes.byref(lay)), "EP buffer layout")
        return lay


class PeerSet:
    """Every rank's EP buffer as this rank sees it.

    ``connect`` maps the other processes' buffers with CUDA IPC (set-up only:
    one all-gather of the handles over the process group); ``local`` builds all
    ranks' buffers in this process on one device, for running the ranks one
    after another on a single GPU.
    """

    def __init__(self, shape: EpShape, rank: int, own: Tensor, pointers: list[int],
                 mapped: list[int] | None = None):
        self.shape = shape
        self.rank = rank
        self.own = own
        self.pointers = pointers
        self._mapped = mapped or []
        self.dims = shape.dims(rank)
        self.peers = _lib.EpPeers()
        for r, p in enumerate(pointers):
            self.peers.buffers[r] = p

    @staticmethod
    def _allocate(shape: EpShape, device) -> Tensor:
        # zero-filled once: flags, epoch and counters start at 0
        return torch.zeros(int(shape.layout().total), device=device, dtype=torch.uint8)

    @classmethod
    def connect(cls, shape: EpShape, group=None) -> "PeerSet":
        import torch.distributed as dist
        rank, ranks = dist.get_rank(group), dist.get_world_size(group)
        if ranks != shape.ranks:
            raise ValueError(f"process group has {ranks} ranks, the EP shape {shape.ranks}")
        lib = _lib.load()
        own = cls._allocate(shape, torch.device("cuda", torch.cuda.current_device()))
        handle = (ctypes.c_ubyte * 64)()
        offset = ctypes.c_ulonglong()
        _lib.check(lib.parrot_ipc_export(ctypes.c_void_p(own.data_ptr()), handle,
                                         ctypes.byref(offset)), "parrot_ipc_export")
        torch.cuda.synchronize()  # the zero fill is done before any peer writes
        gathered: list = [None] * ranks
        dist.all_gather_object(gathered, (bytes(handle), offset.value), group=group)
        pointers, mapped = [], []
        for r, (h, off) in enumerate(gathered):
            if r == rank:
                pointers.append(own.data_ptr())
                continue
            ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
            buf = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            _lib.check(lib.parrot_ipc_import(buf, off, ctypes.byref(ptr), ctypes.byref(base)),
                       "parrot_ipc_import")
            pointers.append(ptr.value)
            mapped.append(base.value)
        dist.barrier(group=group)
        return cls(shape, rank, own, pointers, mapped)

    @classmethod
    def local(cls, shape: EpShape, device) -> list["PeerSet"]:
        bufs = [cls._allocate(shape, device) for _ in range(shape.ranks)]
        ptrs = [b.data_ptr() for b in bufs]
        return [cls(shape, r, bufs[r], ptrs) for r in range(shape.ranks)]

    def status(self) -> list[int]:
        """The EP buffer's status word {code, site, info, 0} (synchronises)."""
        out = (ctypes.c_int * 4)()
        _lib.check(_lib.load().parrot_ep_read_status(
            ctypes.byref(self.dims), ctypes.c_void_p(self.own.data_ptr()), out,
            bridge._stream()), "parrot_ep_read_status")
        return list(out)

    def received_rows(self) -> int:
        """Rows this rank received in its last call (reads the device; synchronises)."""
        lay = self.shape.layout()
        n = self.own[lay.back_n:lay.back_n + 4 * self.shape.ranks].view(torch.int32)
        return int(n.sum().item())

    def close(self) -> None:
        lib = _lib.load()
        for base in self._mapped:
            lib.parrot_ipc_close(ctypes.c_void_p(base))
        self._mapped = []


class PeerExpertParallelMoE:
    """One MoE layer expert-parallel over the ranks of ``peers``, exchanged
    through peer memory.  ``__call__`` enqueues the whole layer on the current
    stream with no host synchronisation; every rank must call it the same
    number of times (with zero tokens if it has none).  The three phases are
    also callable on their own (``send``, ``experts``, ``finish``) so that
    ranks sharing one GPU can run one after another in tests.

    ``fused`` (default ``FUSED_EXCHANGE``): the grouping kernel and the down
    GEMM store the rows into the peers' regions themselves; otherwise
    separate send and return copy kernels move them.  Both leave the same
    bytes in every region, so ranks may differ in this setting.

    ``overlap_shared`` (default ``OVERLAP_SHARED``): the shared expert, which
    needs only the layer input, runs on a side stream forked when the layer
    starts and joined before the combine, so it overlaps the dispatch and the
    exchange instead of following them; otherwise it runs on the layer's
    stream between the send and the receive.  Both capture in a CUDA graph."""

    def __init__(self, module, peers: PeerSet, fused: bool | None = None,
                 overlap_shared: bool | None = None):
        cfg = module.cfg
        shape = peers.shape
        if (shape.dim, shape.n_experts, shape.expert_dim) != (cfg.dim, cfg.n_experts,
                                                             cfg.expert_dim):
            raise ValueError("EP shape does not match the MoE module's dims")
        self.peers = peers
        self.ops = B200EpOps(module, peers.rank, shape.ranks, shape.slots(peers.rank))
        self.cfg = cfg
        self.fused = FUSED_EXCHANGE if fused is None else bool(fused)
        self.overlap_shared = OVERLAP_SHARED if overlap_shared is None else bool(overlap_shared)
        self._side: torch.cuda.Stream | None = None
        self._shared_on_side = False
        self._pending: tuple | None = None
        # (name, event) after each phase when a list is set (instrumentation only)
        self.marks: list | None = None

    def _mark(self, name: str) -> None:
        if self.marks is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.marks.append((name, ev))

    def send(self, x: Tensor) -> None:
        ops, peers = self.ops, self.peers
        bridge._require_device(x, "MoE")
        bridge._require_inference("MoE")
        x = x.contiguous()
        T = x.shape[0]
        if T > peers.shape.max_tokens:
            raise ValueError(f"{T} tokens, more than the EP set's max_tokens "
                             f"{peers.shape.max_tokens}")
        dims = bridge.moe_dims(self.cfg, T, capacity=-1)
        ws = ops._workspace(dims)
        w = bridge._weights_struct(ops.packed, ops.bias)
        lib, stream = _lib.load(), bridge._stream()
        outputs = _lib.MoeOutputs(None, None, None, None, None, None, None, None)
        self._shared_on_side = self.overlap_shared
        if self.overlap_shared:
            # the shared expert writes only its own workspace regions (its
            # hidden rows and output), disjoint from what the router, the
            # grouping and the exchange touch
            main = torch.cuda.current_stream()
            if self._side is None:
                self._side = torch.cuda.Stream(device=x.device)
            self._side.wait_stream(main)
            with torch.cuda.stream(self._side):
                self._shared(x, dims, ws, w)
            x.record_stream(self._side)
        if self.fused:
            _lib.check(lib.parrot_moe_ep_dispatch_send_bf16(
                ctypes.byref(dims), ctypes.byref(w), bridge._p(x), ctypes.byref(outputs),
                ctypes.byref(peers.dims), ctypes.byref(peers.peers), bridge._p(ws), ws.numel(),
                stream), "parrot_moe_ep_dispatch_send_bf16")
            self._mark("dispatch")
            self._mark("send")
            self._pending = (x, dims, ws, w)
            return
        _lib.check(lib.parrot_moe_ep_dispatch_planned_bf16(
            ctypes.byref(dims), ctypes.byref(w), bridge._p(x), ctypes.byref(outputs),
            ctypes.byref(peers.dims), bridge._p(ws), ws.numel(), stream),
            "parrot_moe_ep_dispatch_planned_bf16")
        self._mark("dispatch")
        _lib.check(lib.parrot_moe_ep_send_bf16(
            ctypes.byref(dims), ctypes.byref(peers.dims), ctypes.byref(peers.peers), bridge._p(ws),
            ws.numel(), stream), "parrot_moe_ep_send_bf16")
        self._mark("send")
        self._pending = (x, dims, ws, w)

    def experts(self) -> None:
        x, dims, ws, w = self._pending
        ops, peers = self.ops, self.peers
        lib, stream = _lib.load(), bridge._stream()
        own = ctypes.c_void_p(peers.own.data_ptr())
        if not self._shared_on_side:
            # the shared expert runs while the other ranks' rows arrive
            self._shared(x, dims, ws, w)
        self._mark("shared")
        _lib.check(lib.parrot_moe_ep_receive(ctypes.byref(peers.dims), own, stream),
                   "parrot_moe_ep_receive")
        self._mark("receive")
        if self.fused:
            _lib.check(lib.parrot_moe_ep_experts_return_bf16(
                ctypes.byref(peers.dims), ctypes.byref(peers.peers), bridge._p(ops.gate_up),
                bridge._p(ops.down), stream), "parrot_moe_ep_experts_return_bf16")
            self._mark("experts")
            self._mark("return")
            return
        _lib.check(lib.parrot_moe_ep_experts_bf16(
            ctypes.byref(peers.dims), own, bridge._p(ops.gate_up), bridge._p(ops.down), stream),
            "parrot_moe_ep_experts_bf16")
        self._mark("experts")
        _lib.check(lib.parrot_moe_ep_return_bf16(ctypes.byref(peers.dims),
                                                 ctypes.byref(peers.peers), stream),
                   "parrot_moe_ep_return_bf16")
        self._mark("return")

    def _shared(self, x: Tensor, dims, ws: Tensor, w) -> None:
        _lib.check(_lib.load().parrot_moe_shared_ffn_bf16(
            ctypes.byref(dims), ctypes.byref(w), bridge._p(x), bridge._p(ws), ws.numel(),
            bridge._stream()), "parrot_moe_shared_ffn_bf16")

    def finish(self, residual: Tensor | None = None) -> Tensor:
        x, dims, ws, _ = self._pending
        self._pending = None
        if self._shared_on_side:
            torch.cuda.current_stream().wait_stream(self._side)  # the shared output is ready
            self._shared_on_side = False
        out = torch.empty_like(x)
        if residual is not None:
            residual = residual.reshape(out.shape).contiguous()
        _lib.check(_lib.load().parrot_moe_ep_combine_peer_bf16(
            ctypes.byref(dims), ctypes.byref(self.peers.dims),
            ctypes.c_void_p(self.peers.own.data_ptr()), bridge._p(ws), ws.numel(),
            bridge._p(residual), bridge._p(out), bridge._stream()),
            "parrot_moe_ep_combine_peer_bf16")
        self._mark("combine")
        return out

    def __call__(self, x: Tensor, residual: Tensor | None = None) -> Tensor:
        self._mark("start")
        self.send(x)
        self.experts()
        return self.finish(residual)
