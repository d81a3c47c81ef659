"""Test-side pieces for the expert-parallel MoE: the oracle's arithmetic behind
the ``EpOps`` interface (CPU ranks over gloo), and an in-process communicator
that lets several ranks share one GPU as threads."""
from __future__ import annotations

import threading

import torch
import torch.nn.functional as F

from oracle import parrot_oracle as po
from parrot_b200 import ep


class OracleEpOps:
    """One rank's local compute restated from the oracle (``model.py:521-551``).

    ``dispatch`` packs the assignments destination-major exactly as the
    kernels do; ``combine`` adds the weighted expert outputs to the shared
    output in ascending expert id, rows ascending, as the oracle's loop does.
    """

    def __init__(self, moe: po.MoE, rank: int, ranks: int):
        self.moe = moe
        self.ranks = ranks
        self.local = ep.local_experts(rank, ranks, moe.cfg.n_experts)

    def dispatch(self, x):
        E, G = self.moe.cfg.n_experts, self.ranks
        logits = F.linear(x.float(), self.moe.router.weight.float())
        if self.moe.router_bias is not None:
            logits = logits + self.moe.router_bias.float()
        probs = logits.softmax(-1)
        w, idx = probs.topk(2, dim=-1)
        self.w = w / w.sum(-1, keepdim=True)
        self.idx = idx
        self.x = x
        T = x.shape[0]
        self.positions = torch.full((2 * T,), -1, dtype=torch.int64)
        order = []
        for r in range(G):
            for j in range(E // G):
                tok, lane = torch.where(idx == r + j * G)
                order.append(2 * tok + lane)
        order = torch.cat(order) if order else torch.zeros(0, dtype=torch.int64)
        self.positions[order] = torch.arange(order.numel())
        rows = x[order // 2]
        counts = torch.bincount(idx.flatten(), minlength=E).to(torch.int32)
        return rows, counts

    def shared(self, x):
        self.shared_y = self.moe.shared(x)

    def experts(self, rows, seg: ep.Segments):
        y = torch.empty_like(rows)
        for n, b, j in zip(seg.rows, seg.base, seg.expert):
            if n:
                y[b:b + n] = self.moe.experts[self.local[j]](rows[b:b + n])
        return y

    def combine(self, y, residual):
        out = self.shared_y
        for e in range(self.moe.cfg.n_experts):
            tok, lane = torch.where(self.idx == e)
            if tok.numel():
                rows = y[self.positions[2 * tok + lane]]
                out = out.index_add(0, tok, rows * self.w[tok, lane, None].to(out.dtype))
        return out if residual is None else residual + out


class ThreadGroup:
    """Shared state of ranks that run as threads of one process."""

    def __init__(self, size: int):
        self.size = size
        self.barrier = threading.Barrier(size, timeout=120)
        self.slots = [None] * size


class ThreadComm:
    """``ep.Comm`` for ranks that are threads (the exchange is a local copy)."""

    def __init__(self, group: ThreadGroup, rank: int):
        self.group = group
        self.rank = rank
        self.size = group.size

    def all_to_all(self, out, inp, out_splits, in_splits, async_op=False):
        G = self.size
        if in_splits is None:
            in_splits = [inp.shape[0] // G] * G
        self.group.slots[self.rank] = list(inp.split(in_splits))
        self.group.barrier.wait()
        pieces = [self.group.slots[src][self.rank] for src in range(G)]
        if out.numel():
            torch.cat(pieces, out=out)
        self.group.barrier.wait()
        return None


def run_threads(group: ThreadGroup, fn):
    """Run ``fn(rank)`` on one thread per rank; re-raise the first failure."""
    size = group.size
    results, errors = [None] * size, []

    def body(r):
        try:
            results[r] = fn(r)
        except BaseException as exc:  # noqa: BLE001 - reported below
            errors.append(exc)
            group.barrier.abort()  # release ranks waiting in an exchange

    threads = [threading.Thread(target=body, args=(r,)) for r in range(size)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(300)
    if errors:
        raise errors[0]
    return results
