"""Failure paths of the expert-parallel exchange, injected on the host (gloo
CPU ranks, the oracle's arithmetic as each rank's compute).

Each case runs one good step, then makes one rank misbehave between steps or
inside the next one: it leaves, it sends a row buffer shorter than its
counts promise, or it sends a count table whose total disagrees with its
counts.  Every rank must end with an exception — none may hang — well within
a bound set by the process group's short timeout.
"""
import datetime
import multiprocessing as mp_std
import os
import time

import pytest
import torch
import torch.distributed as dist

from parrot_b200 import ep
from parrot_b200.workloads import make_hidden_states
from tests.ep_support import OracleEpOps
from tests.test_ep_cpu import DIM, EXPERTS, free_port, oracle_moe

PG_TIMEOUT_S = 4
BOUND_S = 60  # every rank reports within this (process start, two steps, the timeout)


class FaultyComm:
    """``ep.TorchComm`` with one injected fault on ``rank``'s exchange number ``at``."""

    def __init__(self, comm, rank: int, fault: str, at: int):
        self.comm, self.rank, self.size = comm, comm.rank, comm.size
        self.fault, self.bad_rank, self.at = fault, rank, at
        self.calls = 0

    def all_to_all(self, out, inp, out_splits, in_splits, async_op=False):
        n = self.calls
        self.calls += 1
        if self.rank == self.bad_rank and n == self.at:
            if self.fault == "short_rows" and in_splits is not None:
                inp = inp[:max(0, inp.shape[0] - 1)]  # one row short of the splits
            elif self.fault == "bad_counts" and in_splits is None:
                inp = inp.clone()
                inp[0] += 1  # a count that its total does not include
        return self.comm.all_to_all(out, inp, out_splits, in_splits, async_op)


def _report(queue, item) -> None:
    queue.put(item)
    queue.close()
    queue.join_thread()  # flushed before the process exits


def _rank(rank, ranks, port, fault, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ranks,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    t0 = time.monotonic()
    outcome = "ok"
    try:
        moe = oracle_moe(seed=3, skew=False)
        x = make_hidden_states(64, DIM, seed=5 + rank)
        # exchanges per step: counts (0), rows (1), outputs (2); the fault is in step 2
        comm = FaultyComm(ep.TorchComm(), rank=1, fault=fault, at=3 + (1 if fault == "short_rows"
                                                                       else 0))
        layer = ep.ExpertParallelMoE(OracleEpOps(moe, rank, ranks), comm, EXPERTS,
                                     max_rows_per_source=2 * 64)
        with torch.no_grad():
            layer(x)
            if fault == "leaves" and rank == 1:
                _report(queue, (rank, "left", time.monotonic() - t0))
                os._exit(0)  # between steps, nothing in flight
            layer(x)
    except Exception as exc:  # noqa: BLE001 - reported to the test
        outcome = f"{type(exc).__name__}: {str(exc)[:160]}"
    _report(queue, (rank, outcome, time.monotonic() - t0))
    os._exit(0)  # skip process-group teardown: the peer may be gone


def _run(fault: str, ranks: int = 2) -> dict:
    ctx = mp_std.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, ranks, port, fault, queue)) for r in range(ranks)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.monotonic() + BOUND_S + 30
    while len(results) < ranks and time.monotonic() < deadline:
        try:
            r, outcome, dt = queue.get(timeout=1)
            results[r] = (outcome, dt)
        except Exception:  # noqa: BLE001 - queue.Empty: keep waiting until the deadline
            pass
    for p in procs:
        p.join(10)
        if p.is_alive():
            p.kill()
            p.join()
    return results


def test_a_rank_that_leaves_between_steps_fails_the_others():
    res = _run("leaves")
    assert res[1][0] == "left"
    outcome, dt = res[0]
    assert outcome != "ok" and outcome.split(":")[0] in ("RuntimeError", "DistBackendError"), res
    assert dt < BOUND_S, res


def test_a_row_buffer_shorter_than_its_counts_fails_every_rank():
    res = _run("short_rows")
    assert set(res) == {0, 1}, res
    for r, (outcome, dt) in res.items():
        assert outcome != "ok", res
        assert dt < BOUND_S, res


def test_an_inconsistent_count_table_is_rejected():
    res = _run("bad_counts")
    assert set(res) == {0, 1}, res
    assert res[0][0].startswith("ExchangeError"), res  # the receiver of the bad table
    assert "inconsistent count table from rank 1" in res[0][0]
    assert res[1][0] != "ok", res  # its peer then fails in the row exchange
    assert max(dt for _, dt in res.values()) < BOUND_S, res


def test_count_table_checks():
    good = torch.tensor([[3, 1, 4], [0, 0, 0]], dtype=torch.int32)
    ep.check_count_table(good, 0, max_rows=4)
    with pytest.raises(ep.ExchangeError, match="from rank 1"):
        ep.check_count_table(torch.tensor([[3, 1, 4], [1, 0, 0]], dtype=torch.int32), 0, None)
    with pytest.raises(ep.ExchangeError, match="from rank 0"):
        ep.check_count_table(torch.tensor([[3, 1, 4], [0, 0, 0]], dtype=torch.int32), 0, 3)
    with pytest.raises(ep.ExchangeError):
        ep.check_count_table(torch.tensor([[-1, 1, 0]], dtype=torch.int32), 0, None)
