"""Expert-parallel MoE orchestration on CPU ranks (gloo), with the oracle's
arithmetic as each rank's local compute: the exchange logic (placement,
count and row all-to-alls, segment tables, return order, combine) must give
every rank the oracle MoE layer's output on its own tokens."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import parrot_oracle as po
from parrot_b200 import ep
from parrot_b200.workloads import make_hidden_states, make_moe_layer_weights
from tests.ep_support import OracleEpOps, ThreadComm, ThreadGroup, run_threads

DIM, EXPERTS, HIDDEN, SHARED = 128, 8, 128, 64


def oracle_moe(seed: int, skew: bool) -> po.MoE:
    cfg = po.OracleConfig(dim=DIM, n_experts=EXPERTS, expert_dim=HIDDEN, shared_expert_dim=SHARED)
    moe = po.MoE(cfg)
    moe.load_state_dict(make_moe_layer_weights(DIM, EXPERTS, HIDDEN, SHARED, seed=seed))
    if skew:  # most tokens pick experts 0 and 1: some ranks receive far more rows
        moe.router_bias = torch.tensor([3.0, 2.5] + [0.0] * (EXPERTS - 2))
    return moe.eval()


def token_splits(total: int, ranks: int) -> list[int]:
    # ragged on purpose; with more ranks some hold no tokens at all
    gen = torch.Generator().manual_seed(ranks)
    inner = sorted(int(v) for v in torch.randint(0, total + 1, (ranks - 1,), generator=gen))
    cuts = [0] + inner + [total]
    sizes = [b - a for a, b in zip(cuts, cuts[1:])]
    if ranks >= 4:  # the last rank sends nothing and still receives rows
        sizes[-2] += sizes[-1]
        sizes[-1] = 0
    return sizes


def check_rank(rank: int, ranks: int, comm, skew: bool, total: int = 96):
    moe = oracle_moe(seed=3, skew=skew)
    x_all = make_hidden_states(total, DIM, seed=5)
    sizes = token_splits(total, ranks)
    start = sum(sizes[:rank])
    x = x_all[start:start + sizes[rank]]
    residual = torch.randn(x.shape, generator=torch.Generator().manual_seed(rank))
    layer = ep.ExpertParallelMoE(OracleEpOps(moe, rank, ranks), comm, EXPERTS)
    with torch.no_grad():
        got = layer(x, residual)
        want = residual + moe(x)[0]
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
    return layer.last_recv_rows


def _gloo_rank(rank, ranks, port, skew):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ranks)
    try:
        check_rank(rank, ranks, ep.TorchComm(), skew)
    finally:
        dist.destroy_process_group()


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("ranks,skew", [(2, False), (2, True), (4, True)])
def test_expert_parallel_over_gloo_matches_oracle(ranks, skew):
    mp.spawn(_gloo_rank, args=(ranks, free_port(), skew), nprocs=ranks, join=True)


@pytest.mark.parametrize("ranks", [1, 2, 8])
def test_expert_parallel_in_threads_matches_oracle(ranks):
    group = ThreadGroup(ranks)
    received = run_threads(group, lambda r: check_rank(r, ranks, ThreadComm(group, r), True))
    assert sum(received) == 2 * 96  # every assignment is computed exactly once


def test_placement_and_segment_tables():
    assert ep.local_experts(1, 4, 16) == [1, 5, 9, 13]
    assert all(ep.owner(e, 4) == 1 for e in ep.local_experts(1, 4, 16))
    counts = torch.arange(16, dtype=torch.int32)
    tab = ep.send_counts(counts, 4)
    assert tab.tolist()[2] == [2, 6, 10, 14]  # rows bound for rank 2, by local expert
    seg = ep.receive_segments([[3, 0], [1, 2]])
    assert (seg.rows, seg.base, seg.expert, seg.total) == ([3, 0, 1, 2], [0, 3, 3, 4], [0, 1, 0, 1], 6)
    with pytest.raises(ValueError):
        ep.local_experts(0, 3, 16)


ZIPF_COUNTS = [11965, 5210, 3213, 2265, 1733, 1423, 1143, 979, 847, 749, 694, 617, 553, 488,
               463, 426]  # the config-4 routing of 16384 tokens


def _busiest_share(p: ep.Placement, counts) -> float:
    """Largest share of the assignments one rank computes, rows of replicated
    experts split evenly over the sources."""
    total = sum(counts)
    load = [0.0] * p.ranks
    for e, n in enumerate(counts):
        if e in p.replicated:
            for q in range(p.ranks):
                load[q] += n / p.ranks
        else:
            load[p.dest(0, e)] += n
    return max(load) / total


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_balanced_placement_plans(ranks):
    p = ep.Placement.balanced(ZIPF_COUNTS, ranks)
    rr = ep.Placement.round_robin(ranks, 16)
    assert _busiest_share(p, ZIPF_COUNTS) <= _busiest_share(rr, ZIPF_COUNTS)
    if ranks >= 4:  # expert 0 (36.5% of the rows) is replicated, so no rank exceeds its share
        assert 0 in p.replicated
        assert _busiest_share(p, ZIPF_COUNTS) < 0.5 * _busiest_share(rr, ZIPF_COUNTS) + 0.1
    for source in range(ranks):
        plan = p.plan(source)
        sent = [e for row in plan for e in row if e >= 0]
        assert sorted(sent) == list(range(16))        # every expert once per source
        for e in p.replicated:
            assert plan[source][p.slots[source].index(e)] == e  # its own rows, computed locally
    assert rr.slots[-1] == tuple(ep.local_experts(ranks - 1, ranks, 16))


def test_placement_rejects_partial_replication():
    with pytest.raises(ValueError):
        ep.Placement(3, 4, ((0, 1), (0, 2), (3,)))   # expert 0 on two of three ranks
    with pytest.raises(ValueError):
        ep.Placement(2, 4, ((0, 1), (2,)))           # expert 3 nowhere


def test_ep_dims_carry_the_plan():
    p = ep.Placement.balanced(ZIPF_COUNTS, 4)
    shape = ep.EpShape(4, 64, 768, 16, 512, placement=p)
    d = shape.dims(2)
    assert d.slots == len(p.slots[2])
    for q in range(4):
        row = [d.plan[q][j] for j in range(32)]
        assert row[:len(p.slots[q])] == p.plan(2)[q]
        assert all(v == -1 for v in row[len(p.slots[q]):])
