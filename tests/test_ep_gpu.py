"""Expert-parallel MoE on the GPU, through the C ABI.

Ranks that share one GPU run as threads (the exchange is a device copy);
with two or more GPUs one NCCL process per GPU runs the same orchestration.
Each rank's output must equal the single-device MoE block on that rank's
tokens bit for bit, and the packed grouping mode must equal the capacity
layout bit for bit.
"""
import ctypes
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from parrot_b200 import _lib, bridge, ep
from parrot_b200.workloads import tune_zipf_router_bias
from tests.ep_support import ThreadComm, ThreadGroup, run_threads
from tests.gpu_helpers import build_moe_pair, hidden_states, moe_config

pytestmark = pytest.mark.gpu


def zipf_module(seed: int, tokens: int):
    cfg = moe_config()
    module, oracle = build_moe_pair(cfg, seed=seed)
    x = hidden_states(tokens, cfg.dim, seed=seed + 100)
    bias = tune_zipf_router_bias(x.float(), oracle.router.weight)
    module.router_bias = bias.cuda()
    return module, x.cuda()


def shard_sizes(total: int, ranks: int) -> list[int]:
    gen = torch.Generator().manual_seed(total + ranks)
    inner = sorted(int(v) for v in torch.randint(0, total + 1, (ranks - 1,), generator=gen))
    cuts = [0] + inner + [total]
    sizes = [b - a for a, b in zip(cuts, cuts[1:])]
    if ranks >= 4:
        sizes[-2] += sizes[-1]
        sizes[-1] = 0
    return sizes


def _forward_packed(module, x, capacity):
    cfg = module.cfg
    dims = bridge.moe_dims(cfg, x.shape[0], capacity=capacity)
    lay = bridge.workspace_layout(dims)
    ws = torch.zeros(int(lay.total), device="cuda", dtype=torch.uint8)
    out = torch.empty_like(x)
    outputs = _lib.MoeOutputs(out.data_ptr(), None, None, None, None, None, None, None)
    w = bridge._weights_struct(bridge.pack_weights(module), bridge._router_bias(module))
    _lib.check(_lib.load().parrot_moe_forward_bf16(
        ctypes.byref(dims), ctypes.byref(w), bridge._p(x), ctypes.byref(outputs), bridge._p(ws),
        ws.numel(), bridge._stream()), "parrot_moe_forward_bf16")
    status = (ctypes.c_int * 4)()
    _lib.check(_lib.load().parrot_moe_read_status(bridge._p(ws), ctypes.byref(dims), status,
                                                  bridge._stream()), "read status")
    assert list(status) == [0, 0, 0, 0]
    return out


@pytest.mark.parametrize("tokens,zipf", [(512, False), (2048, True), (37, False)])
def test_packed_grouping_equals_capacity_layout(tokens, zipf):
    with torch.inference_mode():
        if zipf:
            module, x = zipf_module(seed=8, tokens=tokens)
        else:
            cfg = moe_config()
            module, _ = build_moe_pair(cfg, seed=8)
            x = hidden_states(tokens, cfg.dim, seed=9).cuda()
        want = _forward_packed(module, x, 0)
        got = _forward_packed(module, x, -1)
        torch.cuda.synchronize()
        assert torch.equal(got, want)


def _ep_threads(module, x, ranks, residual):
    sizes = shard_sizes(x.shape[0], ranks)
    starts = [sum(sizes[:r]) for r in range(ranks)]
    group = ThreadGroup(ranks)
    ops = [ep.B200EpOps(module, r, ranks) for r in range(ranks)]

    def rank_fn(r):
        xs = x[starts[r]:starts[r] + sizes[r]]
        rs = residual[starts[r]:starts[r] + sizes[r]]
        layer = ep.ExpertParallelMoE(ops[r], ThreadComm(group, r), module.cfg.n_experts)
        with torch.inference_mode():
            return layer(xs, rs), layer.last_recv_rows

    results = run_threads(group, rank_fn)
    torch.cuda.synchronize()
    return sizes, starts, results


@pytest.mark.parametrize("ranks,zipf", [(2, False), (4, True), (8, True), (16, False)])
def test_expert_parallel_threads_equal_single_device_block(ranks, zipf):
    tokens = 3000
    with torch.inference_mode():
        if zipf:
            module, x = zipf_module(seed=12, tokens=tokens)
        else:
            cfg = moe_config()
            module, _ = build_moe_pair(cfg, seed=12)
            x = hidden_states(tokens, cfg.dim, seed=13).cuda()
        residual = hidden_states(tokens, module.cfg.dim, seed=14).cuda()
        sizes, starts, results = _ep_threads(module, x, ranks, residual)
        assert sum(n for _, n in results) == 2 * tokens
        for r in range(ranks):
            xs = x[starts[r]:starts[r] + sizes[r]]
            if sizes[r] == 0:
                assert results[r][0].shape[0] == 0
                continue
            # router statistics on: the tensor-core path at every shard size
            want, _, _ = bridge.b200_moe(module, xs, True,
                                         residual[starts[r]:starts[r] + sizes[r]])
            torch.cuda.synchronize()
            assert torch.equal(results[r][0], want), f"rank {r}"


def _nccl_rank(rank, ranks, port, seed, tokens):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=ranks,
                            device_id=torch.device("cuda", rank))
    try:
        with torch.inference_mode():
            module, x = zipf_module(seed=seed, tokens=tokens)
            sizes = shard_sizes(tokens, ranks)
            start = sum(sizes[:rank])
            xs = x[start:start + sizes[rank]]
            layer = ep.ExpertParallelMoE(ep.B200EpOps(module, rank, ranks), ep.TorchComm(),
                                         module.cfg.n_experts)
            got = layer(xs)
            want, _, _ = bridge.b200_moe(module, xs, True) if sizes[rank] else (got, 0, 0)
            torch.cuda.synchronize()
            assert torch.equal(got, want), f"rank {rank}"
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_expert_parallel_over_nccl_equals_single_device_block():
    ranks = min(torch.cuda.device_count(), 8)
    mp.spawn(_nccl_rank, args=(ranks, _free_port(), 21, 4096), nprocs=ranks, join=True)


# ---- the peer-memory exchange -------------------------------------------------

def _fused(exchange: str, rank: int) -> bool:
    """The row exchange a rank uses: the grouping kernel and the down GEMM
    store into the peers' regions and the shared expert runs on a side stream
    ("fused"), separate copy kernels move the rows and the shared expert runs
    in line ("copies"), or the ranks alternate ("mixed": even ranks fused)."""
    return exchange == "fused" or (exchange == "mixed" and rank % 2 == 0)


def _layer(module, peers, exchange, rank):
    on = _fused(exchange, rank)
    return ep.PeerExpertParallelMoE(module, peers, fused=on, overlap_shared=on)


def _peer_layers(module, sizes, wait_ns=200_000_000, placement=None, exchange="fused"):
    cfg = module.cfg
    shape = ep.EpShape(len(sizes), max(1, max(sizes)), cfg.dim, cfg.n_experts, cfg.expert_dim,
                       wait_ns, placement)
    peers = ep.PeerSet.local(shape, torch.device("cuda"))
    return peers, [_layer(module, p, exchange, r) for r, p in enumerate(peers)]


def _balanced(module, x, ranks):
    """Load-balanced placement from this batch's routing counts."""
    _, _, util = bridge.b200_moe(module, x, True)
    counts = (util.float() * 2 * x.shape[0]).round().int().tolist()
    return ep.Placement.balanced(counts, ranks)


_IN_TURN = [(1, False, "rr"), (2, False, "rr"), (4, True, "rr"), (8, True, "rr"),
            (2, True, "balanced"), (4, True, "balanced"), (8, True, "balanced")]


@pytest.mark.parametrize("ranks,zipf,placement,exchange",
                         [c + (x,) for x in ("fused", "copies") for c in _IN_TURN] +
                         [(2, True, "balanced", "mixed"), (4, False, "rr", "mixed")])
def test_peer_exchange_ranks_in_turn_equal_single_device_block(ranks, zipf, placement, exchange):
    """All ranks' buffers on one GPU, the ranks' phases issued in turn on one
    stream: every send before any receive, every return before any combine, so
    each flag a kernel waits for was raised by a kernel that already finished.
    Two calls in a row (the epoch advances, the regions are reused).  Round-
    robin placement, and load-balanced placements whose hot experts are
    replicated (each source computes its own rows of them).  The rows move
    by the grouping kernel and the down GEMM themselves, by the copy kernels,
    or by both (ranks alternating)."""
    tokens = 3000
    with torch.inference_mode():
        if zipf:
            module, x = zipf_module(seed=12, tokens=tokens)
        else:
            cfg = moe_config()
            module, _ = build_moe_pair(cfg, seed=12)
            x = hidden_states(tokens, cfg.dim, seed=13).cuda()
        residual = hidden_states(tokens, module.cfg.dim, seed=14).cuda()
        sizes = shard_sizes(tokens, ranks)
        starts = [sum(sizes[:r]) for r in range(ranks)]
        plan = _balanced(module, x, ranks) if placement == "balanced" else None
        if plan is not None and ranks >= 4:
            assert plan.replicated  # the Zipf head is computed where its rows are
        peers, layers = _peer_layers(module, sizes, placement=plan, exchange=exchange)
        for call in range(2):
            xs = [x[starts[r]:starts[r] + sizes[r]] * (1 + call) for r in range(ranks)]
            rs = [residual[starts[r]:starts[r] + sizes[r]] for r in range(ranks)]
            for r in range(ranks):
                layers[r].send(xs[r])
            for r in range(ranks):
                layers[r].experts()
            outs = [layers[r].finish(rs[r]) for r in range(ranks)]
            torch.cuda.synchronize()
            for r in range(ranks):
                assert peers[r].status() == [0, 0, 0, 0], f"rank {r}"
                if sizes[r] == 0:
                    assert outs[r].shape[0] == 0
                    continue
                want, _, _ = bridge.b200_moe(module, xs[r], True, rs[r])
                torch.cuda.synchronize()
                assert torch.equal(outs[r], want), f"call {call}, rank {r}"


@pytest.mark.parametrize("exchange", ["fused", "copies"])
def test_peer_exchange_single_rank_captured_in_a_graph(exchange):
    """A one-rank set runs the whole layer on one GPU (its own flags are
    raised earlier on the same stream), so the layer can be captured in a
    CUDA graph here: with the shared expert forked onto a side stream and
    joined before the combine, and with it in line.  Replays with new inputs
    equal the single-device block."""
    tokens = 1500
    with torch.inference_mode():
        module, x = zipf_module(seed=41, tokens=tokens)
        residual = hidden_states(tokens, module.cfg.dim, seed=42).cuda()
        peers, (layer,) = _peer_layers(module, [tokens], exchange=exchange)
        static_x = x.clone()
        layer(static_x, residual)  # first call outside the capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            static_out = layer(static_x, residual)
        for scale in (1.0, 0.5, 2.0):
            static_x.copy_(x * scale)
            graph.replay()
            torch.cuda.synchronize()
            want, _, _ = bridge.b200_moe(module, static_x, True, residual)
            torch.cuda.synchronize()
            assert peers[0].status() == [0, 0, 0, 0]
            assert torch.equal(static_out, want), f"scale {scale}"
        del graph


def test_peer_exchange_wait_for_a_missing_rank_times_out_with_status():
    """A two-rank set whose second rank never runs: rank 0's wait for its rows
    (and later for its returned outputs) runs out after the short limit, the
    status word says so, and the device stays usable."""
    cfg = moe_config()
    with torch.inference_mode():
        module, _ = build_moe_pair(cfg, seed=3)
        x = hidden_states(64, cfg.dim, seed=4).cuda()
        peers, layers = _peer_layers(module, [64, 64], wait_ns=50_000_000)
        layers[0].send(x)
        layers[0].experts()
        layers[0].finish()
        torch.cuda.synchronize()
        code, site, info, _ = peers[0].status()
        assert (code, site, info) == (1, 21, 1)  # timeout, receive wait, source rank 1
        want, _, _ = bridge.b200_moe(module, x, True)
        torch.cuda.synchronize()
        assert torch.isfinite(want).all()


def _peer_rank(rank, ranks, port, seed, tokens, balanced, exchange):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=ranks,
                            device_id=torch.device("cuda", rank))
    peers = None
    try:
        with torch.inference_mode():
            module, x = zipf_module(seed=seed, tokens=tokens)
            residual = hidden_states(tokens, module.cfg.dim, seed=seed + 1).cuda()
            sizes = shard_sizes(tokens, ranks)
            start = sum(sizes[:rank])
            xs = x[start:start + sizes[rank]]
            rs = residual[start:start + sizes[rank]]
            cfg = module.cfg
            plan = _balanced(module, x, ranks) if balanced else None
            shape = ep.EpShape(ranks, max(sizes), cfg.dim, cfg.n_experts, cfg.expert_dim,
                               1_000_000_000, plan)
            peers = ep.PeerSet.connect(shape)
            layer = _layer(module, peers, exchange, rank)
            want = bridge.b200_moe(module, xs, True, rs)[0] if sizes[rank] else None
            for _ in range(3):
                got = layer(xs, rs)
            torch.cuda.synchronize()
            assert peers.status() == [0, 0, 0, 0], f"rank {rank}"
            if want is not None:
                assert torch.equal(got, want), f"rank {rank}"
            # the same layer captured once and replayed
            graph = torch.cuda.CUDAGraph()
            dist.barrier()
            with torch.cuda.graph(graph):
                static_out = layer(xs, rs)
            for _ in range(2):
                graph.replay()
            torch.cuda.synchronize()
            assert peers.status() == [0, 0, 0, 0], f"rank {rank} (graph)"
            if want is not None:
                assert torch.equal(static_out, want), f"rank {rank} (graph)"
            del graph
        dist.barrier()
    finally:
        if peers is not None:
            peers.close()
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
@pytest.mark.parametrize("balanced,exchange", [(False, "fused"), (True, "fused"),
                                               (False, "copies"), (True, "mixed")])
def test_peer_exchange_over_nvlink_equals_single_device_block(balanced, exchange):
    ranks = min(torch.cuda.device_count(), 8)
    mp.spawn(_peer_rank, args=(ranks, _free_port(), 31, 4096, balanced, exchange), nprocs=ranks,
             join=True)
