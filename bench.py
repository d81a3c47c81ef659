#!/usr/bin/env python
"""Parrot XL bf16 forward (1 x 512) on B200 — tokens/s, MoE-layer latency and roofline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

A step is one full ``Parrot.forward`` of the default Parrot XL model (random
init, seed 0) on one 1 x 512 batch of uniform token ids, including the full
[1, 512, 32768] logits.  ``value`` is device-timed with the ids resident in
HBM; ``e2e`` adds, every step, the pinned host->device copy of the ids and the
device->host copy of the logits.  For N > 1 (torchrun, one rank per GPU) every
rank runs its own replica on its own batch (weak scaling, no collective on the
data path); time is the max over ranks.  ``--impl reference`` times the CPU
restatement of the reference's ``moe_backend="pytorch"`` forward on the host
cores instead (rank 0 only).
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "parrot-h200-worker_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "Parrot XL bf16 prefill tokens/sec (1x512)"
UNIT = "tokens/s"
SEQ = 512
L2_BYTES = 126 * 1024 * 1024


def parse_args():
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("b200", "reference"), default="b200")
    p.add_argument("--skip-cpu-baseline", action="store_true")
    return p.parse_args()


def ncu_traffic(kernel: str) -> float | None:
    """Per-launch DRAM bytes of ``kernel`` from the committed ncu summary."""
    path = ROOT / "profiles" / "traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) == 2 and parts[0] == kernel:
            return float(parts[1])
    return None


def measured_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown",
              "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={','.join(self.FIELDS)}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "20"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, power, reasons = [], [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) != len(self.FIELDS):
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
                power.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[3:]):
                if flag.lower() in ("active", "1", "yes"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def cpu_reference_forward(steps: int, warmup: int) -> dict:
    """The reference's pytorch-backend forward, restated on the CPU (the oracle)."""
    from oracle import parrot_oracle as po
    from parrot_b200.workloads import random_token_ids
    cores = po.oracle_threads()
    torch.manual_seed(0)
    model = po.OracleParrot(po.OracleConfig()).eval()
    ids = random_token_ids(1, SEQ, 32768, seed=0)
    with torch.no_grad():
        for _ in range(warmup):
            model(ids)
        times = []
        for _ in range(steps):
            t0 = time.perf_counter()
            model(ids)
            times.append(time.perf_counter() - t0)
    total = sum(times)
    return {"value": SEQ * steps / total, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{steps} x Parrot XL fp32 forward 1x{SEQ} on the host CPU "
                      f"(torch {torch.__version__}, {cores} threads), seed-0 weights",
            "seconds_per_step": total / steps}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # a CPU forward takes ~0.2 s: the requested counts (bounded) keep the run short
    steps = max(1, min(args.steps, 100))
    warmup = max(1, min(args.warmup, 10))
    base = cpu_reference_forward(steps, warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": steps, "warmup": warmup,
        "ms_per_step": 1000 * base["seconds_per_step"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": "Parrot XL forward 1x512 (BASELINE config 3)",
                   "global_batch": 1, "seq_len": SEQ, "parallelism": "cpu",
                   "path": "reference moe_backend=pytorch restated (oracle), CPU"},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_moe_kernels(model, tokens: int, replays: int = 20) -> dict:
    """CUDA-event timing of the gate_up grouped GEMM and of the whole MoE block.

    Each is captured as one CUDA graph of 16 back-to-back launches that cycle
    through the model's 16 MoE layers, so every launch streams its own 26 MB
    of expert weights from HBM (16 x 26 MB > the 126 MB L2); the graph is
    replayed ``replays`` times between two events on the launching stream.
    """
    from parrot_b200 import _lib, bridge
    from parrot_b200.graphs import capture_calls
    lib = _lib.load()
    cfg = model.config
    layers = [b.moe for b in model.blocks]
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(tokens, cfg.dim, device="cuda", generator=g).to(torch.bfloat16)
    with torch.inference_mode():
        bridge.b200_route(layers[0], x, False)
        dims = bridge.moe_dims(cfg, tokens)
        ws = bridge.workspace(x.device, dims)
        structs = [bridge._weights_struct(bridge.pack_weights(m), None) for m in layers]

        def gemm_cycle():
            sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
            for w in structs:
                _lib.check(lib.parrot_moe_gemm_bf16(
                    ctypes.byref(dims), ctypes.byref(w), ctypes.c_void_p(x.data_ptr()),
                    ctypes.c_void_p(ws.data_ptr()), ws.numel(), 0, sp), "parrot_moe_gemm_bf16")

        def moe_cycle():
            for m in layers:
                bridge.b200_moe(m, x, False)

        out = {}
        for name, fn in (("gemm", gemm_cycle), ("moe", moe_cycle)):
            graph = capture_calls(fn)
            graph.replay()
            torch.cuda.synchronize()
            stream = torch.cuda.current_stream()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(replays):
                graph.replay()
            b.record(stream)
            torch.cuda.synchronize()
            out[f"{name}_ms"] = a.elapsed_time(b) / (replays * len(layers))
            del graph
    E, H, Hs, d = cfg.n_experts, cfg.expert_dim, cfg.shared_expert_dim, cfg.dim
    A = 2 * tokens
    out["gemm_bytes"] = 2 * (E * 2 * H * d + 2 * Hs * d + A * d + tokens * d + A * H + tokens * Hs)
    out["launches"] = replays * len(layers)
    return out


def time_moe_breakdown(model, tokens: int = 256, replays: int = 10) -> dict:
    """BASELINE config 2 kernel by kernel: one CUDA graph of 16 MoE blocks
    (cycling the model's 16 layers, so every launch streams its own weights
    from HBM) replayed under the torch profiler (CUPTI device timestamps, not
    ncu).  The block runs in slot mode: the router also groups the rows, so
    there is no grouping kernel.  Per kernel kind: mean device duration per block, the exposed part
    (not overlapped by the previous kernel's tail: launches are programmatic
    dependent launches), algorithmic bytes, and bytes / duration against the
    measured HBM bandwidth."""
    import collections

    from torch.profiler import ProfilerActivity, profile

    from parrot_b200 import bridge
    from parrot_b200.graphs import capture_calls
    cfg = model.config
    layers = [b.moe for b in model.blocks]
    g = torch.Generator(device="cuda").manual_seed(1)
    x = torch.randn(tokens, cfg.dim, device="cuda", generator=g).to(torch.bfloat16)
    with torch.inference_mode():
        for m in layers:
            bridge.b200_moe(m, x, False)
        graph = capture_calls(lambda: [bridge.b200_moe(m, x, False) for m in layers])
        graph.replay()
        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(replays):
                graph.replay()
            torch.cuda.synchronize()
        del graph
    evs = sorted((e.time_range.start, e.time_range.end, e.name) for e in prof.events()
                 if e.device_type == torch.autograd.DeviceType.CUDA)
    dur, exp = collections.defaultdict(float), collections.defaultdict(float)
    prev_end, gemms = evs[0][0], 0
    for start, end, name in evs:
        if "route_kernel" in name or "route_small_kernel" in name:
            kind, gemms = "route", 0  # each block starts at its router
        elif "group_kernel" in name:
            kind = "group"
        elif "grouped_gemm" in name:
            kind = "gate_up_swiglu" if gemms == 0 else "down"
            gemms += 1
        elif "combine_kernel" in name:
            kind = "combine"
        else:
            kind = "other"
        dur[kind] += end - start
        exp[kind] += max(0.0, end - max(start, prev_end))
        prev_end = max(prev_end, end)
    n = replays * len(layers)
    T, d, E, H, Hs = tokens, cfg.dim, cfg.n_experts, cfg.expert_dim, cfg.shared_expert_dim
    A = 2 * T
    # the router groups the rows itself (slot mode): its bytes include the
    # two grouped copies of every token row
    algo = {"route": 2 * T * d + 2 * E * d + 16 * T + 4 * T * d,
            "group": 2 * T * d + 4 * T * d,
            "gate_up_swiglu": 2 * (E * 2 * H * d + 2 * Hs * d + A * d + T * d + A * H + T * Hs),
            "down": 2 * (E * d * H + d * Hs + A * H + T * Hs + A * d + T * d),
            "combine": 2 * (A * d + T * d) + 2 * T * d}
    flops = {"gate_up_swiglu": 2 * (A * d * 2 * H + T * d * 2 * Hs),
             "down": 2 * (A * H * d + T * Hs * d)}
    peaks, _ = measured_peaks()
    out = {}
    for kind in ("route", "group", "gate_up_swiglu", "down", "combine", "other"):
        if kind not in dur:
            continue
        us = dur[kind] / n
        row = {"us": us, "exposed_us": exp[kind] / n}
        if kind in algo:
            gbs = algo[kind] / (us * 1e-6) / 1e9
            row.update(bytes=algo[kind], gbs=gbs, hbm_frac=gbs / float(peaks["hbm_gbs"]))
        if kind in flops:
            row["tflops"] = flops[kind] / (us * 1e-6) / 1e12
        out[kind] = row
    return {"tokens": tokens, "kernels": out,
            "block_exposed_us": sum(exp.values()) / n,
            "timing": "CUPTI device timestamps (torch profiler) over a graph of 16 blocks, "
                      f"{replays} replays; per block"}


def cpu_baselines() -> dict:
    """The oracle (the reference's pytorch path restated) on the host cores for
    BASELINE configs 2, 4 and 5, fp32 and bf16: median of 5 runs after a
    warm-up, except config 4 (one run each, as the plan allows) and config 5
    (16 decode steps after an untimed prefill)."""
    from oracle import parrot_oracle as po
    from parrot_b200.workloads import (make_hidden_states, make_moe_layer_weights,
                                       random_token_ids, tune_zipf_router_bias)
    cores = po.oracle_threads()
    cfg = po.OracleConfig()
    w = make_moe_layer_weights(cfg.dim, cfg.n_experts, cfg.expert_dim, cfg.shared_expert_dim, 1)
    out = {"cores": cores, "kind": "port"}

    def med(fn, runs):
        ts = []
        for _ in range(runs):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    with torch.no_grad():
        for dtype in (torch.float32, torch.bfloat16):
            name = "fp32" if dtype == torch.float32 else "bf16"
            moe = po.MoE(cfg)
            moe.load_state_dict(w)
            moe = moe.to(dtype).eval()
            x = make_hidden_states(256, cfg.dim, 0).to(dtype)
            moe(x)
            out[f"config2_moe_layer_T256_{name}_ms"] = 1000 * med(lambda: moe(x), 5)
            x4 = make_hidden_states(16384, cfg.dim, 0)
            moe.router_bias = tune_zipf_router_bias(x4, w["router.weight"])
            x4 = x4.to(dtype)
            out[f"config4_zipf_moe_layer_T16384_{name}_ms"] = 1000 * med(lambda: moe(x4), 1)
        torch.manual_seed(0)
        model = po.OracleParrot(cfg).eval()
        decode = {}
        for b in (1, 8, 64):
            ids = random_token_ids(b, 128, cfg.vocab_size, seed=b)
            logits, state = model.prefill(ids)
            nxt = logits.argmax(-1)
            t0 = time.perf_counter()
            for _ in range(16):
                logits, state = model.decode_step(nxt, state)
                nxt = logits.argmax(-1)
            decode[f"B{b}"] = 16 * b / (time.perf_counter() - t0)
            del state
        out["config5_decode_fp32_tokens_per_s"] = decode
        out["config5_decode_bf16"] = ("not run: the reference's absorbed MLA decode gives SDPA "
                                      "an fp32 query with a bf16 latent cache, which torch rejects")
    out["sample"] = (f"oracle on {cores} host threads (torch {torch.__version__}): config 2 "
                     "median of 5, config 4 one run, config 5 16 decode steps after prefill 128")
    return out


def time_zipf_layer(tokens: int = 16384, replays: int = 10) -> dict:
    """BASELINE config 4 on one GPU: one XL MoE layer, Zipf(1.2)-skewed routing
    (harness router bias), CUDA-graph replays of the whole block."""
    from parrot_b200 import ModelConfig, bridge
    from parrot_b200.graphs import capture_calls
    from parrot_b200.model import MoE
    from parrot_b200.workloads import (make_hidden_states, make_moe_layer_weights,
                                       tune_zipf_router_bias)
    cfg = ModelConfig()
    w = make_moe_layer_weights(cfg.dim, cfg.n_experts, cfg.expert_dim, cfg.shared_expert_dim, 1)
    moe = MoE(cfg)
    moe.load_state_dict(w)
    x = make_hidden_states(tokens, cfg.dim, 0)
    moe = moe.to("cuda", torch.bfloat16).eval()
    moe.router_bias = tune_zipf_router_bias(x, w["router.weight"]).to("cuda", torch.float32)
    xd = x.to("cuda", torch.bfloat16)
    with torch.inference_mode():
        _, _, util = bridge.b200_moe(moe, xd, True)
        graph = capture_calls(lambda: bridge.b200_moe(moe, xd, False))
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(replays):
            graph.replay()
        b.record()
        torch.cuda.synchronize()
    us = 1000 * a.elapsed_time(b) / replays
    flops = 2 * (2 * tokens * cfg.dim * 3 * cfg.expert_dim + tokens * cfg.dim * 3 *
                 cfg.shared_expert_dim + tokens * cfg.dim * cfg.n_experts)
    capacity = max(8, ((4 * tokens + cfg.n_experts - 1) // cfg.n_experts + 7) // 8 * 8)
    counts = (util.float() * 2 * tokens).round().int().tolist()
    return {"us": us, "tflops": flops / (us * 1e-6) / 1e12, "tokens": tokens,
            "expert_counts": counts, "capacity": capacity,
            "overflow_rows": sum(max(0, c - capacity) for c in counts)}


def time_decode(model, batches=(1, 8, 64), prompt: int = 128, new_tokens: int = 16) -> dict:
    """prefill 128 ids, then 16 greedy decode steps; tokens/s of
    the decode steps, eager (``decode_step``) and replayed from one captured step
    (``Parrot.capture_decode``), CUDA events around the 16 steps."""
    from parrot_b200.workloads import random_token_ids
    out = {"eager": {}, "graph": {}}
    with torch.inference_mode():
        for b in batches:
            ids = random_token_ids(b, prompt, model.config.vocab_size, seed=b).cuda()
            logits, state = model.prefill(ids)
            nxt = logits.argmax(-1)
            model.decode_step(nxt, state)  # warm the decode path once
            for mode in ("eager", "graph"):
                logits, state = model.prefill(ids)
                nxt = logits.argmax(-1)
                step = model.capture_decode(state, next_token_only=True) if mode == "graph" else None
                torch.cuda.synchronize()
                a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                for _ in range(new_tokens):
                    if step is None:
                        nxt, state = model.decode_next(nxt, state)
                    else:
                        nxt = step(nxt)
                e.record()
                torch.cuda.synchronize()
                out[mode][f"B{b}"] = b * new_tokens / (a.elapsed_time(e) * 1e-3)
    return out


def time_ep_layer(dist, rank: int, world: int, total: int = 16384, iters: int = 20,
                  warmup: int = 3) -> dict:
    """BASELINE config 4 expert-parallel: the Zipf-skewed XL MoE layer with its
    16384 tokens split evenly over the ranks.  The product path exchanges rows
    and outputs through the other ranks' memory (``ep.PeerExpertParallelMoE``,
    CUDA IPC over NVLink) with no host synchronisation; it is captured once as
    a CUDA graph and replayed, with a load-balanced placement (rows stored
    into the peers by the grouping kernel and the down GEMM, and, beside it,
    by separate copy kernels) and with round-robin placement.  Per-phase
    times come from CUDA events between the
    phases of one eager call; the NCCL all-to-all path with its host read of
    the split sizes (``ep.ExpertParallelMoE``, round-robin) is timed beside it.
    Every number is the max over ranks."""
    from parrot_b200 import ModelConfig, bridge, ep
    from parrot_b200.model import MoE
    from parrot_b200.workloads import (make_hidden_states, make_moe_layer_weights,
                                       tune_zipf_router_bias)
    cfg = ModelConfig()
    w = make_moe_layer_weights(cfg.dim, cfg.n_experts, cfg.expert_dim, cfg.shared_expert_dim, 1)
    moe = MoE(cfg)
    moe.load_state_dict(w)
    x = make_hidden_states(total, cfg.dim, 0)
    moe = moe.to("cuda", torch.bfloat16).eval()
    moe.router_bias = tune_zipf_router_bias(x, w["router.weight"]).to("cuda", torch.float32)
    per = total // world
    xs = x[rank * per:(rank + 1) * per].to("cuda", torch.bfloat16)
    stream = torch.cuda.current_stream()

    def timed(fn, n) -> float:
        dist.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        return 1000 * a.elapsed_time(b) / n

    def max_all(values: list[float]) -> list[float]:
        t = torch.tensor(values, device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    with torch.inference_mode():
        # routing counts of the whole batch (identical on every rank): the
        # load-balanced placement replicates the experts above 1 / world of them
        _, _, util = bridge.b200_moe(moe, x.to("cuda", torch.bfloat16), True)
        counts = (util.float() * 2 * total).round().int().tolist()
    balanced = ep.Placement.balanced(counts, world)
    # (placement, rows stored by the grouping kernel and the down GEMM
    # themselves or moved by separate copy kernels, shared expert on a side
    # stream or in line)
    variants = {"balanced": (balanced, True, True),
                "balanced_shared_in_line": (balanced, True, False),
                "balanced_copy_kernels": (balanced, False, False),
                "round_robin": (ep.Placement.round_robin(world, cfg.n_experts), True, True)}
    res = {}
    for name, (placement, fused, overlap) in variants.items():
        shape = ep.EpShape(world, per, cfg.dim, cfg.n_experts, cfg.expert_dim,
                           placement=placement)
        peers = ep.PeerSet.connect(shape)
        with torch.inference_mode():
            layer = ep.PeerExpertParallelMoE(moe, peers, fused=fused, overlap_shared=overlap)
            for _ in range(warmup):
                layer(xs)
            eager_us = timed(lambda: layer(xs), iters)
            # one eager call with an event after every phase; the GPU first
            # spins (~1 ms) while the host enqueues the whole layer, so the
            # events time device work, not launch gaps
            dist.barrier()
            torch.cuda.synchronize()
            layer.marks = []
            torch.cuda._sleep(2_000_000)
            layer(xs)
            torch.cuda.synchronize()
            marks, layer.marks = layer.marks, None
            names = [n for n, _ in marks[1:]]
            phase = [1000 * marks[i][1].elapsed_time(marks[i + 1][1])
                     for i in range(len(marks) - 1)]
            received = peers.received_rows()
            graph = torch.cuda.CUDAGraph()
            dist.barrier()
            with torch.cuda.graph(graph):
                layer(xs)
            for _ in range(warmup):
                graph.replay()
            graph_us = timed(graph.replay, iters)
            status = peers.status()
            del graph
        dist.barrier()
        peers.close()
        graph_us, eager_us, *phase = max_all([graph_us, eager_us] + phase)
        recv = torch.tensor([received, status[0]], device="cuda", dtype=torch.int64)
        recv_all = [torch.zeros_like(recv) for _ in range(world)]
        dist.all_gather(recv_all, recv)
        if any(int(r[1].item()) for r in recv_all):
            raise RuntimeError(f"expert-parallel status word set on some rank: {status}")
        res[name] = {"us": graph_us, "eager_us": eager_us, "phase_us": dict(zip(names, phase)),
                     "received_rows_per_rank": [int(r[0].item()) for r in recv_all],
                     "slots": [list(q) for q in placement.slots],
                     "replicated": sorted(placement.replicated)}
    with torch.inference_mode():
        nccl = ep.ExpertParallelMoE(ep.B200EpOps(moe, rank, world), ep.TorchComm(),
                                    cfg.n_experts)
        for _ in range(warmup):
            nccl(xs)
        nccl_us = max_all([timed(lambda: nccl(xs), iters)])[0]
    flops = 2 * (2 * total * cfg.dim * 3 * cfg.expert_dim + total * cfg.dim * 3 *
                 cfg.shared_expert_dim + total * cfg.dim * cfg.n_experts)
    best = res["balanced"]
    return {"us": best["us"], "tokens_total": per * world,
            "tokens_per_s": per * world / (best["us"] * 1e-6),
            "tflops_all_ranks": flops / (best["us"] * 1e-6) / 1e12,
            "ranks": world,
            "placement": "load-balanced from the batch's routing counts: experts above 1/ranks "
                         "of the rows replicated (each source computes its own rows of them), "
                         "the rest largest first onto the least-loaded rank",
            "exchange": "peer memory (CUDA IPC over NVLink): the grouping kernel stores each "
                        "row into its destination's receive region and the down GEMM each "
                        "output into its source's return region; epoch flags, no host read; "
                        "the shared expert on a side stream beside them "
                        "(balanced_shared_in_line: the shared expert after the send; "
                        "balanced_copy_kernels: that and separate send / return copy kernels)",
            "balanced": best, "balanced_shared_in_line": res["balanced_shared_in_line"],
            "balanced_copy_kernels": res["balanced_copy_kernels"],
            "round_robin": res["round_robin"],
            "nccl_all_to_all_host_read_us": nccl_us,
            "timing": "CUDA-graph replay of the whole layer, CUDA events, max over ranks; "
                      "phase_us: one eager call behind a GPU sleep, events between phases, "
                      "max over ranks per phase"}


def run_b200(args):
    from parrot_b200 import ModelConfig, Parrot, _lib
    from parrot_b200 import build as pbuild
    from parrot_b200.workloads import random_token_ids

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    pbuild.build()
    lib = _lib.load()
    if not lib.parrot_b200_device_supported(local):
        raise RuntimeError("bench.py needs an sm_100 GPU")

    cfg = ModelConfig()
    torch.manual_seed(0)
    model = Parrot(cfg).to("cuda", torch.bfloat16).eval()
    ids_host = random_token_ids(1, SEQ, cfg.vocab_size, seed=rank).pin_memory()
    ids = ids_host.cuda()
    stream = torch.cuda.current_stream()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    with torch.inference_mode():
        # eager forward: warm-up, launch count per forward, eager time (context only)
        model(ids)
        l0 = lib.parrot_b200_launch_count()
        model(ids)
        launches_per_forward = lib.parrot_b200_launch_count() - l0
        barrier()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        q0.record(stream)
        for _ in range(3):
            model(ids)
        q1.record(stream)
        torch.cuda.synchronize()
        eager_ms = q0.elapsed_time(q1) / 3

        graphed = model.capture(1, SEQ)
        graphed(ids)
        for _ in range(max(3, args.warmup)):
            graphed.graph.replay()
        barrier()
        sampler = ClockSampler(local)
        sampler.start()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            graphed.graph.replay()
        end.record(stream)
        barrier()
        ms = start.elapsed_time(end)

        # end to end through the public call: every step copies its ids in from
        # pinned host memory, replays the forward and copies its full logits out.
        # Two captured graphs alternate so that step i's logits travel to the
        # host (copy stream) while step i + 1 computes, and step i + 1's ids are
        # staged (their own stream) while step i computes: a small host-to-
        # device copy issued behind a 33.5 MB device-to-host copy waited
        # ~110 us for it.
        graphs = [graphed, model.capture(1, SEQ)]
        out = graphed.output
        logits_host = [torch.empty(out.logits.shape, dtype=out.logits.dtype, pin_memory=True)
                       for _ in graphs]
        copy_stream, h2d_stream = torch.cuda.Stream(), torch.cuda.Stream()
        computed = [torch.cuda.Event() for _ in graphs]
        copied = [torch.cuda.Event() for _ in graphs]
        staged = [torch.cuda.Event() for _ in graphs]
        for g in graphs:  # warm both graphs and both copy paths
            g(ids_host)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h2d_stream.wait_event(e0)
        with torch.cuda.stream(h2d_stream):
            graphs[0].stage(ids_host)
            staged[0].record(h2d_stream)
        for i in range(args.steps):
            j = i % 2
            if i + 1 < args.steps:
                k = (i + 1) % 2
                if i >= 1:
                    h2d_stream.wait_event(computed[k])  # step i - 1 has read its ids
                with torch.cuda.stream(h2d_stream):
                    graphs[k].stage(ids_host)
                    staged[k].record(h2d_stream)
            stream.wait_event(staged[j])
            if i >= 2:
                stream.wait_event(copied[j])  # this graph's previous logits are out
            o = graphs[j].replay()
            computed[j].record(stream)
            copy_stream.wait_event(computed[j])
            with torch.cuda.stream(copy_stream):
                logits_host[j].copy_(o.logits, non_blocking=True)
                copied[j].record(copy_stream)
        stream.wait_stream(copy_stream)
        e1.record(stream)
        barrier()
        clocks = sampler.stop()
        e2e_ms = e0.elapsed_time(e1)
        launches = launches_per_forward * args.steps

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_over_ranks(ms)
    e2e_ms = max_over_ranks(e2e_ms)
    kern = time_moe_kernels(model, SEQ) if rank == 0 else None
    kern256 = time_moe_kernels(model, 256) if rank == 0 else None
    breakdown = time_moe_breakdown(model, 256) if rank == 0 else None
    decode = time_decode(model) if rank == 0 else None
    zipf = time_zipf_layer() if rank == 0 else None
    ep_zipf = time_ep_layer(dist, rank, world) if dist is not None else None
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    peaks, peak_kind = measured_peaks()
    hbm = float(peaks["hbm_gbs"])
    achieved = kern["gemm_bytes"] / (kern["gemm_ms"] * 1e-3) / 1e9
    tokens = world * SEQ * args.steps
    line = {
        "metric": METRIC, "value": tokens / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (uniform token ids, random-init Parrot XL, seed 0)",
        "timing": "CUDA-graph replay of Parrot.forward (Parrot.capture); events on the replay stream",
        "config": {"workload": "Parrot XL forward 1x512 incl. full logits (BASELINE config 3)",
                   "model": "Parrot XL (16 layers, 16 experts top-2, d=768)",
                   "global_batch": world, "seq_len": SEQ,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "moe_backend": "b200", "depth_backend": "b200",
                   "l2": "weights streamed per step (721 MB) exceed the 126 MB L2"},
        "e2e": {"value": tokens / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size(),
                "d2h_bytes_per_step": logits_host[0].numel() * logits_host[0].element_size(),
                "pipelining": "two captured graphs alternate; step i's logits copy to the host "
                              "on a copy stream while step i + 1 computes; step i + 1's ids "
                              "are copied in on their own stream while step i computes"},
        "gpu_launches": int(launches),
        "launches_per_forward": int(launches_per_forward),
        "eager_ms_per_step": eager_ms,
        "roofline": {"kernel": "grouped_gemm_kernel (gate_up + SwiGLU, routed + shared), T=512",
                     "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "peak_source": peak_kind,
                     "algorithmic_bytes": kern["gemm_bytes"], "launch_us": 1000 * kern["gemm_ms"],
                     "traffic": ncu_traffic("grouped_gemm_gate_up_T512"),
                     "traffic_source": "ncu --set full capture, profiles/traffic.txt"},
        "moe_layer_us": {"T512": 1000 * kern["moe_ms"], "T256": 1000 * kern256["moe_ms"],
                         "gate_up_gemm_T256_us": 1000 * kern256["gemm_ms"]},
        "config2_moe_layer_T256": dict(breakdown, fused_block_us=1000 * kern256["moe_ms"],
                                       fused_block_hbm_frac=(38.95e6 + 0.79e6) / (kern256["moe_ms"] * 1e-3)
                                       / 1e9 / hbm),
        "clocks": clocks,
        "config4_zipf_moe_layer": zipf,
        "config4_ep_zipf_moe_layer": ep_zipf,
        "config5_decode_tokens_per_s": decode,
    }
    if world == 1 and not args.skip_cpu_baseline:
        base = cpu_reference_forward(steps=10, warmup=2)
        line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
        line["cpu_baselines_other_configs"] = cpu_baselines()
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
