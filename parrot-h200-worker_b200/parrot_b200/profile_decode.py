"""Per-kernel timeline of a graph-replayed Parrot XL decode step (or, with
``--forward``, of the graph-replayed 1 x 512 forward the bench times).

Builds Parrot XL (seed 0, bf16), prefills 128 random ids per batch row,
captures one decode step (``Parrot.capture_decode``) and replays it under the
torch profiler (CUDA activity only).  For each kernel kind it prints the
launches per step, the summed duration, and the exposed time (the part of its
duration not overlapped by the kernels before it), averaged over the replays.
The per-step span includes the host gaps between replays.
"""
from __future__ import annotations

import argparse
import collections
import sys
from pathlib import Path

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch  # noqa: E402
from torch.profiler import ProfilerActivity, profile  # noqa: E402

from parrot_b200 import ModelConfig, Parrot  # noqa: E402
from parrot_b200.workloads import random_token_ids  # noqa: E402


def timeline(prof, steps: int, top: int) -> list[str]:
    evs = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    ks = sorted((e.time_range.start, e.time_range.end, e.name) for e in evs)
    exposed, dur, cnt = collections.defaultdict(float), collections.defaultdict(float), \
        collections.Counter()
    prev_end = ks[0][0]
    for s, e, n in ks:
        short = n.replace("(anonymous namespace)::", "").split("(")[0].replace("void ", "")[:56]
        exposed[short] += max(0.0, e - max(s, prev_end))
        dur[short] += e - s
        cnt[short] += 1
        prev_end = max(prev_end, e)
    busy = sum(exposed.values()) / steps
    lines = [f"span {(ks[-1][1] - ks[0][0]) / steps:.1f} us/step, kernels busy "
             f"{busy:.1f} us/step, {len(ks) / steps:.0f} launches/step"]
    for k, v in sorted(exposed.items(), key=lambda kv: -kv[1])[:top]:
        lines.append(f"  {k:56s} n={cnt[k] / steps:5.1f} exposed={v / steps:7.1f} us "
                     f"dur={dur[k] / steps:7.1f} us")
    return lines


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--batches", type=int, nargs="+", default=[1, 8, 64])
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--top", type=int, default=14)
    p.add_argument("--forward", action="store_true", help="the 1 x 512 forward instead")
    a = p.parse_args()
    torch.manual_seed(0)
    model = Parrot(ModelConfig()).to("cuda", torch.bfloat16).eval()
    if a.forward:
        with torch.inference_mode():
            ids = random_token_ids(1, 512, 32768, 0).cuda()
            graphed = model.capture(1, 512)
            for _ in range(3):
                graphed(ids)
            torch.cuda.synchronize()
            with profile(activities=[ProfilerActivity.CUDA], acc_events=True) as prof:
                for _ in range(a.steps):
                    graphed.replay()
                torch.cuda.synchronize()
        print("== graphed forward 1 x 512: " + "\n".join(timeline(prof, a.steps, a.top)))
        return
    with torch.inference_mode():
        for b in a.batches:
            ids = random_token_ids(b, 128, 32768, seed=b).cuda()
            logits, state = model.prefill(ids)
            nxt = logits.argmax(-1)
            step = model.capture_decode(state, next_token_only=True)
            for _ in range(3):
                nxt = step(nxt)
            torch.cuda.synchronize()
            with profile(activities=[ProfilerActivity.CUDA], acc_events=True) as prof:
                for _ in range(a.steps):
                    nxt = step(nxt)
                torch.cuda.synchronize()
            print(f"== graphed decode B={b}: " + "\n".join(timeline(prof, a.steps, a.top)))


if __name__ == "__main__":
    main()
