"""Small, fixed workloads for profiling the B200 kernels under Nsight Compute.

    python parrot-h200-worker_b200/parrot_b200/profile_moe.py --tokens 512 --iters 3
    python parrot-h200-worker_b200/parrot_b200/profile_moe.py --forward --iters 2

``--tokens T`` runs ``iters`` eager calls of one Parrot XL MoE block (seeded
weights ~N(0, 0.02), x ~ N(0, 1)); each call launches route, group,
gate_up GEMM, down GEMM and combine, in that order.  ``--forward`` runs
``iters`` eager Parrot XL forwards on 1 x 512 ids.  ``--vocab B`` runs ``iters``
greedy next-token calls (the tied LM head fused with the argmax) for B rows
over the 32768 x 768 embedding.  ``--norms ROWS`` runs
``iters`` rounds of RMSNorm, then the depth mix over 4 and over 8 sources
(each with the consumer RMSNorm), on [ROWS, 768] bf16 rows.  Device memory stays under
2 GB, so ``ncu`` captures of these commands end in seconds.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

if __package__ in (None, ""):
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

import torch  # noqa: E402

from parrot_b200 import ModelConfig, Parrot  # noqa: E402
from parrot_b200.model import MoE  # noqa: E402
from parrot_b200.workloads import (make_hidden_states, make_moe_layer_weights,  # noqa: E402
                                   random_token_ids, tune_zipf_router_bias)


def moe_block(tokens: int, iters: int, zipf: bool) -> None:
    cfg = ModelConfig()
    moe = MoE(cfg)
    w = make_moe_layer_weights(cfg.dim, cfg.n_experts, cfg.expert_dim, cfg.shared_expert_dim, 1)
    moe.load_state_dict(w)
    x = make_hidden_states(tokens, cfg.dim, 0)
    moe = moe.to("cuda", torch.bfloat16).eval()
    if zipf:
        moe.router_bias = tune_zipf_router_bias(x, w["router.weight"]).to("cuda", torch.float32)
    xd = x.to("cuda", torch.bfloat16)
    with torch.inference_mode():
        for _ in range(iters):
            moe(xd)
    torch.cuda.synchronize()


def norms(rows: int, iters: int) -> None:
    from parrot_b200.model import DepthMix, RMSNorm
    cfg = ModelConfig()
    g = torch.Generator().manual_seed(0)
    src = [torch.randn(rows, cfg.dim, generator=g).to("cuda", torch.bfloat16) for _ in range(8)]
    norm = RMSNorm(cfg.dim, cfg.norm_eps).to("cuda", torch.bfloat16)
    depth = DepthMix(cfg).to("cuda", torch.bfloat16)
    with torch.no_grad():
        depth.query.copy_(0.5 * torch.randn(cfg.dim, generator=g))
    with torch.inference_mode():
        for _ in range(iters):
            norm(src[0])
            depth.normalized(src[:4], norm)
            depth.normalized(src, norm)
    torch.cuda.synchronize()


def vocab(rows: int, iters: int) -> None:
    from parrot_b200 import bridge
    g = torch.Generator().manual_seed(0)
    w = (0.02 * torch.randn(32768, 768, generator=g)).to("cuda", torch.bfloat16)
    h = torch.randn(rows, 1, 768, generator=g).to("cuda", torch.bfloat16)
    with torch.inference_mode():
        for _ in range(iters):
            bridge.b200_vocab_argmax(h, w)
    torch.cuda.synchronize()


def forward(iters: int) -> None:
    torch.manual_seed(0)
    model = Parrot(ModelConfig()).to("cuda", torch.bfloat16).eval()
    ids = random_token_ids(1, 512, 32768, 0).cuda()
    with torch.inference_mode():
        for _ in range(iters):
            model(ids)
    torch.cuda.synchronize()


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--forward", action="store_true")
    p.add_argument("--zipf", action="store_true", help="Zipf(1.2) router bias (overflow path)")
    p.add_argument("--norms", type=int, default=0, help="rows for the RMSNorm / depth-mix workload")
    p.add_argument("--vocab", type=int, default=0, help="rows for the fused LM-head argmax")
    a = p.parse_args()
    if a.vocab:
        vocab(a.vocab, a.iters)
    elif a.norms:
        norms(a.norms, a.iters)
    elif a.forward:
        forward(a.iters)
    else:
        moe_block(a.tokens, a.iters, a.zipf)
    print("profile workload done")


if __name__ == "__main__":
    main()
