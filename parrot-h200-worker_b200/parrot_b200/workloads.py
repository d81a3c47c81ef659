"""Seeded synthetic workloads for the Parrot XL MoE block.

The reference measures on synthetic inputs only (no dataset); these helpers
draw them deterministically so the CUDA path, the CPU baseline and the parity
tests all see identical tensors.
"""
from __future__ import annotations

import torch
from torch import Tensor

#: Target Zipf(s=1.2) assignment shares over 16 routed experts.
ZIPF_16 = (0.365, 0.159, 0.098, 0.069, 0.053, 0.043, 0.035, 0.030,
           0.026, 0.023, 0.021, 0.019, 0.017, 0.015, 0.014, 0.013)


def make_moe_layer_weights(dim: int, n_experts: int, expert_dim: int, shared_dim: int,
                           seed: int, std: float = 0.02) -> dict[str, Tensor]:
    """``torch.nn.Linear``-layout ([out, in]) weights for one MoE layer.

    Keys match the reference ``MoE`` module's ``state_dict``
    (``parrot/model.py:467, 493-503``).  Every tensor is drawn from one
    generator in a fixed order, so a seed names one weight set everywhere.
    """
    g = torch.Generator().manual_seed(seed)

    def draw(*shape):
        return torch.randn(*shape, generator=g) * std

    w = {"router.weight": draw(n_experts, dim)}
    for e in range(n_experts):
        w[f"experts.{e}.gate.weight"] = draw(expert_dim, dim)
        w[f"experts.{e}.up.weight"] = draw(expert_dim, dim)
        w[f"experts.{e}.down.weight"] = draw(dim, expert_dim)
    w["shared.gate.weight"] = draw(shared_dim, dim)
    w["shared.up.weight"] = draw(shared_dim, dim)
    w["shared.down.weight"] = draw(dim, shared_dim)
    return w


def make_hidden_states(tokens: int, dim: int, seed: int) -> Tensor:
    """``x ~ N(0, 1)``, ``[tokens, dim]`` fp32 on the CPU."""
    return torch.randn(tokens, dim, generator=torch.Generator().manual_seed(seed))


def tune_zipf_router_bias(x: Tensor, router_weight: Tensor,
                          target=ZIPF_16, iterations: int = 300) -> Tensor:
    """Per-expert router logit offsets whose top-2 assignment shares follow ``target``.

    The reference router has no bias (``parrot/model.py:467``).  The skewed
    stress workload adds a harness-only offset ``b[e]`` to the fp32 router
    logits before the softmax, identically on every path.  The offsets are
    fitted on the given sample by damped fixed-point steps
    ``b += clamp(log(target / achieved) / 2, -s, s)`` with a shrinking step
    limit ``s`` (undamped steps oscillate: a share of 0 makes the log step
    huge).  Deterministic: the same (x, weights) always gives the same bias.
    The top-2 of the logits equals the top-2 of the softmax, so the fit
    works on logits.
    """
    logits = (x.float() @ router_weight.float().t()).double()
    target_t = torch.tensor(target, dtype=torch.float64)
    target_t = target_t / target_t.sum()
    bias = torch.log(target_t)
    n = logits.shape[1]
    for it in range(iterations):
        idx = (logits + bias).topk(2, dim=-1).indices
        share = torch.bincount(idx.flatten(), minlength=n).double() / idx.numel()
        limit = 0.25 * 0.985 ** it
        step = 0.5 * torch.log(target_t.clamp_min(1e-9) / share.clamp_min(1e-4))
        bias = bias + step.clamp(-limit, limit)
        bias = bias - bias.max()
    return bias.float()


def random_token_ids(batch: int, length: int, vocab: int, seed: int) -> Tensor:
    """Uniform token ids in ``[0, vocab)``, as the reference benchmarks draw them."""
    return torch.randint(0, vocab, (batch, length),
                         generator=torch.Generator().manual_seed(seed))
