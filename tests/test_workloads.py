"""The synthetic workloads the benchmarks use (no GPU needed)."""
import torch

from oracle import parrot_oracle as po
from parrot_b200.workloads import (ZIPF_16, make_hidden_states, make_moe_layer_weights,
                                   tune_zipf_router_bias)


def test_zipf_router_bias_reaches_target_shares_and_overflows():
    # the skewed stress layer: 16384 tokens, XL widths, weights seed 1, x seed 0
    w = make_moe_layer_weights(768, 16, 512, 256, seed=1)
    x = make_hidden_states(16384, 768, seed=0)
    bias = tune_zipf_router_bias(x, w["router.weight"])
    logits = x @ w["router.weight"].t() + bias
    idx = logits.softmax(-1).topk(2, dim=-1).indices
    counts = torch.bincount(idx.flatten(), minlength=16)
    share = counts.double() / idx.numel()
    target = torch.tensor(ZIPF_16, dtype=torch.float64)
    assert (share - target / target.sum()).abs().max() < 5e-3, share.tolist()
    capacity = po.expert_capacity(idx.numel(), 16)
    assert capacity == 4096
    assert counts[0] > capacity and counts[1] > capacity and counts[2] < capacity
