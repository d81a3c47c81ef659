"""Freeze golden vectors from the reference's own ``moe_backend="pytorch"`` path.

Run in the build container, where the reference package imports read-only::

    PYTHONPATH=<reference checkout> PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_golden.py <reference checkout>

It writes ``tests/golden/*.npz`` plus ``meta.json`` (torch version, seeds).
Nothing on the GPU box reads the reference; tests read only these files.

Fixtures
--------
``tiny_forward``   BASELINE config 1: the frozen tiny stand-in config, seed 0,
                   fp32 CPU forward on 1x512 ids (seed 0).  Parameter
                   checksums, logits summaries, per-layer MoE in/out and
                   router decisions, aux loss and utilisation.
``moe_layer``      BASELINE config 2 shape: one XL MoE layer, T=256, x~N(0,1)
                   (seed 0), weights ~N(0, 0.02) (seed 1), fp32 CPU.
``micro``          A small model whose every parameter (depth queries and norm
                   weights included) is randomised, batch 2 x 37 positions:
                   forward with labels, prefill and three decode steps.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "parrot-h200-worker_b200"))

from parrot_b200.workloads import make_moe_layer_weights  # noqa: E402


def tiny_kwargs():
    return dict(vocab_size=32768, dim=128, n_layers=4, n_heads=4, n_kv_heads=2,
                head_dim=32, kv_latent_dim=32, n_experts=8, top_k=2,
                expert_dim=128, shared_expert_dim=64, window_size=128,
                max_seq_len=512)


def micro_kwargs():
    return dict(vocab_size=96, dim=64, n_layers=2, n_heads=2, n_kv_heads=1,
                head_dim=16, kv_latent_dim=16, global_every=2, n_experts=4, top_k=2,
                expert_dim=32, shared_expert_dim=16, window_size=8,
                local_query_chunk=16, max_seq_len=64)


def checksums(model) -> dict:
    out = {}
    for name, p in model.state_dict().items():
        v = p.detach().double()
        out[name] = [float(v.sum()), float(v.abs().sum()), float(v.flatten()[0]),
                     float(v.flatten()[-1])]
    return out


def route_like_reference(flat, weight, top_k):
    # model.py:522-527, evaluated on the captured MoE input
    probs = torch.nn.functional.linear(flat.float(), weight.float()).softmax(-1)
    w, idx = probs.topk(top_k, dim=-1)
    return probs, w / w.sum(-1, keepdim=True), idx


def where_order(idx, n_experts):
    """Per expert, the flattened assignment ids in ``torch.where`` order."""
    k = idx.shape[1]
    order = []
    for e in range(n_experts):
        rows, slots = torch.where(idx == e)
        order.append((rows * k + slots).numpy().astype(np.int32))
    return order


def tiny_forward(ModelConfig, Parrot):
    cfg = ModelConfig(**tiny_kwargs())
    torch.manual_seed(0)
    model = Parrot(cfg).eval()
    ids = torch.randint(0, 32768, (1, 512), generator=torch.Generator().manual_seed(0))
    captured = {}

    def hook(index):
        def fn(module, args, output):
            captured[index] = (args[0].detach().clone(), output[0].detach().clone())
        return fn

    handles = [b.moe.register_forward_hook(hook(i)) for i, b in enumerate(model.blocks)]
    with torch.no_grad():
        out = model(ids)
    for h in handles:
        h.remove()
    logits = out.logits[0]
    arrays = {
        "ids": ids.numpy().astype(np.int32),
        "argmax": logits.argmax(-1).numpy().astype(np.int32),
        "lse": torch.logsumexp(logits, -1).numpy(),
        "rows_pos": np.array([0, 1, 127, 128, 255, 256, 511], dtype=np.int32),
        "aux_loss": np.array(float(out.aux_loss)),
        "utilization": out.expert_utilization.numpy(),
    }
    arrays["rows"] = logits[arrays["rows_pos"]].numpy()
    for i, (x, y) in captured.items():
        flat = x.reshape(-1, cfg.dim)
        probs, w, idx = route_like_reference(flat, model.blocks[i].moe.router.weight, 2)
        arrays[f"moe{i}_idx"] = idx.numpy().astype(np.int8)
        arrays[f"moe{i}_w"] = w.numpy()
        if i in (0, cfg.n_layers - 1):
            arrays[f"moe{i}_x"] = flat.numpy()
            arrays[f"moe{i}_y"] = y.reshape(-1, cfg.dim).numpy()
    np.savez_compressed(HERE / "tiny_forward.npz", **arrays)
    return {"tiny_forward": {"config": tiny_kwargs(), "seed": 0,
                             "checksums": checksums(model)}}


def moe_layer(ModelConfig, MoE):
    cfg = ModelConfig()
    moe = MoE(cfg)
    weights = make_moe_layer_weights(cfg.dim, cfg.n_experts, cfg.expert_dim,
                                     cfg.shared_expert_dim, seed=1)
    moe.load_state_dict(weights)
    moe.eval()
    x = torch.randn(256, cfg.dim, generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        y, aux, util = moe(x)
    probs, w, idx = route_like_reference(x, moe.router.weight, 2)
    order = where_order(idx, cfg.n_experts)
    arrays = {
        "idx": idx.numpy().astype(np.int8),
        "w": w.numpy(),
        "probs": probs.numpy(),
        "y_rows": y[:64].numpy(),
        "y_rowsum": y.double().sum(-1).numpy(),
        "y_abssum": y.double().abs().sum(-1).numpy(),
        "aux": np.array(float(aux)),
        "util": util.numpy(),
    }
    for e, o in enumerate(order):
        arrays[f"order{e}"] = o
    np.savez_compressed(HERE / "moe_layer.npz", **arrays)
    return {"moe_layer": {"tokens": 256, "x_seed": 0, "weight_seed": 1, "std": 0.02}}


def micro(ModelConfig, Parrot):
    cfg = ModelConfig(**micro_kwargs())
    torch.manual_seed(5)
    model = Parrot(cfg).eval()
    g = torch.Generator().manual_seed(11)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("query"):
                p.copy_(torch.randn(p.shape, generator=g) * 0.5)
            elif p.ndim == 1:
                p.copy_(1.0 + 0.2 * torch.randn(p.shape, generator=g))
    ids = torch.randint(0, cfg.vocab_size, (2, 37), generator=torch.Generator().manual_seed(3))
    with torch.no_grad():
        out = model(ids, labels=ids)
        logits_p, state = model.prefill(ids[:, :20])
        steps = []
        nxt = logits_p.argmax(-1)
        for _ in range(3):
            lg, state = model.decode_step(nxt, state)
            steps.append(lg)
            nxt = lg.argmax(-1)
    arrays = {f"param::{k}": v.numpy() for k, v in model.state_dict().items()}
    arrays.update({
        "ids": ids.numpy().astype(np.int32),
        "logits": out.logits.numpy(),
        "loss": np.array(float(out.loss)),
        "lm_loss": np.array(float(out.lm_loss)),
        "aux_loss": np.array(float(out.aux_loss)),
        "utilization": out.expert_utilization.numpy(),
        "prefill_logits": logits_p.numpy(),
        "decode_logits": torch.stack(steps).numpy(),
    })
    np.savez_compressed(HERE / "micro.npz", **arrays)
    return {"micro": {"config": micro_kwargs(), "prompt": 20, "decode_steps": 3}}


def main():
    from parrot import ModelConfig, Parrot
    from parrot.model import MoE
    torch.set_num_threads(8)
    meta = {"torch": torch.__version__, "generator": "tests/golden/make_golden.py"}
    with torch.no_grad():
        meta.update(tiny_forward(ModelConfig, Parrot))
        meta.update(moe_layer(ModelConfig, MoE))
        meta.update(micro(ModelConfig, Parrot))
    (HERE / "meta.json").write_text(json.dumps(meta, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
