"""Pin the CPU oracle against golden vectors frozen from the reference itself.

The fixtures under ``tests/golden`` were produced by running the reference's
``moe_backend="pytorch"`` path (``tests/golden/make_golden.py``).  Routing
decisions and grouping order must match exactly; floating-point outputs match
to fp32 round-off.
"""
import json

import numpy as np
import pytest
import torch

from oracle import parrot_oracle as po


def _load(golden_dir, name):
    return np.load(golden_dir / f"{name}.npz")


@pytest.fixture(scope="module")
def meta(golden_dir):
    return json.loads((golden_dir / "meta.json").read_text())


@pytest.fixture(scope="module")
def tiny(meta, golden_dir):
    torch.manual_seed(0)
    model = po.OracleParrot(po.tiny_config()).eval()
    return model, _load(golden_dir, "tiny_forward")


def test_tiny_config_matches_frozen_stand_in(meta):
    frozen = meta["tiny_forward"]["config"]
    cfg = po.tiny_config()
    for key, value in frozen.items():
        assert getattr(cfg, key) == value, key


def test_seeded_init_reproduces_reference_weights(tiny, meta):
    model, _ = tiny
    sums = meta["tiny_forward"]["checksums"]
    state = model.state_dict()
    assert sorted(state) == sorted(sums)
    for name, (s, a, first, last) in sums.items():
        v = state[name].double()
        assert float(v.flatten()[0]) == first, name
        assert float(v.flatten()[-1]) == last, name
        assert abs(float(v.sum()) - s) <= 1e-9 * max(1.0, abs(a)), name


def test_tiny_forward_logits(tiny):
    model, g = tiny
    ids = torch.from_numpy(g["ids"].astype(np.int64))
    with torch.no_grad():
        out = model(ids)
    logits = out.logits[0]
    np.testing.assert_array_equal(logits.argmax(-1).numpy(), g["argmax"])
    np.testing.assert_allclose(torch.logsumexp(logits, -1).numpy(), g["lse"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(logits[g["rows_pos"]].numpy(), g["rows"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(float(out.aux_loss), float(g["aux_loss"]), rtol=1e-5)
    np.testing.assert_allclose(out.expert_utilization.numpy(), g["utilization"], atol=0)


def test_tiny_per_layer_router_decisions(tiny):
    model, g = tiny
    ids = torch.from_numpy(g["ids"].astype(np.int64))
    traces = {}

    def hook(i):
        def fn(m, args, out):
            traces[i] = m.last_trace
        return fn

    hs = [b.moe.register_forward_hook(hook(i)) for i, b in enumerate(model.blocks)]
    with torch.no_grad():
        model(ids)
    for h in hs:
        h.remove()
    for i, tr in traces.items():
        np.testing.assert_array_equal(tr.indices.numpy(), g[f"moe{i}_idx"].astype(np.int64))
        np.testing.assert_allclose(tr.weights.numpy(), g[f"moe{i}_w"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("layer", [0, 3])
def test_tiny_moe_layer_io(tiny, layer):
    model, g = tiny
    x = torch.from_numpy(g[f"moe{layer}_x"])
    with torch.no_grad():
        y, _, _ = model.blocks[layer].moe(x)
    np.testing.assert_allclose(y.numpy(), g[f"moe{layer}_y"], rtol=1e-4, atol=1e-6)


@pytest.fixture(scope="module")
def xl_moe(golden_dir):
    from parrot_b200.workloads import make_moe_layer_weights, make_hidden_states
    cfg = po.OracleConfig()
    moe = po.MoE(cfg)
    moe.load_state_dict(make_moe_layer_weights(cfg.dim, cfg.n_experts, cfg.expert_dim,
                                               cfg.shared_expert_dim, seed=1))
    x = make_hidden_states(256, cfg.dim, seed=0)
    with torch.no_grad():
        y, aux, util = moe(x)
    return moe, x, y, aux, util, _load(golden_dir, "moe_layer")


def test_xl_moe_layer_matches_reference(xl_moe):
    moe, x, y, aux, util, g = xl_moe
    tr = moe.last_trace
    np.testing.assert_array_equal(tr.indices.numpy(), g["idx"].astype(np.int64))
    np.testing.assert_allclose(tr.weights.numpy(), g["w"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(tr.probabilities.numpy(), g["probs"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(y[:64].numpy(), g["y_rows"], rtol=1e-4, atol=1e-6)
    np.testing.assert_allclose(y.double().sum(-1).numpy(), g["y_rowsum"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(y.double().abs().sum(-1).numpy(), g["y_abssum"], rtol=1e-5)
    np.testing.assert_allclose(float(aux), float(g["aux"]), rtol=1e-6)
    np.testing.assert_array_equal(util.numpy(), g["util"])


def test_grouping_restatement_matches_reference_where_order(xl_moe):
    """The stable counting sort equals ``torch.where(indices == e)`` order."""
    *_, g = xl_moe
    idx = g["idx"].astype(np.int64)
    grouping = po.group_assignments(idx, 16)
    for e in range(16):
        np.testing.assert_array_equal(np.array(grouping.order[e]), g[f"order{e}"])
        for rank, a in enumerate(grouping.order[e]):
            assert grouping.slots[a] == rank
    assert sum(grouping.counts) == idx.size
    assert grouping.capacity == po.expert_capacity(512, 16) == 64


def test_grouped_rows_layout_and_overflow():
    # 3 experts, capacity 8: expert 0 takes 11 assignments -> 3 overflow rows
    idx = np.array([[0, 1]] * 11 + [[2, 0]] * 0 + [[2, 1]] * 2)
    grouping = po.group_assignments(idx, 3, capacity=8)
    rows = po.grouped_rows(grouping, idx)
    assert grouping.counts == [11, 13, 2]
    flat = idx.reshape(-1)
    seen = set()
    for a, (e, r) in enumerate(zip(flat, rows)):
        s = grouping.slots[a]
        if s < 8:
            assert r == e * 8 + s
        else:
            # overflow: expert 0 first (3 rows), then expert 1 (5 rows)
            base = 3 * 8 + (0 if e == 0 else 3)
            assert r == base + s - 8
        assert r not in seen
        seen.add(r)


def test_capacity_formula():
    assert po.expert_capacity(512, 16) == 64
    assert po.expert_capacity(1024, 16) == 128
    assert po.expert_capacity(32768, 16) == 4096
    assert po.expert_capacity(2, 16) == 8
    assert po.expert_capacity(6, 4) == 8


@pytest.fixture(scope="module")
def micro(golden_dir, meta):
    g = _load(golden_dir, "micro")
    cfg = po.OracleConfig(**meta["micro"]["config"])
    model = po.OracleParrot(cfg).eval()
    state = {k[len("param::"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("param::")}
    model.load_state_dict(state)
    return model, g


def test_micro_forward_with_labels(micro):
    model, g = micro
    ids = torch.from_numpy(g["ids"].astype(np.int64))
    with torch.no_grad():
        out = model(ids, labels=ids)
    np.testing.assert_allclose(out.logits.numpy(), g["logits"], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(float(out.loss), float(g["loss"]), rtol=1e-5)
    np.testing.assert_allclose(float(out.lm_loss), float(g["lm_loss"]), rtol=1e-5)
    np.testing.assert_allclose(float(out.aux_loss), float(g["aux_loss"]), rtol=1e-5)


def test_micro_prefill_and_decode(micro):
    model, g = micro
    ids = torch.from_numpy(g["ids"].astype(np.int64))
    logits, state = model.prefill(ids[:, :20])
    np.testing.assert_allclose(logits.numpy(), g["prefill_logits"], rtol=1e-4, atol=1e-5)
    nxt = logits.argmax(-1)
    for step in range(3):
        lg, state = model.decode_step(nxt, state)
        np.testing.assert_allclose(lg.numpy(), g["decode_logits"][step], rtol=1e-4, atol=1e-5)
        nxt = lg.argmax(-1)
    assert state.position == 23
