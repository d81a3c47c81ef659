"""The integration patch applies to the reference package and its config
accepts the B200 backend with the kernels' shape checks (no GPU needed)."""
import pytest

from tests.reference_patch import patched_reference


@pytest.fixture(scope="module")
def ref(tmp_path_factory):
    mod = patched_reference(tmp_path_factory.mktemp("ref"))
    if mod is None:
        pytest.skip("reference package not installed under baseline/_ref")
    return mod


def test_patched_config_selects_b200(ref):
    cfg = ref.ModelConfig(moe_backend="b200", depth_backend="b200")
    assert (cfg.moe_backend, cfg.depth_backend) == ("b200", "b200")
    ref.ModelConfig(moe_backend="b200")           # depth mixing may stay on pytorch
    ref.ModelConfig(depth_backend="b200")


@pytest.mark.parametrize("field,value,msg", [("top_k", 3, "top_k=2"), ("dim", 96, "dim"),
                                             ("n_experts", 64, "routed experts"),
                                             ("expert_dim", 100, "expert widths")])
def test_patched_config_rejects_shapes_the_kernels_do_not_take(ref, field, value, msg):
    with pytest.raises(ValueError, match=msg):
        ref.ModelConfig(moe_backend="b200", **{field: value})


def test_b200_norms_are_keyed_on_the_config(ref):
    model = ref.Parrot(ref.ModelConfig(vocab_size=256, dim=128, n_layers=2, n_heads=4,
                                       n_kv_heads=2, head_dim=32, kv_latent_dim=32,
                                       n_experts=4, expert_dim=64, shared_expert_dim=64,
                                       moe_backend="b200", depth_backend="b200"))
    assert model.final_norm.use_b200
    assert all(b.attention_norm.use_b200 and b.moe_norm.use_b200 for b in model.blocks)
    assert all(d.norm.use_b200 for d in model.depth_mix)
    plain = ref.Parrot(ref.ModelConfig(vocab_size=256, dim=128, n_layers=2, n_heads=4,
                                       n_kv_heads=2, head_dim=32, kv_latent_dim=32,
                                       n_experts=4, expert_dim=64, shared_expert_dim=64))
    assert not plain.final_norm.use_b200
