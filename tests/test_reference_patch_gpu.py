"""The reference's own Parrot, patched to select the B200 backend, on the GPU.

The patch (parrot-h200-worker_b200/integration/reference_model_b200.patch)
adds ``"b200"`` to the reference's ``moe_backend`` / ``depth_backend`` and
branches in ``RMSNorm.forward``, ``DepthMix.forward`` / ``normalized``,
``MoE.forward`` / ``inference`` and ``decode_next``, the places where the
reference selects its Metal backends.  The reference's ``Parrot.forward``
must then take those branches (counted) and give logits within the stated
bounds of the fp32 oracle, next to the reference's own bf16 pytorch path and
the product model on the same weights.
"""
import pytest
import torch

from oracle import parrot_oracle as po
from parrot_b200 import ModelConfig, Parrot, bridge
from tests.gpu_helpers import cosine, err_stats
from tests.reference_patch import patched_reference

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref(tmp_path_factory):
    mod = patched_reference(tmp_path_factory.mktemp("ref"))
    if mod is None:
        pytest.skip("reference package not installed under baseline/_ref")
    return mod


def _count_calls(monkeypatch, names):
    counts = dict.fromkeys(names, 0)
    for name in names:
        fn = getattr(bridge, name)

        def wrapped(*args, _fn=fn, _name=name, **kwargs):
            counts[_name] += 1
            return _fn(*args, **kwargs)

        monkeypatch.setattr(bridge, name, wrapped)
    return counts


@pytest.mark.parametrize("residual", ["attnres", "standard"])
def test_reference_forward_on_the_b200_backend(ref, monkeypatch, residual):
    torch.manual_seed(0)
    model = ref.Parrot(ref.ModelConfig(moe_backend="b200", depth_backend="b200",
                                       residual=residual)).to("cuda", torch.bfloat16).eval()
    state = model.state_dict()
    plain = ref.Parrot(ref.ModelConfig(residual=residual))
    plain.load_state_dict(state)
    plain = plain.to("cuda", torch.bfloat16).eval()
    prod = Parrot(ModelConfig(residual=residual))
    prod.load_state_dict(state)
    prod = prod.to("cuda", torch.bfloat16).eval()
    okw = {k: v for k, v in ModelConfig(residual=residual).__dict__.items()
           if k in po.OracleConfig.__dataclass_fields__}
    orc = po.OracleParrot(po.OracleConfig(**okw)).eval()
    orc.load_state_dict({k: v.float().cpu() for k, v in state.items()})
    ids = torch.randint(0, 32768, (1, 512), generator=torch.Generator().manual_seed(0))

    counts = _count_calls(monkeypatch, ["b200_moe", "b200_depth_mix_norm", "b200_depth_mix",
                                        "b200_rms_norm"])
    with torch.inference_mode():
        out = model(ids.cuda())
    monkeypatch.undo()
    # the reference's forward mixes (DepthMix.forward) and then normalises
    # (RMSNorm.forward) each of the 32 sublayer inputs and the final output
    assert counts["b200_moe"] == 16, counts
    assert counts["b200_rms_norm"] == 33, counts
    assert counts["b200_depth_mix"] == (33 if residual == "attnres" else 0), counts
    assert out.expert_utilization.shape == (16, 16) and torch.isfinite(out.aux_loss)

    with torch.inference_mode():
        pt = plain(ids.cuda()).logits
        ours = prod(ids.cuda()).logits
    with torch.no_grad():
        exp = orc(ids).logits
    c_b200, c_pt = cosine(out.logits, exp), cosine(pt, exp)
    print(f"{residual}: reference+b200 cosine {c_b200:.6f}, reference bf16 pytorch {c_pt:.6f}, "
          f"vs product {cosine(out.logits, ours):.6f}")
    assert 1 - c_b200 <= 2.25 * (1 - c_pt) + 1e-5, (c_b200, c_pt)
    assert err_stats(out.logits, exp)["rms_rel"] <= 1.5 * err_stats(pt, exp)["rms_rel"] + 1e-3
    assert cosine(out.logits, ours) >= 0.999
