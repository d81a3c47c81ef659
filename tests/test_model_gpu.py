"""End-to-end parity of the B200 Parrot model against the CPU oracle.

The product model (bf16 on the GPU, hot path on sm_100a kernels) and the
oracle (fp32 on the CPU) load identical bf16-representable weights.  The
stated tolerance is relative to the reference algorithm itself executed in
bf16 on the same GPU (the oracle's torch ops in bf16): the b200 logits may
deviate from the fp32 oracle by at most 1.5x the RMS deviation of that bf16
reference execution (+1e-3), and their cosine distance by at most 2.25x its
cosine distance (+1e-5).  At seed-0 weights the bf16 reference execution
itself reaches cosine 0.99938 on Parrot XL, so an absolute 0.9999 bound would
reject the reference too; every case also checks an absolute floor.
"""
import pytest
import torch

from oracle import parrot_oracle as po
from parrot_b200 import ModelConfig, Parrot
from tests.gpu_helpers import cosine, err_stats

pytestmark = pytest.mark.gpu

TINY = dict(vocab_size=32768, dim=128, n_layers=4, n_heads=4, n_kv_heads=2, head_dim=32,
            kv_latent_dim=32, n_experts=8, expert_dim=128, shared_expert_dim=64,
            window_size=128, max_seq_len=512)


def _pair(kw: dict, seed: int = 0, randomize: bool = False, **cfg_extra):
    cfg = ModelConfig(**kw, **cfg_extra)
    torch.manual_seed(seed)
    prod = Parrot(cfg)
    if randomize:
        g = torch.Generator().manual_seed(seed + 100)
        with torch.no_grad():
            for name, p in prod.named_parameters():
                if name.endswith("query"):
                    p.copy_(0.5 * torch.randn(p.shape, generator=g))
                elif p.ndim == 1:
                    p.copy_(1 + 0.2 * torch.randn(p.shape, generator=g))
    prod = prod.to("cuda", torch.bfloat16).eval()
    okw = {k: v for k, v in cfg.__dict__.items()
           if k in po.OracleConfig.__dataclass_fields__}
    orc = po.OracleParrot(po.OracleConfig(**okw)).eval()
    orc.load_state_dict({k: v.float().cpu() for k, v in prod.state_dict().items()})
    return prod, orc


def _reference_bf16(orc: po.OracleParrot) -> po.OracleParrot:
    """The oracle's torch ops in bf16 on the GPU: the reference's own bf16 execution."""
    import copy
    return copy.deepcopy(orc).to("cuda", torch.bfloat16)


def _assert_within_reference(ours, exp, ref, floor):
    co, cr = cosine(ours, exp), cosine(ref, exp)
    so, sr = err_stats(ours, exp)["rms_rel"], err_stats(ref, exp)["rms_rel"]
    assert so <= 1.5 * sr + 1e-3, (so, sr)
    assert 1 - co <= 2.25 * (1 - cr) + 1e-5, (co, cr)
    assert co >= floor, (co, cr)
    return co, cr


@pytest.mark.parametrize("randomize,floor", [(False, 0.999), (True, 0.995)])
def test_tiny_forward_logits(randomize, floor):
    prod, orc = _pair(TINY, randomize=randomize)
    ids = torch.randint(0, 32768, (1, 512), generator=torch.Generator().manual_seed(0))
    with torch.inference_mode():
        got = prod(ids.cuda())
        ref = _reference_bf16(orc)(ids.cuda())
    with torch.no_grad():
        exp = orc(ids)
    _assert_within_reference(got.logits, exp.logits, ref.logits, floor)
    assert abs(float(got.aux_loss) - float(exp.aux_loss)) < 2e-2 * float(exp.aux_loss)
    assert got.expert_utilization.shape == exp.expert_utilization.shape
    torch.testing.assert_close(got.expert_utilization.sum(-1).cpu(),
                               torch.ones(TINY["n_layers"]), rtol=0, atol=1e-6)


def test_tiny_forward_matches_golden_reference(golden_dir):
    """Config 1 against the reference's own frozen fp32 outputs (seed-0 weights)."""
    import numpy as np
    g = np.load(golden_dir / "tiny_forward.npz")
    cfg = ModelConfig(**TINY)
    torch.manual_seed(0)
    prod = Parrot(cfg).to("cuda", torch.bfloat16).eval()
    ids = torch.from_numpy(g["ids"].astype(np.int64)).cuda()
    with torch.inference_mode():
        logits = prod(ids).logits[0].float().cpu()
    rows = torch.from_numpy(g["rows"])
    pos = torch.from_numpy(g["rows_pos"].astype(np.int64))
    assert cosine(logits[pos], rows) >= 0.999
    lse = torch.logsumexp(logits, -1)
    assert float((lse - torch.from_numpy(g["lse"])).abs().max()) < 5e-2
    agree = (logits.argmax(-1).numpy() == g["argmax"]).mean()
    assert agree >= 0.99  # measured on a B200: 512 of 512


def test_forward_with_labels_bag4_and_supervised_only():
    prod, orc = _pair(TINY, seed=3)
    ids = torch.randint(0, 32768, (2, 128), generator=torch.Generator().manual_seed(4))
    with torch.inference_mode():
        got = prod(ids.cuda(), labels=ids.cuda(), bag_size=4, supervised_logits_only=True)
        ref = _reference_bf16(orc)(ids.cuda(), labels=ids.cuda(), bag_size=4,
                                   supervised_logits_only=True)
    with torch.no_grad():
        exp = orc(ids, labels=ids, bag_size=4, supervised_logits_only=True)
    assert got.logits.shape == exp.logits.shape == (2, 31, 32768)
    _assert_within_reference(got.logits, exp.logits, ref.logits, 0.999)
    # the reference test's loss tolerance (tests/test_cuda_training.py:56)
    torch.testing.assert_close(got.loss.float().cpu(), exp.loss, atol=2e-2, rtol=2e-2)


def test_standard_residual_variant():
    prod, orc = _pair(TINY, seed=5, residual="standard")
    ids = torch.randint(0, 32768, (1, 96), generator=torch.Generator().manual_seed(6))
    with torch.inference_mode():
        got = prod(ids.cuda())
        ref = _reference_bf16(orc)(ids.cuda())
    with torch.no_grad():
        exp = orc(ids)
    _assert_within_reference(got.logits, exp.logits, ref.logits, 0.999)


@pytest.mark.parametrize("batch", [1, 3])
def test_prefill_and_decode(batch):
    prod, orc = _pair(TINY, seed=7)
    ids = torch.randint(0, 32768, (batch, 150), generator=torch.Generator().manual_seed(8))
    lp, state = prod.prefill(ids[:, :140].cuda())
    le, ostate = orc.prefill(ids[:, :140])
    ref_lp, _ = _reference_bf16(orc).prefill(ids[:, :140].cuda())
    _assert_within_reference(lp, le, ref_lp, 0.999)
    for step in range(4):
        nxt = ids[:, 140 + step:141 + step]
        lp, state = prod.decode_step(nxt.cuda(), state)
        le, ostate = orc.decode_step(nxt, ostate)
        assert cosine(lp, le) >= 0.999, step
    assert state.position == 144
    tok, state = prod.decode_next(ids[:, 144:145].cuda(), state)
    assert tok.shape == (batch, 1)
    assert state.position == 145


@pytest.mark.parametrize("next_only", [False, True])
def test_graphed_decode_equals_eager(next_only):
    """One captured decode step replayed at successive positions gives the
    eager decode's outputs exactly (the window is exceeded along the way)."""
    prod, _ = _pair(TINY, seed=12)
    ids = torch.randint(0, 32768, (2, 134), generator=torch.Generator().manual_seed(13))
    with torch.inference_mode():
        _, eager_state = prod.prefill(ids[:, :126].cuda())
        _, graph_state = prod.prefill(ids[:, :126].cuda())
        graphed = prod.capture_decode(graph_state, next_token_only=next_only)
        for step in range(8):
            nxt = ids[:, 126 + step:127 + step]
            if next_only:
                want, eager_state = prod.decode_next(nxt.cuda(), eager_state)
            else:
                want, eager_state = prod.decode_step(nxt.cuda(), eager_state)
            got = graphed(nxt)
            assert torch.equal(got, want), step
            assert graph_state.position == eager_state.position == 127 + step
        assert int(graph_state.position_device.item()) == graph_state.position


def test_xl_forward_1x512():
    """Parrot XL default, seed 0, bf16 forward on 1x512 ids."""
    prod, orc = _pair({}, seed=0)
    ids = torch.randint(0, 32768, (1, 512), generator=torch.Generator().manual_seed(0))
    with torch.inference_mode():
        got = prod(ids.cuda())
        ref = _reference_bf16(orc)(ids.cuda())
    with torch.no_grad():
        exp = orc(ids)
    _assert_within_reference(got.logits, exp.logits, ref.logits, 0.999)


def test_forward_requires_inference_mode():
    prod, _ = _pair(TINY)
    ids = torch.randint(0, 32768, (1, 16)).cuda()
    with pytest.raises(RuntimeError, match="inference-only"):
        prod(ids)


def test_graphed_forward_equals_eager():
    prod, _ = _pair(TINY, seed=9)
    ids = torch.randint(0, 32768, (2, 64), generator=torch.Generator().manual_seed(10))
    with torch.inference_mode():
        eager = prod(ids.cuda())
        graphed = prod.capture(2, 64)
        out = graphed(ids)  # host ids: copied into the captured buffer
        assert torch.equal(out.logits, eager.logits)
        assert torch.equal(out.expert_utilization, eager.expert_utilization)
        ids2 = torch.randint(0, 32768, (2, 64), generator=torch.Generator().manual_seed(11))
        again = graphed(ids2.cuda()).logits.clone()
        assert torch.equal(again, prod(ids2.cuda()).logits)


@pytest.mark.parametrize("kw,batch,seq", [(TINY, 2, 64), ({}, 1, 512)])
def test_deferred_moe_combine_is_bit_identical(kw, batch, seq):
    """Each MoE block's combine folded into the next depth mix (the default)
    gives exactly the logits, prefill logits and decode outputs of running
    the combine kernel."""
    from parrot_b200 import bridge
    prod, _ = _pair(kw, seed=3)
    ids = torch.randint(0, 32768, (batch, seq), generator=torch.Generator().manual_seed(4))
    outs = {}
    try:
        for defer in (True, False):
            bridge.DEFER_MOE_COMBINE = defer
            with torch.inference_mode():
                fwd = prod(ids.cuda())
                logits = torch.cat([fwd.logits.flatten().float(), fwd.aux_loss.flatten().float(),
                                    fwd.expert_utilization.flatten().float()])
                lp, state = prod.prefill(ids[:, :seq - 8].cuda())
                steps = [prod.decode_step(ids[:, seq - 8 + i:seq - 7 + i].cuda(), state)[0].clone()
                         for i in range(3)]
            outs[defer] = (logits, lp.clone(), steps)
    finally:
        bridge.DEFER_MOE_COMBINE = True
    assert torch.equal(outs[True][0], outs[False][0])
    assert torch.equal(outs[True][1], outs[False][1])
    for a, b in zip(outs[True][2], outs[False][2]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("batch", [1, 8, 64])
def test_xl_cached_generation_matches_oracle(batch):
    """BASELINE config 5 at Parrot XL: prefill 128 ids, then 16 decode steps
    (model.py:817-931) against the oracle's decode_step, teacher-forced with
    the oracle's greedy tokens.  B = 1 takes the small-batch decode MoE and
    projection kernels, B = 8 the grouped-GEMM MoE with the small-batch
    projections, B = 64 the grouped GEMMs and cuBLAS projections; the greedy
    token comes from the fused vocabulary argmax up to 8 rows.

    Yardstick: the reference's own bf16 execution at the same positions (its
    forward over the teacher-forced sequence; its bf16 decode cannot run: the
    absorbed MLA attention gives SDPA an fp32 query and a bf16 latent cache,
    which PyTorch rejects).  Per (row, step) logits cosine to the fp32
    oracle: the mean deficit must stay within 2.25x the reference's (+1e-4)
    and no row may fall below 0.97 (a bf16 router near-tie that flips one of
    a token's two experts moves single rows to ~0.98 in the reference and
    in every decode path alike).  The decode_next token must equal the
    oracle's argmax wherever the oracle's top-2 margin exceeds twice the
    row's largest logit deviation plus the bf16 rounding of the top logit."""
    prod, orc = _pair({}, seed=0)
    ids = torch.randint(0, 32768, (batch, 128), generator=torch.Generator().manual_seed(batch))
    with torch.inference_mode():
        lp, state = prod.prefill(ids.cuda())
        _, state_next = prod.prefill(ids.cuda())
    with torch.no_grad():
        le, ostate = orc.prefill(ids)
    ours, theirs, fed = [lp[:, -1].float().cpu()], [le[:, -1].float()], []
    nxt = le.argmax(-1)
    checked = 0
    for step in range(16):
        fed.append(nxt)
        with torch.inference_mode():
            lp, state = prod.decode_step(nxt.cuda(), state)
            tok, state_next = prod.decode_next(nxt.cuda(), state_next)
        with torch.no_grad():
            le, ostate = orc.decode_step(nxt, ostate)
        ours.append(lp[:, -1].float().cpu())
        theirs.append(le[:, -1].float())
        top2 = le.float().topk(2, dim=-1).values
        dev = (lp.float().cpu() - le.float()).abs().amax(-1)
        slack = 2 * dev + top2[..., 0].abs() * 2.0 ** -7
        clear = (top2[..., 0] - top2[..., 1]) > slack
        want = le.argmax(-1)
        assert torch.equal(tok.cpu()[clear], want[clear]), step
        checked += int(clear.sum())
        nxt = want
    assert state.position == state_next.position == 128 + 16
    # the reference in bf16: logits at positions 127 .. 143 of the fed sequence
    seq = torch.cat([ids] + fed, dim=1)
    with torch.inference_mode():
        ref = _reference_bf16(orc)(seq.cuda()).logits[:, 127:].float().cpu()

    def row_cos(a, b):
        return torch.nn.functional.cosine_similarity(a.double(), b.double(), dim=-1)

    want_all = torch.stack(theirs, 1)
    c_ours = row_cos(torch.stack(ours, 1), want_all)
    c_ref = row_cos(ref, want_all)
    d_ours, d_ref = float((1 - c_ours).mean()), float((1 - c_ref).mean())
    print(f"B={batch}: mean cosine deficit {d_ours:.2e} (bf16 reference {d_ref:.2e}), "
          f"min {float(c_ours.min()):.5f} (reference {float(c_ref.min()):.5f}); greedy tokens "
          f"compared at {checked} of {16 * batch} steps")
    assert d_ours <= 2.25 * d_ref + 1e-4, (d_ours, d_ref)
    assert float(c_ours.min()) >= 0.97, float(c_ours.min())
