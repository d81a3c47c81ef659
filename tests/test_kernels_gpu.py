"""GPU parity of the sm_100a kernels against the CPU oracle, through the C ABI.

Contract: expert assignment and grouping permutation are bit-exact given
identical router probabilities; floating-point outputs match the fp32 oracle
within the bf16 tolerance of ``tests.gpu_helpers.assert_bf16_close``
(|a - e| <= 4e-2 (rms(e) + |e|) per element, rms(a - e) <= 1e-2 rms(e)); the
MoE block additionally matches the reference algorithm executed in bf16 on
the same GPU element for element.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import parrot_oracle as po
from parrot_b200 import _lib, bridge
from parrot_b200 import model as pm
from parrot_b200.workloads import tune_zipf_router_bias
from tests.gpu_helpers import (assert_bf16_close, build_moe_pair, call_moe_forward, err_stats,
                               hidden_states, moe_config, workspace_view)

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _inference():
    with torch.inference_mode():
        yield


# ---------------------------------------------------------------------------
# RMSNorm
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("rows,dim", [(1, 768), (7, 768), (512, 768), (33, 128), (5, 64),
                                      (16, 2048)])
def test_rmsnorm_matches_oracle(rows, dim):
    g = torch.Generator().manual_seed(rows * 1000 + dim)
    x = (torch.randn(rows, dim, generator=g) * 3).to(torch.bfloat16)
    w = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16)
    norm = pm.RMSNorm(dim, 1e-6)
    norm.weight.data.copy_(w.float())
    norm = norm.to("cuda", torch.bfloat16)
    out = norm(x.cuda()).cpu()
    ref = po.RMSNorm(dim, 1e-6)
    ref.weight.data.copy_(w.float())
    exp = ref(x.float())
    assert_bf16_close(out, exp, "rmsnorm")
    # bf16 reference semantics: one rounding of the fp32 result
    diff = (out.float() - exp.to(torch.bfloat16).float()).abs()
    assert float(diff.max()) <= float(exp.abs().max()) * 2 ** -7


@pytest.mark.parametrize("n_sources,rows,base", [(3, 512, True), (1, 37, False), (6, 64, True)])
def test_depth_mix_with_deferred_moe_combine(n_sources, rows, base):
    """parrot_depthmix_moe_bf16 == the combine kernel's arithmetic
    bf16(base + bf16(bf16(shared + c_lo) + c_hi)) as the last source, then the
    plain depth mix (which the other tests pin to the oracle)."""
    dim = 768
    g = torch.Generator().manual_seed(rows + n_sources)
    rnd = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16).cuda()
    srcs = [rnd(rows, dim) for _ in range(n_sources - 1)]
    shared, contrib = rnd(rows, dim), rnd(2 * rows, dim) * 0.5
    b = rnd(rows, dim) if base else None
    q, kw, ow = rnd(dim) * 0.5, 1 + 0.2 * rnd(dim), 1 + 0.2 * rnd(dim)
    lib = _lib.load()
    out = torch.empty(rows, dim, device="cuda", dtype=torch.bfloat16)
    value = torch.empty_like(out)
    ptrs = (ctypes.c_void_p * n_sources)(*([s.data_ptr() for s in srcs] + [value.data_ptr()]))
    _lib.check(lib.parrot_depthmix_moe_bf16(
        out.data_ptr(), ptrs, n_sources, q.data_ptr(), kw.data_ptr(), 1e-6, ow.data_ptr(), 1e-6,
        None, None if b is None else b.data_ptr(), shared.data_ptr(), contrib.data_ptr(),
        value.data_ptr(), rows, dim, bridge._stream()), "parrot_depthmix_moe_bf16")
    moe = ((shared.float() + contrib[0::2].float()).to(torch.bfloat16).float()
           + contrib[1::2].float()).to(torch.bfloat16)
    want_value = moe if b is None else (b.float() + moe.float()).to(torch.bfloat16)
    want = torch.empty_like(out)
    all_srcs = srcs + [want_value]
    ptrs2 = (ctypes.c_void_p * n_sources)(*[s.data_ptr() for s in all_srcs])
    _lib.check(lib.parrot_depthmix_bf16(
        want.data_ptr(), ptrs2, n_sources, q.data_ptr(), kw.data_ptr(), 1e-6, ow.data_ptr(), 1e-6,
        None, None, None, None, rows, dim, bridge._stream()), "parrot_depthmix_bf16")
    torch.cuda.synchronize()
    assert torch.equal(value, want_value)
    assert torch.equal(out, want)


# ---------------------------------------------------------------------------
# SiLU of the SwiGLU epilogue, every bf16 input
# ---------------------------------------------------------------------------
def test_silu_matches_pytorch_bf16_for_every_input():
    """parrot_silu_bf16 runs the epilogue's SiLU (fast path + table fallback);
    it must equal F.silu on a bf16 tensor (parrot/model.py:448) bit for bit
    for all 65,536 bf16 bit patterns (NaNs: NaN in both)."""
    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16)
    x = bits.view(torch.bfloat16).cuda()
    y = torch.empty_like(x)
    _lib.check(_lib.load().parrot_silu_bf16(x.data_ptr(), y.data_ptr(), x.numel(),
                                            bridge._stream()), "parrot_silu_bf16")
    want = torch.nn.functional.silu(x)
    torch.cuda.synchronize()
    nan = torch.isnan(want)
    assert torch.equal(torch.isnan(y), nan)
    same = y.view(torch.int16) == want.view(torch.int16)
    assert bool(same[~nan].all()), x[~nan & ~same][:8].float().tolist()


# ---------------------------------------------------------------------------
# Block AttnRes depth mix (+ consumer RMSNorm, + deferred residual)
# ---------------------------------------------------------------------------
def _depth_modules(dim, seed, q_std=0.5):
    g = torch.Generator().manual_seed(seed)
    q = (q_std * torch.randn(dim, generator=g)).to(torch.bfloat16).float()
    kw = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).float()
    ow = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).float()
    cfg = moe_config(dim=dim if dim % 128 == 0 else 128)
    prod = pm.DepthMix(cfg) if dim == cfg.dim else None
    ocfg = po.OracleConfig(dim=dim)
    orc = po.DepthMix(ocfg)
    orc.query.data.copy_(q)
    orc.norm.weight.data.copy_(kw)
    onorm = po.RMSNorm(dim, 1e-6)
    onorm.weight.data.copy_(ow)
    return prod, orc, onorm, (q, kw, ow)


def _sources(n, rows, dim, seed):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(rows, dim, generator=g) * (1 + i)).to(torch.bfloat16) for i in range(n)]


@pytest.mark.parametrize("n_sources", [1, 2, 5, 9, 16])
@pytest.mark.parametrize("rows", [1, 7, 512])
@pytest.mark.parametrize("q_std", [0.05, 0.5])
def test_depth_mix_norm_matches_oracle(n_sources, rows, q_std):
    """q_std 0.5 makes the source softmax nearly one-hot (scores ~ N(0, 14^2))."""
    dim = 768
    prod, orc, onorm, (q, kw, ow) = _depth_modules(dim, n_sources + rows, q_std)
    prod.query.data.copy_(q)
    prod.norm.weight.data.copy_(kw)
    prod = prod.to("cuda", torch.bfloat16)
    pnorm = pm.RMSNorm(dim, 1e-6)
    pnorm.weight.data.copy_(ow)
    pnorm = pnorm.to("cuda", torch.bfloat16)
    srcs = _sources(n_sources, rows, dim, 7 * rows + n_sources)
    got_mix = prod([s.cuda() for s in srcs]).cpu()
    got = prod.normalized([s.cuda() for s in srcs], pnorm).cpu()
    exp_mix = orc([s.float() for s in srcs])
    exp = onorm(exp_mix)
    assert_bf16_close(got_mix, exp_mix, "mix")
    assert_bf16_close(got, exp, "mix+norm")
    if q_std < 0.1:
        # with a soft mixture the oracle run in bf16 (the reference's CUDA dtype),
        # which rounds keys and weights to bf16, agrees as well
        orc_b = orc.to(torch.bfloat16)
        onorm_b = onorm.to(torch.bfloat16)
        exp_b = onorm_b(orc_b(srcs))
        assert_bf16_close(got, exp_b, "vs bf16 oracle")


def test_depth_mix_pending_residual_resolves_the_add():
    dim, rows = 768, 64
    prod, orc, onorm, (q, kw, ow) = _depth_modules(dim, 3)
    prod.query.data.copy_(q)
    prod.norm.weight.data.copy_(kw)
    prod = prod.to("cuda", torch.bfloat16)
    pnorm = pm.RMSNorm(dim, 1e-6)
    pnorm.weight.data.copy_(ow)
    pnorm = pnorm.to("cuda", torch.bfloat16)
    srcs = _sources(4, rows, dim, 11)
    delta = _sources(1, rows, dim, 12)[0]
    resolved_ref = (srcs[-1].cuda() + delta.cuda())
    got, resolved = prod.normalized([s.cuda() for s in srcs], pnorm, delta.cuda())
    assert torch.equal(resolved, resolved_ref)
    plain = prod.normalized([s.cuda() for s in srcs[:-1]] + [resolved_ref], pnorm)
    assert torch.equal(got, plain)


@pytest.mark.parametrize("mode,pos,batch", [("local", 0, 1), ("local", 31, 1), ("local", 32, 1),
                                            ("local", 127, 3), ("local", 128, 2), ("local", 2300, 2),
                                            ("local", 1000, 64), ("local", 2300, 64), ("mla", 0, 1),
                                            ("mla", 5, 2), ("mla", 700, 1), ("mla", 900, 64)])
def test_decode_attention_matches_sdpa(mode, pos, batch):
    """parrot_decode_attention_bf16 at XL shapes against PyTorch SDPA on the
    same cache contents: local GQA (8 heads x 96 over 2 KV heads, window
    2048) and absorbed MLA (fp32 query over the 128-wide latent); one chunk
    (finished in one CTA), chunk edges, the window edge, and batch 64 (four
    CTAs per group, each looping over chunks)."""
    g = torch.Generator().manual_seed(pos + batch)
    S = 4096
    position = torch.full((1,), pos, device="cuda", dtype=torch.int32)
    if mode == "local":
        H, KVH, D, window = 8, 2, 96, 2048
        kc = torch.randn(batch, KVH, S, D, generator=g).to("cuda", torch.bfloat16)
        vc = torch.randn(batch, KVH, S, D, generator=g).to("cuda", torch.bfloat16)
        qkv = torch.randn(batch, (H + 2 * KVH) * D, generator=g).to("cuda", torch.bfloat16)
        qw, kw = H * D, KVH * D
        q, kn, vn = qkv[:, :qw], qkv[:, qw:qw + kw], qkv[:, qw + kw:]
        out = bridge.b200_decode_attention(q, kn, vn, kc, vc, position, H, KVH, D, window,
                                           D ** -0.5, torch.bfloat16)
        # a second call (the arrival counters were reset) gives the same bits
        assert torch.equal(out, bridge.b200_decode_attention(
            q, kn, vn, kc, vc, position, H, KVH, D, window, D ** -0.5, torch.bfloat16))
        assert torch.equal(kc[:, :, pos], kn.view(batch, KVH, D))
        assert torch.equal(vc[:, :, pos], vn.view(batch, KVH, D))
        lo = max(0, pos - window + 1)
        ref = torch.nn.functional.scaled_dot_product_attention(
            q.view(batch, H, 1, D).float(), kc[:, :, lo:pos + 1].float(),
            vc[:, :, lo:pos + 1].float(), enable_gqa=True).view(batch, H * D)
        torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    else:
        H, L, hd = 8, 128, 96
        lat = torch.randn(batch, S, L, generator=g).to("cuda", torch.bfloat16)
        q = (0.1 * torch.randn(batch, H * L, generator=g)).to("cuda")
        new = torch.randn(batch, L, generator=g).to("cuda", torch.bfloat16)
        out = bridge.b200_decode_attention(q, new, None, lat.unsqueeze(1), None, position, H, 1,
                                           L, 0, hd ** -0.5, torch.float32)
        assert torch.equal(out, bridge.b200_decode_attention(
            q, new, None, lat.unsqueeze(1), None, position, H, 1, L, 0, hd ** -0.5, torch.float32))
        assert torch.equal(lat[:, pos], new)
        seen = lat[:, :pos + 1].float()[:, None].expand(-1, H, -1, -1)
        ref = torch.nn.functional.scaled_dot_product_attention(
            q.view(batch, H, 1, L), seen, seen, scale=hd ** -0.5).view(batch, H * L)
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("rows", [1, 3, 8])
@pytest.mark.parametrize("n,k,xt,wt,yt", [
    (1152, 768, torch.bfloat16, torch.bfloat16, torch.bfloat16),  # local qkv
    (768, 768, torch.bfloat16, torch.bfloat16, torch.bfloat16),   # local out
    (128, 768, torch.bfloat16, torch.bfloat16, torch.bfloat16),   # MLA latent down
    (1024, 768, torch.bfloat16, torch.float32, torch.float32),    # absorbed query
    (768, 1024, torch.float32, torch.float32, torch.bfloat16),    # absorbed output
])
def test_linear_small_matches_fp64(rows, n, k, xt, wt, yt):
    """parrot_linear_small (decode projections) against the fp64 product of
    the same operands: fp32 accumulation, one rounding to the output type."""
    g = torch.Generator().manual_seed(rows * 7 + n + k)
    x = torch.randn(rows, k, generator=g).to("cuda", xt)
    w = (0.05 * torch.randn(n, k, generator=g)).to("cuda", wt)
    with torch.inference_mode():
        y = bridge.b200_linear_small(x, w, yt)
    assert y.dtype == yt and y.shape == (rows, n)
    ref = x.double() @ w.double().T
    if yt == torch.bfloat16:
        # within one bf16 rounding of the exact value (fp32 accumulation error is far smaller)
        err = (y.double() - ref).abs()
        assert bool((err <= ref.abs() * 2.0 ** -8 + 1e-6).all())
    else:
        torch.testing.assert_close(y.double(), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("pos,batch", [(0, 1), (135, 1), (31, 3), (2300, 2), (700, 64)])
def test_decode_attention_rope_fused_is_bit_identical(pos, batch):
    """parrot_decode_attention_rope_bf16 (RoPE of q and the new key inside the
    kernel) against parrot_rope_inplace_at_bf16 followed by
    parrot_decode_attention_bf16: same output bits, same appended cache rows,
    and the projection left unrotated."""
    g = torch.Generator().manual_seed(1000 + pos + batch)
    S, H, KVH, D, window = 4096, 8, 2, 96, 2048
    position = torch.full((1,), pos, device="cuda", dtype=torch.int32)
    angle = torch.arange(S).float()[:, None] * (10000.0 ** -(torch.arange(0, D, 2).float() / D))
    cos, sin = angle.cos().to("cuda", torch.bfloat16), angle.sin().to("cuda", torch.bfloat16)
    kc = torch.randn(batch, KVH, S, D, generator=g).to("cuda", torch.bfloat16)
    vc = torch.randn(batch, KVH, S, D, generator=g).to("cuda", torch.bfloat16)
    qkv = torch.randn(batch, 1, (H + 2 * KVH) * D, generator=g).to("cuda", torch.bfloat16)
    qw, kw = H * D, KVH * D
    raw = qkv.clone()
    kc2, vc2 = kc.clone(), vc.clone()
    flat = qkv.view(batch, -1)
    fused = bridge.b200_decode_attention(flat[:, :qw], flat[:, qw:qw + kw], flat[:, qw + kw:],
                                         kc, vc, position, H, KVH, D, window, D ** -0.5,
                                         torch.bfloat16, rope=(cos, sin))
    assert torch.equal(qkv, raw)
    bridge.b200_rope_at_(qkv, cos, sin, H + KVH, D, position)
    flat = qkv.view(batch, -1)
    plain = bridge.b200_decode_attention(flat[:, :qw], flat[:, qw:qw + kw], flat[:, qw + kw:],
                                         kc2, vc2, position, H, KVH, D, window, D ** -0.5,
                                         torch.bfloat16)
    assert torch.equal(fused, plain)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)


@pytest.mark.parametrize("tokens,residual,zipf", [(1, False, False), (3, True, False),
                                                   (8, True, True), (16, False, True)])
def test_decode_moe_matches_oracle_and_gemm_path(tokens, residual, zipf):
    """parrot_moe_decode_bf16 (small-batch path): routing equal to the oracle's
    wherever its margin is resolvable, output within the bf16 contract of the
    fp32 oracle and equal (bar accumulation-order rounding) to the
    tensor-core path."""
    cfg = moe_config()
    prod, orc = build_moe_pair(cfg, seed=60 + tokens)
    x = hidden_states(tokens, cfg.dim, seed=61 + tokens)
    if zipf:
        bias = torch.tensor([3.0, 2.0] + [0.0] * (cfg.n_experts - 2))
        prod.router_bias = bias.cuda()
        orc.router_bias = bias
    res = hidden_states(tokens, cfg.dim, seed=62) if residual else None
    xd = x.cuda()
    got, _, _ = bridge.b200_moe(prod, xd, False, None if res is None else res.cuda())
    dims = bridge._block_dims(cfg, tokens)  # the workspace the block ran in
    layout = bridge.workspace_layout(dims)
    ws = bridge.workspace(xd.device, dims)
    idx = workspace_view(ws, layout, "indices", torch.int32, (tokens, 2)).cpu().long()
    w = workspace_view(ws, layout, "weights", torch.float32, (tokens, 2)).cpu()
    exp, _, _ = orc(x.float())
    if res is not None:
        exp = res.float() + exp
    trace = orc.last_trace
    top3 = trace.probabilities.topk(3, dim=-1).values
    clear = torch.minimum(top3[:, 0] - top3[:, 1], top3[:, 1] - top3[:, 2]) > 1e-5
    assert torch.equal(idx[clear], trace.indices[clear])
    torch.testing.assert_close(w[clear], trace.weights[clear], rtol=1e-5, atol=1e-6)
    assert_bf16_close(got, exp, "decode moe vs fp32 oracle")
    # the tensor-core path on the same rows (stats on: it does not take the decode path)
    gemm, _, _ = bridge.b200_moe(prod, xd, True, None if res is None else res.cuda())
    st = err_stats(got, gemm)
    assert st["rms_rel"] < 1e-2 and st["mixed"] < 2e-2, st


# ---------------------------------------------------------------------------
# Router, grouping and the whole MoE block
# ---------------------------------------------------------------------------
def _check_routing(ex, module_cfg, oracle_trace, T):
    probs = ex["probs"].float().cpu()
    idx = ex["indices"].cpu()
    # bit-exact selection given the kernel's own probabilities (ties flagged)
    top3 = probs.topk(min(3, module_cfg.n_experts), dim=-1)
    ties = (top3.values[:, 0] == top3.values[:, 1]).sum()
    if module_cfg.n_experts > 2:
        ties += (top3.values[:, 1] == top3.values[:, 2]).sum()
    assert int(ties) == 0, "exact ties in the test inputs"
    np.testing.assert_array_equal(idx.numpy(), probs.topk(2, dim=-1).indices.numpy())
    w = ex["weights"].cpu()
    sel = probs.gather(1, idx)
    torch.testing.assert_close(w, sel / sel.sum(-1, keepdim=True), rtol=0, atol=0)
    # against the oracle's own routing: equal wherever its decision margin is resolvable
    op = oracle_trace.probabilities
    torch.testing.assert_close(probs, op, rtol=1e-4, atol=1e-6)
    margin = torch.minimum(op.topk(3, dim=-1).values[:, 1] - op.topk(3, dim=-1).values[:, 2],
                           op.topk(2, dim=-1).values[:, 0] - op.topk(2, dim=-1).values[:, 1]) \
        if module_cfg.n_experts > 2 else torch.ones(T)
    clear = margin > 1e-5
    np.testing.assert_array_equal(idx[clear].numpy(), oracle_trace.indices[clear].numpy())
    # grouping: stable counting sort of the kernel's indices, exactly
    grouping = po.group_assignments(idx.numpy(), module_cfg.n_experts)
    rows = po.grouped_rows(grouping, idx.numpy())
    np.testing.assert_array_equal(ex["positions"].cpu().numpy(), np.array(rows, dtype=np.int32))
    np.testing.assert_array_equal(ex["counts"].cpu().numpy(), np.array(grouping.counts))
    return grouping


@pytest.mark.parametrize("tokens,zipf", [(8192, False), (16384, True)])
def test_xl_moe_layer_large_batch_matches_oracle(tokens, zipf):
    """Large batches (128-token router tiles streamed through the router's
    4-slot ring; with the skewed bias, the capacity-overflow path): routing,
    grouping, statistics and output against the fp32 oracle."""
    cfg = moe_config()
    prod, orc = build_moe_pair(cfg, seed=2)
    x = hidden_states(tokens, cfg.dim, seed=3)
    if zipf:
        bias = torch.tensor([3.0, 2.0, 1.0] + [0.0] * (cfg.n_experts - 3))
        prod.router_bias = bias.cuda()
        orc.router_bias = bias
    out, ex, ws, layout = call_moe_forward(prod, x.cuda())
    assert ex["status"][0] == 0, ex["status"]
    exp, aux, util = orc(x.float())
    _check_routing(ex, cfg, orc.last_trace, tokens)
    if zipf:
        assert int(ex["counts"].max()) > layout.capacity  # the overflow path ran
    assert_bf16_close(out, exp, "large-batch moe vs fp32 oracle")
    stats = ex["stats"].cpu()
    torch.testing.assert_close(stats[:-1], util, rtol=0, atol=2.0 / (2 * tokens))
    torch.testing.assert_close(stats[-1], aux, rtol=2e-3, atol=1e-6)
    grouped = workspace_view(ws, layout, "grouped", torch.bfloat16,
                             (layout.grouped_rows, cfg.dim)).cpu()
    pos = ex["positions"].cpu().long()
    tok = torch.arange(2 * tokens) // 2
    assert torch.equal(grouped[pos], x[tok])


@pytest.mark.parametrize("tokens", [256, 512])
def test_xl_moe_layer_matches_oracle(tokens):
    cfg = moe_config()
    prod, orc = build_moe_pair(cfg, seed=1)
    x = hidden_states(tokens, cfg.dim, seed=0)
    out, ex, ws, layout = call_moe_forward(prod, x.cuda())
    assert ex["status"][0] == 0, ex["status"]
    exp, aux, util = orc(x.float())
    _check_routing(ex, cfg, orc.last_trace, tokens)
    assert_bf16_close(out, exp, "moe vs fp32 oracle")
    # the reference algorithm executed in bf16 on this GPU (torch CUDA ops)
    ref_b, _, _ = orc.to("cuda", torch.bfloat16)(x.cuda())
    same = (out == ref_b).float().mean()
    assert float(same) >= 0.999, float(same)
    assert err_stats(out, ref_b)["mixed"] <= 2 ** -7
    stats = ex["stats"].cpu()
    own = torch.bincount(ex["indices"].cpu().flatten(), minlength=cfg.n_experts).float() / (2 * tokens)
    torch.testing.assert_close(stats[:-1], own, rtol=0, atol=0)
    torch.testing.assert_close(stats[:-1], util, rtol=0, atol=2.0 / (2 * tokens))
    torch.testing.assert_close(stats[-1], aux, rtol=2e-3, atol=1e-6)
    # every assignment's token row was scattered to its grouped row
    grouped = workspace_view(ws, layout, "grouped", torch.bfloat16,
                             (layout.grouped_rows, cfg.dim)).cpu()
    pos = ex["positions"].cpu().long()
    tok = torch.arange(2 * tokens) // 2
    assert torch.equal(grouped[pos], x[tok])


def test_xl_moe_layer_intermediates_match_oracle_experts():
    """gate_up+SwiGLU and down GEMM outputs, per grouped row, vs the oracle experts."""
    cfg = moe_config()
    T = 256
    prod, orc = build_moe_pair(cfg, seed=1)
    x = hidden_states(T, cfg.dim, seed=0)
    out, ex, ws, layout = call_moe_forward(prod, x.cuda())
    R = layout.grouped_rows
    hidden = workspace_view(ws, layout, "hidden", torch.bfloat16, (R, cfg.expert_dim)).cpu()
    contrib = workspace_view(ws, layout, "contrib", torch.bfloat16, (2 * T, cfg.dim)).cpu()
    sh = workspace_view(ws, layout, "shared_hidden", torch.bfloat16, (T, cfg.shared_expert_dim)).cpu()
    sy = workspace_view(ws, layout, "shared_y", torch.bfloat16, (T, cfg.dim)).cpu()
    idx = ex["indices"].cpu()
    pos = ex["positions"].cpu().long()
    w = ex["weights"].cpu()
    xf = x.float()
    # contribution slot of assignment a = 2t + (0 if its expert is the token's lower id)
    other = idx.flip(-1).flatten()
    slot = (torch.arange(2 * T) & ~1) + (idx.flatten() > other).long()
    for e in range(cfg.n_experts):
        a = torch.nonzero(idx.flatten() == e).flatten()
        if a.numel() == 0:
            continue
        tokens = a // 2
        ex_mod = orc.experts[e]
        g = ex_mod.gate(xf[tokens])
        u = ex_mod.up(xf[tokens])
        h_ref = torch.nn.functional.silu(g) * u
        assert_bf16_close(hidden[pos[a]], h_ref, f"hidden e{e}")
        y_ref = ex_mod.down(hidden[pos[a]].float()) * w.flatten()[a, None]
        assert_bf16_close(contrib[slot[a]], y_ref, f"contribution e{e}")
    hs_ref = torch.nn.functional.silu(orc.shared.gate(xf)) * orc.shared.up(xf)
    assert_bf16_close(sh, hs_ref, "shared hidden")
    assert_bf16_close(sy, orc.shared.down(sh.float()), "shared y")


@pytest.mark.parametrize("tokens,experts,dim,hidden,shared", [
    (1, 16, 768, 512, 256), (2, 16, 768, 512, 256), (7, 4, 128, 64, 64),
    (33, 2, 128, 128, 64), (100, 32, 256, 128, 128), (130, 8, 128, 192, 64),
])
def test_moe_edge_shapes(tokens, experts, dim, hidden, shared):
    cfg = moe_config(dim=dim, n_experts=experts, expert_dim=hidden, shared_dim=shared)
    prod, orc = build_moe_pair(cfg, seed=tokens + experts)
    x = hidden_states(tokens, dim, seed=tokens)
    out, ex, _, _ = call_moe_forward(prod, x.cuda())
    assert ex["status"][0] == 0, ex["status"]
    exp, _, _ = orc(x.float())
    _check_routing(ex, cfg, orc.last_trace, tokens)
    assert_bf16_close(out, exp, "edge shape")


@pytest.mark.parametrize("capacity", [8, 16, 40])
def test_forced_overflow_is_exact(capacity):
    """Tiny capacities push most assignments through the overflow segments."""
    cfg = moe_config(dim=256, n_experts=8, expert_dim=128, shared_dim=64)
    prod, orc = build_moe_pair(cfg, seed=5)
    T = 300
    x = hidden_states(T, cfg.dim, seed=9)
    out, ex, ws, layout = call_moe_forward(prod, x.cuda(), capacity=capacity)
    assert ex["status"][0] == 0, ex["status"]
    counts = ex["counts"].cpu()
    assert int((counts - capacity).clamp_min(0).sum()) > 0
    exp, _, _ = orc(x.float())
    idx = ex["indices"].cpu()
    grouping = po.group_assignments(idx.numpy(), cfg.n_experts, capacity=capacity)
    rows = po.grouped_rows(grouping, idx.numpy())
    np.testing.assert_array_equal(ex["positions"].cpu().numpy(), np.array(rows, dtype=np.int32))
    assert_bf16_close(out, exp, "forced overflow")


def test_zipf_skew_overflow_matches_oracle():
    """BASELINE config-4 routing skew (Zipf 1.2 over 16 experts) at 2048 tokens."""
    cfg = moe_config()
    prod, orc = build_moe_pair(cfg, seed=1)
    T = 2048
    x = hidden_states(T, cfg.dim, seed=0)
    bias = tune_zipf_router_bias(x.float(), orc.router.weight.detach())
    prod.router_bias = bias
    orc.router_bias = bias
    out, ex, _, layout = call_moe_forward(prod, x.cuda())
    assert ex["status"][0] == 0, ex["status"]
    counts = ex["counts"].cpu()
    assert int(counts.max()) > layout.capacity  # the overflow path ran
    exp, _, _ = orc(x.float())
    _check_routing(ex, cfg, orc.last_trace, T)
    assert_bf16_close(out, exp, "zipf")


PARTNER_BIAS = [0.9, 0.6, 0.45, 0.3, 0.15] + [0.0] * 11


def _primary_partners(counts, capacity: int, bn: int) -> set:
    """Which primary-partner cases the grouped GEMM meets (its rule, restated):
    1 = expert e's capacity segment has exactly two token tiles, 2 = it has one
    and its overflow fits one."""
    kinds = set()
    for c in counts:
        rows, over = (min(c, capacity), max(c - capacity, 0)) if capacity > 0 else (c, 0)
        if rows > bn:
            kinds.add(1 if rows <= 2 * bn else 0)
        else:
            kinds.add(2 if 0 < over <= bn else 0)
    return kinds


@pytest.mark.parametrize("tokens,capacity,kinds", [
    (512, 0, {2}), (512, 96, {2}), (512, 200, {1}), (512, -1, {1}),
    (4096, 200, {2}), (4096, 384, {1}),
])
def test_gemm_primary_partner_tiles(tokens, capacity, kinds):
    """A primary CTA takes the expert's second token tile, or its overflow
    segment, into its own K loop (the other TMEM accumulator).  Skewed routing
    at T = 512 (128-token tiles) and T = 4096 (256-token tiles of the down
    GEMM) under capacities that produce both kinds: the output matches the
    oracle and is bit-identical across capacities (the same products, tiled
    differently)."""
    cfg = moe_config()
    prod, orc = build_moe_pair(cfg, seed=4)
    x = hidden_states(tokens, cfg.dim, seed=6)
    bias = torch.tensor(PARTNER_BIAS)
    prod.router_bias = bias.cuda()
    orc.router_bias = bias
    out, ex, _, layout = call_moe_forward(prod, x.cuda(), capacity=capacity)
    assert ex["status"][0] == 0, ex["status"]
    bn = 256 if 2 * tokens >= 4096 else 128  # the launch's token tile
    got = _primary_partners(ex["counts"].cpu().tolist(), layout.capacity if capacity != -1 else 0,
                            bn)
    assert kinds <= got, (got, ex["counts"].cpu().tolist())
    exp, _, _ = orc(x.float())
    assert_bf16_close(out, exp, f"partner tiles T={tokens} C={capacity}")
    packed, _, _, _ = call_moe_forward(prod, x.cuda(), capacity=-1 if capacity != -1 else 0)
    assert torch.equal(out, packed)


@pytest.mark.parametrize("tokens,experts,zipf", [
    (37, 16, False), (256, 16, False), (512, 16, False), (1024, 16, False), (2048, 16, False),
    (4096, 16, False), (100, 32, False), (130, 8, False), (8192, 16, False), (16384, 16, True)])
def test_slot_mode_grouping_equals_the_group_kernel(tokens, experts, zipf):
    """Slot mode (capacity -2: a 2T-row region per expert): the router takes each assignment's slot with an
    atomic and copies the row, no group kernel runs.  Against the default
    capacity layout (the group kernel): the block output, counts and
    statistics are bit-identical; each expert's positions fill its region and
    every grouped row holds its token's row; a second call (the counters were
    left at zero) repeats the output."""
    cfg = moe_config(n_experts=experts) if experts == 16 else \
        moe_config(dim=256, n_experts=experts, expert_dim=128, shared_dim=128)
    prod, _ = build_moe_pair(cfg, seed=experts + tokens)
    x = hidden_states(tokens, cfg.dim, seed=tokens).cuda()
    if zipf:  # above 4096 tokens the tensor-core router; skewed, the overflow path on the left
        prod.router_bias = torch.tensor([3.0, 2.0, 1.0] + [0.0] * (experts - 3)).cuda()
    ref, ex_ref, _, _ = call_moe_forward(prod, x)
    out, ex, ws, layout = call_moe_forward(prod, x, capacity=-2)
    assert ex["status"][0] == 0, ex["status"]
    assert layout.capacity == 2 * tokens
    assert torch.equal(out, ref)
    for k in ("indices", "weights", "counts", "stats"):
        assert torch.equal(ex[k], ex_ref[k]), k
    C = layout.capacity
    cnt, pos, idx = ex["counts"].cpu(), ex["positions"].cpu().long(), ex["indices"].cpu().flatten()
    for e in range(cfg.n_experts):
        got = torch.sort(pos[idx == e]).values
        assert torch.equal(got, e * C + torch.arange(int(cnt[e]))), e
    grouped = workspace_view(ws, layout, "grouped", torch.bfloat16,
                             (layout.grouped_rows, cfg.dim)).cpu()
    assert torch.equal(grouped[pos], x.cpu()[torch.arange(2 * tokens) // 2])
    again, _, _, _ = call_moe_forward(prod, x, capacity=-2)
    assert torch.equal(again, ref)


def test_residual_is_fused_into_combine():
    cfg = moe_config()
    prod, orc = build_moe_pair(cfg, seed=2)
    x = hidden_states(64, cfg.dim, seed=4).cuda()
    r = hidden_states(64, cfg.dim, seed=5).cuda()
    plain, _, _, _ = call_moe_forward(prod, x)
    fused, _, _, _ = call_moe_forward(prod, x, residual=r)
    assert torch.equal(fused, (r + plain))


def test_moe_is_deterministic():
    cfg = moe_config()
    prod, _ = build_moe_pair(cfg, seed=3)
    x = hidden_states(512, cfg.dim, seed=1).cuda()
    a, ea, _, _ = call_moe_forward(prod, x)
    b, eb, _, _ = call_moe_forward(prod, x)
    assert torch.equal(a, b)
    for k in ("indices", "positions", "counts", "weights"):
        assert torch.equal(ea[k], eb[k]), k


def test_zero_tokens_is_a_no_op():
    cfg = moe_config()
    prod, _ = build_moe_pair(cfg, seed=3)
    x = torch.empty(0, cfg.dim, device="cuda", dtype=torch.bfloat16)
    out, _, _ = bridge.b200_moe(prod, x, True)
    assert out.shape == (0, cfg.dim)


def test_route_then_experts_equals_fused():
    cfg = moe_config()
    prod, orc = build_moe_pair(cfg, seed=6)
    x = hidden_states(200, cfg.dim, seed=2).cuda()
    probs, w, idx, pos, counts = bridge.b200_route(prod, x, True)
    staged = bridge.b200_experts(prod, x, idx, w, pos, counts)
    fused, _, _ = bridge.b200_moe(prod, x, False)
    assert torch.equal(staged, fused)
    assert idx.dtype == torch.int64 and pos.dtype == torch.int32
    with pytest.raises(ValueError):
        bridge.b200_experts(prod, x.clone(), idx, w, pos, counts)


def test_large_token_count_tensor_core_path():
    """T = 4096: many token tiles per expert; checked through size-independent
    properties plus sampled rows against the oracle."""
    cfg = moe_config()
    prod, orc = build_moe_pair(cfg, seed=7)
    T = 4096
    x = hidden_states(T, cfg.dim, seed=3)
    out, ex, ws, layout = call_moe_forward(prod, x.cuda(), want_probs=True)
    assert ex["status"][0] == 0
    counts = ex["counts"].cpu()
    assert int(counts.sum()) == 2 * T
    sample = torch.arange(0, T, 61)
    exp, _, _ = orc(x.float()[sample])
    assert_bf16_close(out.cpu()[sample], exp, "T=4096 sample")


# ---------------------------------------------------------------------------
# Rotary embedding (local attention q/k)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("batch,seq,start", [(1, 512, 0), (3, 37, 0), (2, 1, 700)])
def test_rope_inplace_is_bit_exact_to_reference_bf16(batch, seq, start):
    from parrot_b200.model import _rope_tables
    cfg = po.OracleConfig()
    H, KV, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    g = torch.Generator().manual_seed(seq + start)
    qkv = torch.randn(batch, seq, (H + 2 * KV) * hd, generator=g).to("cuda", torch.bfloat16)
    qw, kw = H * hd, KV * hd
    # the oracle's rotation evaluated in bf16 (the reference's expression)
    q_ref = po._apply_rope(cfg, qkv[..., :qw].view(batch, seq, H, hd).transpose(1, 2), start)
    k_ref = po._apply_rope(cfg, qkv[..., qw:qw + kw].view(batch, seq, KV, hd).transpose(1, 2),
                           start)
    v_ref = qkv[..., qw + kw:].clone()
    cos, sin = _rope_tables(moe_config(), qkv.device, qkv.dtype)
    bridge.b200_rope_(qkv, cos, sin, H + KV, hd, start)
    assert torch.equal(qkv[..., :qw].view(batch, seq, H, hd).transpose(1, 2), q_ref)
    assert torch.equal(qkv[..., qw:qw + kw].view(batch, seq, KV, hd).transpose(1, 2), k_ref)
    assert torch.equal(qkv[..., qw + kw:], v_ref)


# ---------------------------------------------------------------------------
# Greedy next token: LM-head projection fused with the vocabulary argmax
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("rows,dim", [(1, 768), (2, 768), (3, 768), (5, 768), (8, 768),
                                      (9, 768), (64, 768), (3, 128), (8, 1024)])
def test_vocab_argmax_matches_linear_argmax(rows, dim):
    """decode_next's F.linear(h, W).argmax(-1) (model.py:927-931).  The fused
    kernel (<= 8 rows) and the GEMM + row-argmax path (> 8) must pick a token
    whose exact logit is a maximum up to bf16 rounding of the logits, and the
    very token torch picks wherever the exact top-2 margin exceeds that
    rounding."""
    vocab = 32768
    g = torch.Generator().manual_seed(100 + rows)
    w = (torch.randn(vocab, dim, generator=g) * 0.02).to(torch.bfloat16)
    h = torch.randn(rows, 1, dim, generator=g).to(torch.bfloat16)
    got = bridge.b200_vocab_argmax(h.cuda(), w.cuda())
    want = torch.nn.functional.linear(h.cuda(), w.cuda()).argmax(-1)
    torch.cuda.synchronize()
    assert got.shape == (rows, 1) and got.dtype == torch.int64
    exact = h.double().reshape(rows, dim) @ w.double().t()
    top2 = exact.topk(2, dim=-1).values
    ulp = 2.0 ** (torch.floor(torch.log2(top2[:, 0].abs())) - 7)  # bf16 spacing at the max
    got_c = got.cpu().reshape(rows)
    picked = exact.gather(1, got_c[:, None]).squeeze(1)
    assert (picked >= top2[:, 0] - 2 * ulp).all()
    clear = (top2[:, 0] - top2[:, 1]) > 2 * ulp
    assert clear.sum() >= rows // 2
    assert torch.equal(got_c[clear], exact.argmax(-1)[clear])
    assert torch.equal(got_c[clear], want.cpu().reshape(rows)[clear])


@pytest.mark.parametrize("rows", [1, 4, 16])
def test_vocab_argmax_ties_go_to_the_lowest_index(rows):
    vocab, dim = 32768, 768
    g = torch.Generator().manual_seed(7)
    w = (torch.randn(vocab, dim, generator=g) * 0.02).to(torch.bfloat16)
    h = torch.randn(rows, 1, dim, generator=g).to(torch.bfloat16)
    hot = (h[0, 0].float() * 0.5).to(torch.bfloat16)  # one row far above the rest, copied thrice
    for v in (30001, 100, 5000):
        w[v] = hot
    h[:] = h[0]
    got = bridge.b200_vocab_argmax(h.cuda(), w.cuda())
    torch.cuda.synchronize()
    assert got.cpu().reshape(rows).tolist() == [100] * rows


def test_vocab_argmax_is_repeatable_and_graph_capturable():
    vocab, dim = 32768, 768
    g = torch.Generator().manual_seed(9)
    w = (torch.randn(vocab, dim, generator=g) * 0.02).to(torch.bfloat16).cuda()
    h = torch.randn(4, 1, dim, generator=g).to(torch.bfloat16).cuda()
    first = bridge.b200_vocab_argmax(h, w)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        static = bridge.b200_vocab_argmax(h, w)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(static, first)


# ---------------------------------------------------------------------------
# The router folded into the depth mix that produces the MoE input
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("rows,n_sources,pending,slots", [
    (512, 6, True, False), (37, 3, False, False), (4096, 9, True, False), (9, 1, False, False),
    (512, 6, True, True), (37, 3, False, True), (1024, 9, True, True), (9, 1, False, True),
    (4096, 4, False, True)])
def test_depth_mix_with_router_matches_separate_kernels(rows, n_sources, pending, slots):
    """parrot_depthmix_route_bf16 + parrot_moe_forward_routed_bf16 against
    parrot_depthmix_bf16 + parrot_moe_forward_bf16: the mix is bit-identical;
    expert ids agree wherever the router's top-2 / top-3 probability margin
    exceeds 1e-5 and equal top-2 of the fused call's own probabilities; the
    block output is identical on every token routed alike.  Slot mode
    (capacity -2: the depth mix groups the rows itself, no group kernel):
    each expert's positions fill its region, every grouped row holds its
    token's row, counts and statistics equal the grouping kernel's, and a
    second call (the counters were left at zero) gives the same output."""
    cfg = moe_config()
    module, _ = build_moe_pair(cfg, seed=31)
    dim = cfg.dim
    g = torch.Generator().manual_seed(rows + n_sources)
    srcs = [(torch.randn(rows, dim, generator=g) * (1 + i)).to(torch.bfloat16).cuda()
            for i in range(n_sources)]
    query = (0.3 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    key_w = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    out_w = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    delta = torch.randn(rows, dim, generator=g).to(torch.bfloat16).cuda() if pending else None
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptrs = (ctypes.c_void_p * n_sources)(*[s.data_ptr() for s in srcs])
    w = bridge._weights_struct(bridge.pack_weights(module), None)
    results = {}
    for fused in (False, True):
        dims = bridge.moe_dims(cfg, rows, -2 if (fused and slots) else 0)
        out = torch.empty(rows, dim, device="cuda", dtype=torch.bfloat16)
        pend_out = torch.empty_like(out) if pending else None
        layout = bridge.workspace_layout(dims)
        ws = torch.zeros(int(layout.total), device="cuda", dtype=torch.uint8)
        probs = torch.empty(rows, cfg.n_experts, device="cuda")
        idx = torch.empty(rows, 2, device="cuda", dtype=torch.int64)
        y = torch.empty(rows, dim, device="cuda", dtype=torch.bfloat16)
        pos = torch.full((2 * rows,), -1, device="cuda", dtype=torch.int32)
        counts = torch.full((cfg.n_experts,), -1, device="cuda", dtype=torch.int32)
        stats = torch.full((cfg.n_experts + 1,), float("nan"), device="cuda")
        args = (ctypes.c_void_p(out.data_ptr()), ptrs, n_sources, ctypes.c_void_p(query.data_ptr()),
                ctypes.c_void_p(key_w.data_ptr()), 1e-6, ctypes.c_void_p(out_w.data_ptr()), 1e-6,
                None, bridge._p(srcs[-1] if pending else None), bridge._p(delta),
                bridge._p(pend_out), rows, dim)
        if fused:
            ro = _lib.MoeOutputs(None, None, probs.data_ptr(), idx.data_ptr(), None, None, None,
                                 None)
            _lib.check(lib.parrot_depthmix_route_bf16(
                *args, ctypes.byref(dims), ctypes.byref(w), ctypes.byref(ro),
                ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream), "depthmix_route")
            mo = _lib.MoeOutputs(y.data_ptr(), None, None, None, None, pos.data_ptr(),
                                 counts.data_ptr(), stats.data_ptr())
            _lib.check(lib.parrot_moe_forward_routed_bf16(
                ctypes.byref(dims), ctypes.byref(w), ctypes.c_void_p(out.data_ptr()),
                ctypes.byref(mo), 0, ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream),
                "moe_forward_routed")
        else:
            _lib.check(lib.parrot_depthmix_bf16(*args, stream), "depthmix")
            mo = _lib.MoeOutputs(y.data_ptr(), None, probs.data_ptr(), idx.data_ptr(), None,
                                 pos.data_ptr(), counts.data_ptr(), stats.data_ptr())
            _lib.check(lib.parrot_moe_forward_bf16(
                ctypes.byref(dims), ctypes.byref(w), ctypes.c_void_p(out.data_ptr()),
                ctypes.byref(mo), ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream),
                "moe_forward")
        torch.cuda.synchronize()
        status = (ctypes.c_int * 4)()
        _lib.check(lib.parrot_moe_read_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(dims),
                                              status, stream), "status")
        assert list(status) == [0, 0, 0, 0]
        results[fused] = (out.clone(), None if pend_out is None else pend_out.clone(),
                          probs.cpu(), idx.cpu(), y.clone())
        if fused and slots:
            C = layout.capacity
            cnt, pos_c, idx_c = counts.cpu(), pos.cpu().long(), idx.cpu().flatten()
            assert C >= 2 * rows and int(cnt.sum()) == 2 * rows
            assert torch.equal(cnt, torch.bincount(idx_c, minlength=cfg.n_experts).int())
            for e in range(cfg.n_experts):
                got = torch.sort(pos_c[idx_c == e]).values
                assert torch.equal(got, e * C + torch.arange(int(cnt[e]))), e
            grouped = workspace_view(ws, layout, "grouped", torch.bfloat16,
                                     (layout.grouped_rows, dim)).cpu()
            assert torch.equal(grouped[pos_c], out.cpu()[torch.arange(2 * rows) // 2])
            util = cnt.float() / (2 * rows)
            assert torch.equal(stats.cpu()[:-1], util)
            aux = cfg.n_experts * float((util * probs.cpu().mean(0)).sum())
            assert abs(float(stats[-1]) - aux) <= 1e-5 * max(1.0, abs(aux))
            # the counters were left at zero: the same call again gives the same block
            y_first = y.clone()
            _lib.check(lib.parrot_depthmix_route_bf16(
                *args, ctypes.byref(dims), ctypes.byref(w), ctypes.byref(ro),
                ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream), "depthmix_route")
            _lib.check(lib.parrot_moe_forward_routed_bf16(
                ctypes.byref(dims), ctypes.byref(w), ctypes.c_void_p(out.data_ptr()),
                ctypes.byref(mo), 0, ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream),
                "moe_forward_routed")
            torch.cuda.synchronize()
            assert torch.equal(y, y_first)
            assert torch.equal(counts.cpu(), cnt)
    (o0, p0, pr0, i0, y0), (o1, p1, pr1, i1, y1) = results[False], results[True]
    assert torch.equal(o0, o1)
    if pending:
        assert torch.equal(p0, p1)
    top = pr1.topk(2, dim=-1).indices
    assert torch.equal(i1, top)                       # own probabilities
    top3 = pr0.topk(3, dim=-1).values
    clear = ((top3[:, 1] - top3[:, 2]) > 1e-5) & ((top3[:, 0] - top3[:, 1]) > 1e-5)
    assert torch.equal(i0[clear], i1[clear])
    torch.testing.assert_close(pr1, pr0, rtol=0, atol=1e-5)
    same = (i0 == i1).all(-1).cuda()
    assert torch.equal(y0[same], y1[same]) or \
        float((y0[same].float() - y1[same].float()).abs().max()) <= 2 ** -6 * float(y0.float().abs().max())


@pytest.mark.parametrize("rows,n_sources", [(1, 5), (3, 8), (4, 2)])
def test_decode_moe_routed_by_the_depth_mix(rows, n_sources):
    """Decode batch sizes: parrot_depthmix_route_bf16 + parrot_moe_decode_routed_bf16
    (the gate/up kernel reads the routing, the down kernel fetches its expert
    rows before its dependency wait) against parrot_depthmix_bf16 +
    parrot_moe_decode_bf16 (the kernels route themselves): the mix is
    bit-identical and the block output identical on every token routed alike."""
    cfg = moe_config()
    module, _ = build_moe_pair(cfg, seed=41 + rows)
    dim = cfg.dim
    g = torch.Generator().manual_seed(100 + rows)
    srcs = [(torch.randn(rows, dim, generator=g) * (1 + i)).to(torch.bfloat16).cuda()
            for i in range(n_sources)]
    query = (0.3 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    key_w = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    out_w = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    res = torch.randn(rows, dim, generator=g).to(torch.bfloat16).cuda()
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptrs = (ctypes.c_void_p * n_sources)(*[s.data_ptr() for s in srcs])
    dims = bridge.moe_dims(cfg, rows)
    w = bridge._weights_struct(bridge.pack_weights(module), None)
    results = {}
    for fused in (False, True):
        out = torch.empty(rows, dim, device="cuda", dtype=torch.bfloat16)
        ws = torch.zeros(int(bridge.workspace_layout(dims).total), device="cuda",
                         dtype=torch.uint8)
        idx = torch.empty(rows, 2, device="cuda", dtype=torch.int64)
        y = torch.empty(rows, dim, device="cuda", dtype=torch.bfloat16)
        args = (ctypes.c_void_p(out.data_ptr()), ptrs, n_sources,
                ctypes.c_void_p(query.data_ptr()), ctypes.c_void_p(key_w.data_ptr()), 1e-6,
                ctypes.c_void_p(out_w.data_ptr()), 1e-6, None, None, None, None, rows, dim)
        if fused:
            ro = _lib.MoeOutputs(None, None, None, idx.data_ptr(), None, None, None, None)
            _lib.check(lib.parrot_depthmix_route_bf16(
                *args, ctypes.byref(dims), ctypes.byref(w), ctypes.byref(ro),
                ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream), "depthmix_route")
            mo = _lib.MoeOutputs(y.data_ptr(), res.data_ptr(), None, None, None, None, None, None)
            _lib.check(lib.parrot_moe_decode_routed_bf16(
                ctypes.byref(dims), ctypes.byref(w), ctypes.c_void_p(out.data_ptr()),
                ctypes.byref(mo), ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream),
                "moe_decode_routed")
        else:
            _lib.check(lib.parrot_depthmix_bf16(*args, stream), "depthmix")
            mo = _lib.MoeOutputs(y.data_ptr(), res.data_ptr(), None, idx.data_ptr(), None, None,
                                 None, None)
            _lib.check(lib.parrot_moe_decode_bf16(
                ctypes.byref(dims), ctypes.byref(w), ctypes.c_void_p(out.data_ptr()),
                ctypes.byref(mo), ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream),
                "moe_decode")
        torch.cuda.synchronize()
        results[fused] = (out.clone(), idx.cpu(), y.clone())
    (o0, i0, y0), (o1, i1, y1) = results[False], results[True]
    assert torch.equal(o0, o1)
    same = (i0 == i1).all(-1)
    assert bool(same.any())
    assert torch.equal(y0[same.cuda()], y1[same.cuda()]) or \
        float((y0[same.cuda()].float() - y1[same.cuda()].float()).abs().max()) <= \
        2 ** -6 * float(y0.float().abs().max())


@pytest.mark.parametrize("rows,n_sources,norm", [(8192, 4, True), (8193, 4, True),
                                                 (9000, 3, False), (8192, 2, True),
                                                 (8192, 8, True)])
def test_two_row_depth_mix_is_bit_identical(rows, n_sources, norm):
    """From 8192 rows the plain depth mix with up to 4 sources runs two rows per
    thread (8 sources: the one-row kernel either way); every
    row's arithmetic is the one-row kernel's, so the output equals the same
    rows mixed in calls below that size (one-row kernel) bit for bit, and
    stays within the bf16 contract of the oracle."""
    dim = 768
    g = torch.Generator().manual_seed(rows + n_sources)
    srcs = [(torch.randn(rows, dim, generator=g) * (1 + i)).to(torch.bfloat16).cuda()
            for i in range(n_sources)]
    q = (0.3 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    kw = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    ow = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    lib = _lib.load()

    def mix(lo, hi):
        n = hi - lo
        out = torch.empty(n, dim, device="cuda", dtype=torch.bfloat16)
        mix_out = torch.empty_like(out)
        parts = [s[lo:hi] for s in srcs]
        ptrs = (ctypes.c_void_p * n_sources)(*[p.data_ptr() for p in parts])
        _lib.check(lib.parrot_depthmix_bf16(
            out.data_ptr(), ptrs, n_sources, q.data_ptr(), kw.data_ptr(), 1e-6,
            ow.data_ptr() if norm else None, 1e-6, mix_out.data_ptr(), None, None, None, n, dim,
            bridge._stream()), "parrot_depthmix_bf16")
        return out, mix_out

    whole, whole_mix = mix(0, rows)
    half = rows // 2  # each part below the two-row threshold
    a, am = mix(0, half)
    b, bm = mix(half, rows)
    torch.cuda.synchronize()
    assert torch.equal(whole, torch.cat([a, b]))
    assert torch.equal(whole_mix, torch.cat([am, bm]))
    _, orc, onorm, _ = _depth_modules(dim, 1)
    orc.query.data.copy_(q.float().cpu())
    orc.norm.weight.data.copy_(kw.float().cpu())
    onorm.weight.data.copy_(ow.float().cpu())
    sample = torch.arange(0, rows, 97)
    exp_mix = orc([s.float().cpu()[sample] for s in srcs])
    assert_bf16_close(whole_mix.cpu()[sample], exp_mix, "two-row mix")
    if norm:
        assert_bf16_close(whole.cpu()[sample], onorm(exp_mix), "two-row mix + norm")


def test_bounded_mbarrier_wait_runs_out_with_status_and_the_device_stays_usable():
    """An mbarrier nobody arrives at, waited on through the tensor-core
    kernels' own bounded wait loop with a 20 ms limit: the wait gives up after
    the limit (not before, and well before the kernels' 2 s), sets the abort
    flag and records {timeout, site 90, block 0}; afterwards a MoE block runs
    on the same context and matches the oracle-checked path."""
    lib = _lib.load()
    out = torch.full((8,), -1, dtype=torch.int32, device="cuda")
    limit_ns = 20_000_000
    _lib.check(lib.parrot_selftest_wait_timeout(limit_ns, ctypes.c_void_p(out.data_ptr()),
                                                bridge._stream()), "selftest")
    torch.cuda.synchronize()
    code, site, block, spare, ok, aborted, waited_us, _ = out.tolist()
    assert (code, site, block, spare) == (1, 90, 0, 0)
    assert (ok, aborted) == (0, 1)
    assert limit_ns // 1000 <= waited_us < 1_000_000
    bad = ctypes.c_void_p(out.data_ptr())
    assert lib.parrot_selftest_wait_timeout(2_000_000_000, bad, bridge._stream()) != 0
    cfg = moe_config()
    with torch.inference_mode():
        module, _ = build_moe_pair(cfg, seed=21)
        x = hidden_states(64, cfg.dim, seed=22).cuda()
        first, _, _ = bridge.b200_moe(module, x, True)
        second, _, _ = bridge.b200_moe(module, x, True)
        torch.cuda.synchronize()
    assert torch.isfinite(first).all() and torch.equal(first, second)


def test_slot_mode_left_over_counters_are_reported_not_written_past():
    """Slot mode keeps per-expert counters in the workspace; a routing call
    whose block never runs leaves them set.  Routing again and again with
    every token on one expert must report the overflow in the status word and
    write nothing past the expert's region; parrot_moe_workspace_init clears
    the counters and the block then runs as usual."""
    cfg = moe_config()
    module, _ = build_moe_pair(cfg, seed=77)
    rows, dim = 256, cfg.dim
    g = torch.Generator().manual_seed(5)
    src = torch.randn(rows, dim, generator=g).to(torch.bfloat16).cuda()
    q = (0.3 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    kw = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    ow = (1 + 0.2 * torch.randn(dim, generator=g)).to(torch.bfloat16).cuda()
    bias = torch.tensor([30.0] + [0.0] * (cfg.n_experts - 1), device="cuda")
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ptrs = (ctypes.c_void_p * 1)(src.data_ptr())
    dims = bridge.moe_dims(cfg, rows, -2)
    layout = bridge.workspace_layout(dims)
    # room past the workspace to see that nothing lands there
    guard = 1 << 20
    buf = torch.zeros(int(layout.total) + guard, device="cuda", dtype=torch.uint8)
    ws = buf[:int(layout.total)]
    w = bridge._weights_struct(bridge.pack_weights(module), bias)
    out = torch.empty(rows, dim, device="cuda", dtype=torch.bfloat16)
    ro = _lib.MoeOutputs()

    def route():
        _lib.check(lib.parrot_depthmix_route_bf16(
            ctypes.c_void_p(out.data_ptr()), ptrs, 1, ctypes.c_void_p(q.data_ptr()),
            ctypes.c_void_p(kw.data_ptr()), 1e-6, ctypes.c_void_p(ow.data_ptr()), 1e-6, None,
            None, None, None, rows, dim, ctypes.byref(dims), ctypes.byref(w), ctypes.byref(ro),
            ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream), "depthmix_route")

    def status():
        st = (ctypes.c_int * 4)()
        _lib.check(lib.parrot_moe_read_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(dims),
                                              st, stream), "status")
        return list(st)

    def block():
        y = torch.empty(rows, dim, device="cuda", dtype=torch.bfloat16)
        mo = _lib.MoeOutputs(y.data_ptr(), None, None, None, None, None, None, None)
        _lib.check(lib.parrot_moe_forward_routed_bf16(
            ctypes.byref(dims), ctypes.byref(w), ctypes.c_void_p(out.data_ptr()),
            ctypes.byref(mo), 0, ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream), "routed")
        torch.cuda.synchronize()
        return y

    route()
    first = block()  # a clean pair leaves the counters at zero
    assert status() == [0, 0, 0, 0]
    for _ in range(3):  # every token's first expert is 0: T slots of its 2T per call
        route()
    torch.cuda.synchronize()
    st = status()
    assert st[0] == 2 and st[1] == 50, st  # a bad index, reported by the routing depth mix
    assert int(buf[int(layout.total):].count_nonzero()) == 0
    _lib.check(lib.parrot_moe_workspace_init(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(dims),
                                             stream), "workspace_init")
    route()
    assert torch.equal(block(), first)
    assert status() == [0, 0, 0, 0]
