"""The allocation-free MoE entry point (parrot_moe_forward_static_bf16).

Callers that cannot allocate device memory where they run the MoE block — for
example a serving runtime that reserves all device memory at start-up and
forbids allocation afterwards — use this entry point, which works out of a
fixed workspace inside the library instead of one the caller passes in.  These
checks call it through the C ABI and compare it with the workspace-taking
entry point, parrot_moe_forward_bf16, on two calls in a row: both run the same
deterministic kernels, so the outputs must be identical bit for bit.
"""
import ctypes

import pytest
import torch

from parrot_b200 import _lib, bridge
from tests.gpu_helpers import build_moe_pair, hidden_states, moe_config

pytestmark = pytest.mark.gpu

STATIC_BYTES = 4 << 20  # the library's compiled-in workspace
MAX_TOKENS = 192        # largest Parrot XL token count whose workspace fits it


def _call(fn_name, module, x, workspace=None, out=None, stats=None):
    cfg = module.cfg
    dims = _lib.MoeDims(x.shape[0], cfg.dim, cfg.n_experts, 2, cfg.expert_dim,
                        cfg.shared_expert_dim, 0)
    weights = bridge._weights_struct(bridge.pack_weights(module), None)
    if out is None:
        out = torch.full_like(x, float("nan"))
    if stats is None:
        stats = torch.full((cfg.n_experts + 1,), float("nan"), device=x.device)
    outputs = _lib.MoeOutputs(out.data_ptr(), None, None, None, None, None, None,
                              stats.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    lib = _lib.load()
    if fn_name == "static":
        rc = lib.parrot_moe_forward_static_bf16(ctypes.byref(dims), ctypes.byref(weights),
                                                ctypes.c_void_p(x.data_ptr()),
                                                ctypes.byref(outputs), stream)
    else:
        rc = lib.parrot_moe_forward_bf16(ctypes.byref(dims), ctypes.byref(weights),
                                         ctypes.c_void_p(x.data_ptr()), ctypes.byref(outputs),
                                         ctypes.c_void_p(workspace.data_ptr()),
                                         workspace.numel(), stream)
    return rc, out, stats


def test_static_entry_point_matches_workspace_entry_point_twice():
    cfg = moe_config()
    with torch.inference_mode():
        module, _ = build_moe_pair(cfg, seed=4)
        for call, (tokens, seed) in enumerate(((64, 21), (MAX_TOKENS, 22))):
            x = hidden_states(tokens, cfg.dim, seed=seed).cuda()
            layout = bridge.workspace_layout(bridge.moe_dims(cfg, tokens))
            ws = torch.zeros(int(layout.total), device="cuda", dtype=torch.uint8)
            rc, expected, exp_stats = _call("workspace", module, x, ws)
            _lib.check(rc, "parrot_moe_forward_bf16")
            rc, got, got_stats = _call("static", module, x)
            _lib.check(rc, "parrot_moe_forward_static_bf16")
            torch.cuda.synchronize()
            assert torch.isfinite(got).all()
            assert torch.equal(got, expected), f"static entry point, call {call + 1}"
            assert torch.equal(got_stats, exp_stats), f"router stats, call {call + 1}"


def test_static_entry_point_allocates_no_device_memory():
    # The library does not allocate through torch's caching allocator, so the
    # driver's free-memory figure is the one that would show an allocation.
    cfg = moe_config()
    with torch.inference_mode():
        module, _ = build_moe_pair(cfg, seed=5)
        x = hidden_states(128, cfg.dim, seed=23).cuda()
        out = torch.empty_like(x)
        stats = torch.empty(cfg.n_experts + 1, device="cuda")
        bridge.pack_weights(module)  # packed once and cached before the measured calls
        _lib.check(_call("static", module, x, out=out, stats=stats)[0], "warm-up call")
        torch.cuda.synchronize()
        first = out.clone()
        free_before = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            _lib.check(_call("static", module, x, out=out, stats=stats)[0], "static call")
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before
        assert torch.equal(out, first)


def test_static_workspace_bound_is_exact_at_parrot_xl_widths():
    cfg = moe_config()
    assert int(bridge.workspace_layout(bridge.moe_dims(cfg, MAX_TOKENS)).total) <= STATIC_BYTES
    assert int(bridge.workspace_layout(bridge.moe_dims(cfg, MAX_TOKENS + 1)).total) > STATIC_BYTES


@pytest.mark.parametrize("tokens", [MAX_TOKENS + 1, 512])
def test_static_entry_point_rejects_oversized_dims(tokens):
    cfg = moe_config()
    with torch.inference_mode():
        module, _ = build_moe_pair(cfg, seed=4)
        x = hidden_states(tokens, cfg.dim, seed=1).cuda()
        rc, out, _ = _call("static", module, x)
        assert rc == _lib.PARROT_EINVAL
        assert b"static workspace" in _lib.load().parrot_b200_last_error()
        torch.cuda.synchronize()
        assert torch.isnan(out).all()  # nothing was launched
