"""The allocation-free MoE entry point (parrot_moe_forward_static_bf16).

Callers that cannot allocate device memory where they run the MoE block — for
example a serving runtime that reserves all device memory at start-up and
forbids allocation afterwards — use this entry point, which works out of a
fixed workspace inside the library instead of one the caller passes in.  These
checks call it through the C ABI and compare it with the workspace-taking
entry point, parrot_moe_forward_bf16, on two calls in a row.
"""
import ctypes

import pytest
import torch

from parrot_b200 import _lib, bridge
from tests.gpu_helpers import assert_bf16_close, build_moe_pair, hidden_states, moe_config

pytestmark = pytest.mark.gpu


def _call(fn_name, module, x, workspace=None):
    cfg = module.cfg
    dims = _lib.MoeDims(x.shape[0], cfg.dim, cfg.n_experts, 2, cfg.expert_dim,
                        cfg.shared_expert_dim, 0)
    weights = bridge._weights_struct(bridge.pack_weights(module), None)
    out = torch.full_like(x, float("nan"))
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
        for call, (tokens, seed) in enumerate(((64, 21), (192, 22))):
            x = hidden_states(tokens, cfg.dim, seed=seed).cuda()
            layout = bridge.workspace_layout(bridge.moe_dims(cfg, tokens))
            ws = torch.zeros(int(layout.total), device="cuda", dtype=torch.uint8)
            rc, expected, exp_stats = _call("workspace", module, x, ws)
            _lib.check(rc, "parrot_moe_forward_bf16")
            rc, got, got_stats = _call("static", module, x)
            _lib.check(rc, "parrot_moe_forward_static_bf16")
            torch.cuda.synchronize()
            assert_bf16_close(got, expected, f"static entry point, call {call + 1}")
            assert torch.isfinite(got).all()
            torch.testing.assert_close(got_stats, exp_stats, rtol=1e-6, atol=1e-7)


def test_static_entry_point_rejects_oversized_dims():
    cfg = moe_config()
    with torch.inference_mode():
        module, _ = build_moe_pair(cfg, seed=4)
        x = hidden_states(512, cfg.dim, seed=1).cuda()
        rc, _, _ = _call("static", module, x)
        assert rc == _lib.PARROT_EINVAL
        assert b"static workspace" in _lib.load().parrot_b200_last_error()
