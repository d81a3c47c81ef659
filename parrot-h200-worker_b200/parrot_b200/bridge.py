"""PyTorch <-> libparrot_b200 bridge for the B200 MoE / depth backends.

Each function mirrors one function of the reference's inference bridge
(``parrot/metal_moe.py``) with the same argument meaning, but calls the
sm_100a kernels through the C ABI.  Tensors stay on the caller's CUDA device
and every launch goes on ``torch.cuda.current_stream()``; outputs are fresh
``torch.empty`` tensors owned by the caller.  There is no CPU or eager-PyTorch
fallback: a CPU tensor, a non-bf16 dtype, autograd, or a missing library all
raise.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn.functional as F
from torch import Tensor

from . import _lib

_SUPPORTED: dict[int, bool] = {}
_WORKSPACES: dict[tuple, Tensor] = {}


# ---------------------------------------------------------------------------
# argument checks (the reference raises the same way, metal_moe.py:154-157)
# ---------------------------------------------------------------------------
def _require_device(t: Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(f"The B200 {what} backend requires CUDA tensors, got {t.device}")
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"The B200 {what} backend requires bfloat16, got {t.dtype}")
    idx = t.device.index if t.device.index is not None else torch.cuda.current_device()
    ok = _SUPPORTED.get(idx)
    if ok is None:
        ok = bool(_lib.load().parrot_b200_device_supported(idx))
        _SUPPORTED[idx] = ok
    if not ok:
        raise RuntimeError(f"The B200 {what} backend requires an sm_100 GPU (device {idx})")


def _require_inference(what: str) -> None:
    if torch.is_grad_enabled():
        raise RuntimeError(
            f"The B200 {what} backend is inference-only; call it under "
            "torch.inference_mode() or torch.no_grad()")


def param_key(p: Tensor) -> tuple:
    """Cache key of a parameter: its version counter when it has one.

    Tensors created under ``torch.inference_mode`` carry no version counter;
    for those the key is the storage identity alone.
    """
    try:
        version = p._version
    except RuntimeError:
        version = -1
    return (version, p.device, p.dtype, p.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t: Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _rows(x: Tensor) -> tuple[Tensor, int, int]:
    x = x.contiguous()
    dim = x.shape[-1]
    return x, x.numel() // dim, dim


# ---------------------------------------------------------------------------
# RMSNorm  (metal_moe.py:37-55)
# ---------------------------------------------------------------------------
def b200_rms_norm(module, x: Tensor) -> Tensor:
    """``module.weight``-scaled RMSNorm of ``x`` over its last dimension."""
    _require_device(x, "RMSNorm")
    _require_inference("RMSNorm")
    x, rows, dim = _rows(x)
    out = torch.empty_like(x)
    lib = _lib.load()
    w = module.weight
    _lib.check(lib.parrot_rmsnorm_bf16(_p(out), _p(x), _p(w), rows, dim, float(module.eps),
                                       _stream()), "parrot_rmsnorm_bf16")
    return out


# ---------------------------------------------------------------------------
# Rotary embedding, in place on the packed q/k/v projection (model.py:206-216)
# ---------------------------------------------------------------------------
def b200_rope_(qkv: Tensor, cos: Tensor, sin: Tensor, rot_heads: int, head_dim: int,
               start: int) -> Tensor:
    """Rotate the first ``rot_heads`` heads of every row of ``qkv`` [b, t, width] in place."""
    _require_device(qkv, "RoPE")
    b, t, width = qkv.shape
    if not qkv.is_contiguous():
        raise RuntimeError("b200_rope_ needs a contiguous projection output")
    lib = _lib.load()
    _lib.check(lib.parrot_rope_inplace_bf16(
        _p(qkv), _p(cos), _p(sin), b * t, width, rot_heads * head_dim, head_dim, t, start,
        cos.shape[0], _stream()), "parrot_rope_inplace_bf16")
    return qkv


def b200_rope_at_(qkv: Tensor, cos: Tensor, sin: Tensor, rot_heads: int, head_dim: int,
                  position: Tensor, status: Tensor | None = None) -> Tensor:
    """``b200_rope_`` for one decode position held in device memory (``position`` int32 [1])."""
    _require_device(qkv, "RoPE")
    b, t, width = qkv.shape
    if not qkv.is_contiguous():
        raise RuntimeError("b200_rope_at_ needs a contiguous projection output")
    _lib.check(_lib.load().parrot_rope_inplace_at_bf16(
        _p(qkv), _p(cos), _p(sin), b * t, width, rot_heads * head_dim, head_dim, t,
        _p(position), cos.shape[0], _p(status), _stream()), "parrot_rope_inplace_at_bf16")
    return qkv


def b200_linear_small(x: Tensor, w: Tensor, out_dtype: torch.dtype) -> Tensor:
    """``F.linear(x, w)`` for a decode step (at most 8 rows; ``model.py:303-328,
    399-432``): x [rows, k] bf16 or fp32, w [n, k] bf16 or fp32, fp32
    accumulation, the result rounded once to ``out_dtype`` (bf16 or fp32)."""
    if x.device.type != "cuda" or w.device != x.device:
        raise RuntimeError(f"The B200 linear_small backend requires CUDA tensors on one device, "
                           f"got {x.device} and {w.device}")
    for t in (x, w):
        if t.dtype not in (torch.bfloat16, torch.float32):
            raise RuntimeError(f"The B200 linear_small backend takes bf16 or fp32, got {t.dtype}")
    _require_inference("linear_small")
    x = x.contiguous()
    w = w.contiguous()
    rows, k = x.shape
    out = torch.empty((rows, w.shape[0]), device=x.device, dtype=out_dtype)
    _lib.check(_lib.load().parrot_linear_small(
        _p(out), int(out_dtype == torch.float32), _p(x), int(x.dtype == torch.float32), _p(w),
        int(w.dtype == torch.float32), rows, w.shape[0], k, _stream()), "parrot_linear_small")
    return out


_DECODE_SCRATCH: dict = {}


def b200_decode_attention(q: Tensor, k_new: Tensor, v_new: Tensor | None, k_cache: Tensor,
                          v_cache: Tensor | None, position: Tensor, n_heads: int,
                          n_kv_heads: int, head_dim: int, window: int, scale: float,
                          out_dtype: torch.dtype,
                          rope: tuple[Tensor, Tensor] | None = None) -> Tensor:
    """One decode step of attention at the device ``position`` (``model.py:303-328, 399-432``).

    ``q`` [B, n_heads * head_dim] (bf16, or fp32 for the absorbed MLA query) and
    ``k_new`` / ``v_new`` [B, n_kv_heads * head_dim] may be row-strided views of
    one projection.  The new key/value are appended to the caches at
    ``position``; returns [B, n_heads * head_dim] in ``out_dtype``.  With
    ``rope = (cos, sin)`` (bf16 tables) ``q`` and ``k_new`` are unrotated and the
    kernel applies the rotary embedding itself (``model.py:206-216``), bit for bit
    like ``b200_rope_at_`` before the call.
    """
    _require_device(k_cache, "decode attention")
    b = q.shape[0]
    s_max = k_cache.shape[-2]
    lib = _lib.load()
    key = (k_cache.device.index, b, n_heads, s_max, head_dim)
    scratch = _DECODE_SCRATCH.get(key)
    if scratch is None:
        n = lib.parrot_decode_attention_scratch_bytes(b, n_heads, s_max, head_dim)
        scratch = torch.zeros(int(n), device=k_cache.device, dtype=torch.uint8)
        _DECODE_SCRATCH[key] = scratch
    out = torch.empty((b, n_heads * head_dim), device=q.device, dtype=out_dtype)
    if rope is not None:
        cos, sin = rope
        _lib.check(lib.parrot_decode_attention_rope_bf16(
            _p(out), int(out_dtype == torch.float32), _p(q), q.stride(0), _p(k_new), _p(v_new),
            k_new.stride(0), _p(k_cache), _p(v_cache), _p(position), b, n_heads, n_kv_heads,
            s_max, head_dim, window, float(scale), _p(cos), _p(sin), cos.shape[0], _p(scratch),
            scratch.numel(), None, _stream()), "parrot_decode_attention_rope_bf16")
        return out
    _lib.check(lib.parrot_decode_attention_bf16(
        _p(out), int(out_dtype == torch.float32), _p(q), int(q.dtype == torch.float32), q.stride(0),
        _p(k_new), _p(v_new), k_new.stride(0), _p(k_cache), _p(v_cache), _p(position), b,
        n_heads, n_kv_heads, s_max, head_dim, window, float(scale), _p(scratch),
        scratch.numel(), None, _stream()), "parrot_decode_attention_bf16")
    return out


_VOCAB_SCRATCH: dict = {}
VOCAB_FUSED_MAX_ROWS = 8


def b200_vocab_argmax(hidden: Tensor, weight: Tensor) -> Tensor:
    """Greedy next token from the tied LM head (``metal_moe.py:329-353``
    ``metal_vocab_argmax``; ``model.py:927-931``): ``hidden`` [batch, (1,) dim]
    bf16, ``weight`` [vocab, dim] bf16 -> token ids [batch, 1] int64, the
    ``F.linear(hidden, weight).argmax(-1)`` of ``decode_next``.  Up to 8 rows
    the projection and the argmax are one kernel and no logits are written;
    above that the projection is a cuBLAS GEMM and the argmax this library's
    row kernel."""
    _require_device(hidden, "vocab argmax")
    _require_inference("vocab argmax")
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise RuntimeError("The B200 vocab argmax takes bf16 hidden states and weights")
    batch, dim = hidden.shape[0], hidden.shape[-1]
    h = hidden.reshape(batch, dim).contiguous()
    w = weight.contiguous()
    out = torch.empty((batch, 1), device=hidden.device, dtype=torch.int64)
    lib = _lib.load()
    if batch <= VOCAB_FUSED_MAX_ROWS:
        key = hidden.device.index
        scratch = _VOCAB_SCRATCH.get(key)
        if scratch is None:
            scratch = torch.zeros(int(lib.parrot_vocab_argmax_scratch_bytes()),
                                  device=hidden.device, dtype=torch.uint8)
            _VOCAB_SCRATCH[key] = scratch
        _lib.check(lib.parrot_vocab_argmax_bf16(
            _p(out), _p(h), _p(w), batch, dim, w.shape[0], _p(scratch), scratch.numel(),
            _stream()), "parrot_vocab_argmax_bf16")
        return out
    logits = F.linear(h, w)
    _lib.check(lib.parrot_argmax_rows_bf16(_p(out), _p(logits), batch, w.shape[0], _stream()),
               "parrot_argmax_rows_bf16")
    return out


# ---------------------------------------------------------------------------
# Block AttnRes depth mixing  (metal_moe.py:419-500)
# ---------------------------------------------------------------------------
# Fold each MoE block's router into the depth mix that produces its input
# (parrot_depthmix_route_bf16: one launch fewer per layer).  False runs the
# router kernel instead.
FUSE_MOE_ROUTER = True


# The router (folded into the depth mix, or the router kernel) also groups the
# rows (slot mode: each assignment takes an atomic slot of its expert and its
# row is written there), so the group kernel does not run.  It needs a
# capacity no expert can overflow (2 T rows per expert region), taken up to
# SLOT_GROUPING_MAX_TOKENS.
SLOT_GROUPING = True
# Up to 4096 tokens the router holds the rows it groups in registers.  Above,
# the tensor-core router reads them again: at T = 16384
# the block measured the same with or without slot mode (139.9 / 140.6 us),
# and its 2T-row regions would take 1.3 GB of workspace.
SLOT_GROUPING_MAX_TOKENS = 4096


def _route_dims(cfg, rows: int) -> _lib.MoeDims:
    """The MoE dims of a block whose router runs inside the depth mix (slot
    mode above the decode batch sizes, whose kernels do not group)."""
    slots = SLOT_GROUPING and DECODE_MOE_MAX_TOKENS < rows <= SLOT_GROUPING_MAX_TOKENS
    return moe_dims(cfg, rows, -2 if slots else 0)


def _block_dims(cfg, rows: int) -> _lib.MoeDims:
    """The MoE dims of a block routed by its own router kernel: slot mode too
    (the router groups the rows) above the decode batch sizes."""
    return _route_dims(cfg, rows) if rows > DECODE_MOE_MAX_TOKENS else moe_dims(cfg, rows)


# At decode batch sizes too (the small-batch kernels then read the routing
# instead of computing it).  False: they route themselves.
ROUTE_DECODE_IN_MIX = True


def _routes_in_mix(route, rows: int) -> bool:
    """Whether the mix producing ``route``'s (an MoE module's, or None) input of
    ``rows`` tokens also routes it: up to 4096 tokens (the grouped-GEMM path,
    and at decode batch sizes the small-batch kernels)."""
    low = 0 if ROUTE_DECODE_IN_MIX else DECODE_MOE_MAX_TOKENS
    return route is not None and FUSE_MOE_ROUTER and low < rows <= 4096


def _depth_call(module, sources: Sequence[Tensor], output_norm, pending_delta: Tensor | None,
                route=None):
    last = sources[-1]
    if isinstance(last, PendingMoE):
        if last.value is not None:  # already materialised: an ordinary source
            out, _ = _depth_call(module, list(sources[:-1]) + [last.value], output_norm, None)
            return out, last.value
        _require_inference("depth")
        out = _resolve_into(last, module.query, module.norm.weight, module.norm.eps,
                            sources[:-1], output_norm)
        return out.view(last.shape), last.value
    first = sources[0]
    _require_device(first, "depth")
    _require_inference("depth")
    n = len(sources)
    if not 1 <= n <= 16:
        raise RuntimeError("B200 depth mixing supports one to sixteen sources")
    flat = [s.reshape(-1, s.shape[-1]).contiguous() for s in sources]
    rows, dim = flat[0].shape
    out = torch.empty((rows, dim), device=first.device, dtype=first.dtype)
    pending_out = None
    base = None
    if pending_delta is not None:
        base = flat[-1]
        pending_delta = pending_delta.reshape(rows, dim).contiguous()
        pending_out = torch.empty_like(out)
    ptrs = (ctypes.c_void_p * n)(*[s.data_ptr() for s in flat])
    lib = _lib.load()
    ow = None if output_norm is None else output_norm.weight
    oe = 0.0 if output_norm is None else float(output_norm.eps)
    if output_norm is not None and _routes_in_mix(route, rows):
        # the mix is the MoE block's input: route it in the same launch
        dims = _route_dims(route.cfg, rows)
        ws = workspace(first.device, dims)
        wst = _weights_struct(pack_weights(route), _router_bias(route))
        outputs = _lib.MoeOutputs(None, None, None, None, None, None, None, None)
        _lib.check(lib.parrot_depthmix_route_bf16(
            _p(out), ptrs, n, _p(module.query), _p(module.norm.weight), float(module.norm.eps),
            _p(ow), oe, None, _p(base), _p(pending_delta), _p(pending_out), rows, dim,
            ctypes.byref(dims), ctypes.byref(wst), ctypes.byref(outputs), _p(ws), ws.numel(),
            _stream()), "parrot_depthmix_route_bf16")
        ws.__dict__["_b200_fused_route"] = out.data_ptr()
    else:
        _lib.check(lib.parrot_depthmix_bf16(
            _p(out), ptrs, n, _p(module.query), _p(module.norm.weight), float(module.norm.eps),
            _p(ow), oe, None, _p(base), _p(pending_delta), _p(pending_out), rows, dim,
            _stream()), "parrot_depthmix_bf16")
    out = out.view_as(first)
    if pending_delta is None:
        return out, None
    return out, pending_out.view_as(first)


def b200_depth_mix(module, sources: Sequence[Tensor]) -> Tensor:
    """``DepthMix.forward``: softmax-weighted sum of the raw sources."""
    return _depth_call(module, sources, None, None)[0]


def b200_depth_mix_norm(module, sources: Sequence[Tensor], output_norm,
                        pending_delta: Tensor | None = None, route=None):
    """``output_norm(DepthMix(sources))`` in one kernel.

    With ``pending_delta``, the last source is ``sources[-1] + pending_delta``
    (a residual add the caller deferred) and the call returns
    ``(normalized, resolved_last_source)``.  When the last source is a
    ``PendingMoE`` the kernel also performs that MoE block's combine and the
    call returns ``(normalized, resolved_last_source)`` too.  Otherwise it
    returns ``normalized``.  ``route``: the MoE module whose input this is;
    up to 4096 rows the kernel routes the output for it as well, and that
    module's next ``b200_moe`` / ``b200_moe_deferred`` call on the output
    starts from the grouping.
    """
    deferred = isinstance(sources[-1], PendingMoE)
    out, resolved = _depth_call(module, sources, output_norm, pending_delta, route)
    return out if pending_delta is None and not deferred else (out, resolved)


# ---------------------------------------------------------------------------
# MoE  (metal_moe.py:58-131, 372-416)
# ---------------------------------------------------------------------------
def pack_weights(module) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """Pack the routed and shared experts once per parameter version.

    Returns ``(router [E,d], gate_up, down, shared_gate_up, shared_down)``;
    the expert matrices are in the C ABI's tiled layout (contiguous 16 KB
    128 x 64 tiles; gate/up rows interleaved for the fused SwiGLU epilogue).  Like ``metal_moe.py:84-131`` the
    packed copy is reused without re-checking versions while the module is in
    eval mode with gradients disabled; ``invalidate_packed_weights`` forces a
    repack after in-place weight edits made in that state.
    """
    cached = module.__dict__.get("_b200_pack")
    if cached is not None and not torch.is_grad_enabled() and not module.training:
        return cached[1]
    params = [module.router.weight]
    for e in module.experts:
        params += [e.gate.weight, e.up.weight, e.down.weight]
    params += [module.shared.gate.weight, module.shared.up.weight, module.shared.down.weight]
    version = tuple(param_key(p) for p in params)
    if cached is not None and cached[0] == version:
        return cached[1]
    for p in params:
        _require_device(p, "MoE")
    lib = _lib.load()
    with torch.no_grad():
        cfg = module.cfg
        E, H, Hs, d = cfg.n_experts, cfg.expert_dim, cfg.shared_expert_dim, cfg.dim
        gate = torch.stack([e.gate.weight.detach() for e in module.experts]).contiguous()
        up = torch.stack([e.up.weight.detach() for e in module.experts]).contiguous()
        gate_up = torch.empty((E, 2 * H, d), device=gate.device, dtype=gate.dtype)
        _lib.check(lib.parrot_pack_gate_up_bf16(_p(gate_up), _p(gate), _p(up), E, H, d,
                                                _stream()), "parrot_pack_gate_up_bf16")
        stacked = torch.stack([e.down.weight.detach() for e in module.experts]).contiguous()
        down = torch.empty_like(stacked)
        _lib.check(lib.parrot_pack_down_bf16(_p(down), _p(stacked), E, d, H, _stream()),
                   "parrot_pack_down_bf16")
        sg = module.shared.gate.weight.detach().contiguous()
        su = module.shared.up.weight.detach().contiguous()
        shared_gate_up = torch.empty((2 * Hs, d), device=sg.device, dtype=sg.dtype)
        _lib.check(lib.parrot_pack_gate_up_bf16(_p(shared_gate_up), _p(sg), _p(su), 1, Hs, d,
                                                _stream()), "parrot_pack_gate_up_bf16")
        sd = module.shared.down.weight.detach().contiguous()
        shared_down = torch.empty_like(sd)
        _lib.check(lib.parrot_pack_down_bf16(_p(shared_down), _p(sd), 1, d, Hs, _stream()),
                   "parrot_pack_down_bf16")
        packed = (module.router.weight.detach().contiguous(), gate_up, down, shared_gate_up,
                  shared_down)
    module.__dict__["_b200_pack"] = (version, packed)
    return packed


def invalidate_packed_weights(module) -> None:
    module.__dict__.pop("_b200_pack", None)


def check_config(cfg) -> None:
    """The shapes the sm_100a kernels take, for a config selecting
    ``moe_backend="b200"`` / ``depth_backend="b200"`` (the b200 counterpart of
    the reference's per-backend checks, ``parrot/model.py:58-80``).  Raises
    ``ValueError`` like them."""
    if cfg.top_k != 2:
        raise ValueError("b200 requires top_k=2")
    if cfg.n_experts > 32 or cfg.n_experts < 2:
        raise ValueError("b200 supports 2 to 32 routed experts")
    if cfg.dim % 128 or cfg.dim > 1024:
        raise ValueError("b200 requires dim divisible by 128 and at most 1024")
    if cfg.expert_dim % 64 or cfg.shared_expert_dim % 64:
        raise ValueError("b200 requires expert widths divisible by 64")
    sources = 1 + (2 * cfg.n_layers + cfg.depth_block_size - 1) // cfg.depth_block_size
    if cfg.residual == "attnres" and sources > 16:
        raise ValueError("b200 depth mixing supports at most sixteen sources")


def moe_dims(cfg, tokens: int, capacity: int = 0) -> _lib.MoeDims:
    return _lib.MoeDims(tokens, cfg.dim, cfg.n_experts, cfg.top_k, cfg.expert_dim,
                        cfg.shared_expert_dim, capacity)


def workspace_layout(dims: _lib.MoeDims) -> _lib.MoeLayout:
    layout = _lib.MoeLayout()
    _lib.check(_lib.load().parrot_moe_workspace_layout(ctypes.byref(dims), ctypes.byref(layout)),
               "parrot_moe_workspace_layout")
    return layout


def _ws_key(device: torch.device, dims: _lib.MoeDims) -> tuple:
    return (device.index if device.index is not None else torch.cuda.current_device(),
            dims.tokens, dims.dim, dims.n_experts, dims.expert_dim, dims.shared_dim,
            dims.capacity)


def _routed_workspace(device: torch.device, cfg, tokens: int, flat: Tensor):
    """(dims, workspace) of a block whose input ``flat`` a depth mix routed,
    or None when it was not routed there (the marker is consumed)."""
    dims = _route_dims(cfg, tokens)
    ws = _WORKSPACES.get(_ws_key(device, dims))
    if ws is None or ws.__dict__.get("_b200_fused_route") != flat.data_ptr():
        return None
    del ws.__dict__["_b200_fused_route"]
    return dims, workspace(device, dims)


def workspace(device: torch.device, dims: _lib.MoeDims) -> Tensor:
    """Zero-initialised workspace shared by all MoE layers of one shape on ``device``.

    Calls that share a workspace must be ordered on one stream.
    """
    key = _ws_key(device, dims)
    ws = _WORKSPACES.get(key)
    if ws is None:
        layout = workspace_layout(dims)
        ws = torch.zeros(int(layout.total), device=device, dtype=torch.uint8)
        _WORKSPACES[key] = ws
    live = _LIVE_PENDING.pop(ws.data_ptr(), None)
    if live is not None:
        live.resolve()  # its combine still reads this workspace: finish it first
    return ws


@dataclass(eq=False)
class PendingMoE:
    """An MoE block output whose combine is left to the next depth mix.

    Its value is ``base + bf16(bf16(shared + contrib[2t]) + contrib[2t + 1])``
    (``base`` optional), the combine of ``model.py:546-551`` plus the residual
    add of ``:702``.  ``shared`` [T, d] and ``contrib`` [2T, d] are views of
    the MoE workspace, so the value is computed (by ``b200_depth_mix_norm`` or
    ``resolve``) before that workspace is used again; ``value`` holds it then.
    """
    base: Tensor | None
    shared: Tensor
    contrib: Tensor
    shape: torch.Size
    workspace_ptr: int
    value: Tensor | None = None

    def resolve(self) -> Tensor:
        """The value, materialised on its own (a one-source depth mix is exact)."""
        if self.value is None:
            dev, dt = self.shared.device, self.shared.dtype
            key = (dev.index, dt, self.shared.shape[1])
            ones = _UNIT_MIX.get(key)
            if ones is None:
                ones = _UNIT_MIX[key] = torch.ones(self.shared.shape[1], device=dev, dtype=dt)
            _resolve_into(self, ones, ones, 1e-6, None)
        return self.value


_LIVE_PENDING: dict[int, PendingMoE] = {}
_UNIT_MIX: dict[tuple, Tensor] = {}


def _resolve_into(p: PendingMoE, query: Tensor, key_w: Tensor, key_eps: float, rest,
                  output_norm=None):
    """One depth-mix launch whose last source is ``p``; returns the normalized
    (or plain) mix and sets ``p.value``.  ``rest``: the other sources (or None)."""
    rows, dim = p.shared.shape
    flat = [] if rest is None else [s.reshape(rows, dim).contiguous() for s in rest]
    n = len(flat) + 1
    if n > 16:
        raise RuntimeError("B200 depth mixing supports one to sixteen sources")
    out = torch.empty((rows, dim), device=p.shared.device, dtype=p.shared.dtype)
    value = torch.empty_like(out)
    base = None if p.base is None else p.base.reshape(rows, dim).contiguous()
    ptrs = (ctypes.c_void_p * n)(*([s.data_ptr() for s in flat] + [value.data_ptr()]))
    ow = None if output_norm is None else output_norm.weight
    oe = 0.0 if output_norm is None else float(output_norm.eps)
    _lib.check(_lib.load().parrot_depthmix_moe_bf16(
        _p(out), ptrs, n, _p(query), _p(key_w), float(key_eps), _p(ow), oe, None, _p(base),
        _p(p.shared), _p(p.contrib), _p(value), rows, dim, _stream()), "parrot_depthmix_moe_bf16")
    p.value = value.view(p.shape)
    if _LIVE_PENDING.get(p.workspace_ptr) is p:
        del _LIVE_PENDING[p.workspace_ptr]
    return out


def _weights_struct(packed, bias: Tensor | None) -> _lib.MoeWeights:
    router, gate_up, down, sgu, sd = packed
    return _lib.MoeWeights(router.data_ptr(), None if bias is None else bias.data_ptr(),
                           gate_up.data_ptr(), down.data_ptr(), sgu.data_ptr(), sd.data_ptr())


def _router_bias(module) -> Tensor | None:
    bias = getattr(module, "router_bias", None)
    if bias is None:
        return None
    return bias.to(device=module.router.weight.device, dtype=torch.float32).contiguous()


# Up to this many flattened tokens (and without router statistics) b200_moe
# takes the small-batch decode kernels instead of route/group/GEMM/combine
# (measured graph-replayed decode of Parrot XL: +8% tokens/s at B = 1, +10% at
# B = 2, +3% at B = 4, -13% at B = 8).
DECODE_MOE_MAX_TOKENS = 4


def b200_moe(module, flat: Tensor, collect_stats: bool, addend: Tensor | None = None):
    """Whole MoE block on ``flat`` [T, d]: returns ``(out, aux, utilization)``.

    ``out = addend + moe(flat)`` when ``addend`` is given (the residual add of
    ``model.py:585`` / ``:702`` fused into the combine).  ``aux`` and
    ``utilization`` are ``None`` unless ``collect_stats``.
    """
    _require_device(flat, "MoE")
    _require_inference("MoE")
    flat = flat.contiguous()
    T, d = flat.shape
    cfg = module.cfg
    packed = pack_weights(module)
    fused = _routed_workspace(flat.device, cfg, T, flat)
    routed = fused is not None
    dims, ws = fused if routed else (_block_dims(cfg, T), None)
    if ws is None:
        ws = workspace(flat.device, dims)
    out = torch.empty_like(flat)
    if addend is not None:
        addend = addend.reshape(T, d).contiguous()
        _require_device(addend, "MoE")
    stats = torch.empty(cfg.n_experts + 1, device=flat.device, dtype=torch.float32) \
        if collect_stats else None
    bias = _router_bias(module)
    outputs = _lib.MoeOutputs(out.data_ptr(), None if addend is None else addend.data_ptr(),
                              None, None, None, None, None,
                              None if stats is None else stats.data_ptr())
    weights = _weights_struct(packed, bias)
    if stats is None and 0 < T <= DECODE_MOE_MAX_TOKENS and cfg.expert_dim <= 1024:
        # decode batch sizes: the two-kernel small-batch path
        fn = "parrot_moe_decode_routed_bf16" if routed else "parrot_moe_decode_bf16"
        _lib.check(getattr(_lib.load(), fn)(
            ctypes.byref(dims), ctypes.byref(weights), _p(flat), ctypes.byref(outputs),
            _p(ws), ws.numel(), _stream()), fn)
    elif routed:
        _lib.check(_lib.load().parrot_moe_forward_routed_bf16(
            ctypes.byref(dims), ctypes.byref(weights), _p(flat), ctypes.byref(outputs), 0,
            _p(ws), ws.numel(), _stream()), "parrot_moe_forward_routed_bf16")
    else:
        _lib.check(_lib.load().parrot_moe_forward_bf16(
            ctypes.byref(dims), ctypes.byref(weights), _p(flat), ctypes.byref(outputs),
            _p(ws), ws.numel(), _stream()), "parrot_moe_forward_bf16")
    if stats is None:
        return out, None, None
    return out, stats[cfg.n_experts], stats[:cfg.n_experts]


# Fold each MoE block's combine into the next depth mix (measured on B200:
# one kernel fewer per layer of the Parrot XL forward).  False runs the
# combine kernel instead; the results are identical.
DEFER_MOE_COMBINE = True


def b200_moe_deferred(module, flat: Tensor, collect_stats: bool, addend: Tensor | None, shape):
    """The MoE block with its combine left to the next depth mix.

    Returns ``(out, aux, utilization)`` like ``b200_moe``, ``out`` a
    ``PendingMoE`` (value ``addend + moe(flat)``, shaped ``shape``); at decode
    batch sizes, where the small-batch kernels combine in place, the finished
    tensor instead.
    """
    _require_device(flat, "MoE")
    _require_inference("MoE")
    flat = flat.contiguous()
    T, d = flat.shape
    cfg = module.cfg
    if (T <= DECODE_MOE_MAX_TOKENS and not collect_stats) or not DEFER_MOE_COMBINE:
        out, aux, util = b200_moe(module, flat, collect_stats, addend)
        return out.view(shape), aux, util
    packed = pack_weights(module)
    fused = _routed_workspace(flat.device, cfg, T, flat)
    dims, ws = fused if fused is not None else (_block_dims(cfg, T), None)
    if ws is None:
        ws = workspace(flat.device, dims)
    if addend is not None:
        addend = addend.reshape(T, d).contiguous()
        _require_device(addend, "MoE")
    stats = torch.empty(cfg.n_experts + 1, device=flat.device, dtype=torch.float32) \
        if collect_stats else None
    outputs = _lib.MoeOutputs(None, None, None, None, None, None, None,
                              None if stats is None else stats.data_ptr())
    wst = _weights_struct(packed, _router_bias(module))
    if fused is not None:
        _lib.check(_lib.load().parrot_moe_forward_routed_bf16(
            ctypes.byref(dims), ctypes.byref(wst), _p(flat), ctypes.byref(outputs), 1, _p(ws),
            ws.numel(), _stream()), "parrot_moe_forward_routed_bf16")
    else:
        _lib.check(_lib.load().parrot_moe_forward_deferred_bf16(
            ctypes.byref(dims), ctypes.byref(wst), _p(flat), ctypes.byref(outputs), _p(ws),
            ws.numel(), _stream()), "parrot_moe_forward_deferred_bf16")
    lay = workspace_layout(dims)
    contrib = ws[lay.contrib:lay.contrib + 2 * T * d * 2].view(flat.dtype).view(2 * T, d)
    shared = ws[lay.shared_y:lay.shared_y + T * d * 2].view(flat.dtype).view(T, d)
    p = PendingMoE(addend, shared, contrib, torch.Size(shape), ws.data_ptr())
    _LIVE_PENDING[ws.data_ptr()] = p
    if stats is None:
        return p, None, None
    return p, stats[cfg.n_experts], stats[:cfg.n_experts]


def b200_route(module, flat: Tensor, collect_stats: bool):
    """Router + grouping: ``(probs|None, weights, indices, positions, counts)``.

    Same outputs as ``metal_route`` (``metal_moe.py:58-81``): fp32 softmax
    probabilities (when ``collect_stats``), renormalised top-2 weights
    [T, 2] fp32, expert ids [T, 2] int64, grouped row of each assignment
    [2T] int32 and per-expert counts [E] int32.  The grouped token rows stay in
    the shared workspace for ``b200_experts``.
    """
    _require_device(flat, "MoE")
    _require_inference("MoE")
    flat = flat.contiguous()
    T, d = flat.shape
    cfg = module.cfg
    packed = pack_weights(module)
    dims = moe_dims(cfg, T)
    ws = workspace(flat.device, dims)
    dev = flat.device
    probs = torch.empty((T, cfg.n_experts), device=dev, dtype=torch.float32) \
        if collect_stats else None
    weights = torch.empty((T, 2), device=dev, dtype=torch.float32)
    indices = torch.empty((T, 2), device=dev, dtype=torch.int64)
    positions = torch.empty(2 * T, device=dev, dtype=torch.int32)
    counts = torch.empty(cfg.n_experts, device=dev, dtype=torch.int32)
    placeholder = torch.empty_like(flat[:1]) if T else flat
    outputs = _lib.MoeOutputs(placeholder.data_ptr(), None, _p(probs), indices.data_ptr(),
                              weights.data_ptr(), positions.data_ptr(), counts.data_ptr(), None)
    wst = _weights_struct(packed, _router_bias(module))
    _lib.check(_lib.load().parrot_moe_route_bf16(
        ctypes.byref(dims), ctypes.byref(wst), _p(flat), ctypes.byref(outputs), _p(ws),
        ws.numel(), _stream()), "parrot_moe_route_bf16")
    ws.__dict__["_b200_routed"] = (flat.data_ptr(), positions.data_ptr())
    return probs, weights, indices, positions, counts


def b200_experts(module, flat: Tensor, indices: Tensor, weights: Tensor,
                 positions: Tensor, counts: Tensor, addend: Tensor | None = None) -> Tensor:
    """Experts + shared expert + combine after ``b200_route`` (``metal_moe.py:372-416``).

    ``positions`` must be the tensor ``b200_route`` returned for this ``flat``:
    the grouped rows it refers to live in the shared workspace.
    """
    _require_device(flat, "MoE")
    _require_inference("MoE")
    flat = flat.contiguous()
    T, d = flat.shape
    packed = pack_weights(module)
    dims = moe_dims(module.cfg, T)
    ws = workspace(flat.device, dims)
    if ws.__dict__.get("_b200_routed") != (flat.data_ptr(), positions.data_ptr()):
        raise ValueError("b200_experts needs the positions returned by b200_route for this input")
    out = torch.empty_like(flat)
    if addend is not None:
        addend = addend.reshape(T, d).contiguous()
    outputs = _lib.MoeOutputs(out.data_ptr(), None if addend is None else addend.data_ptr(),
                              None, None, None, None, None, None)
    wst = _weights_struct(packed, _router_bias(module))
    _lib.check(_lib.load().parrot_moe_experts_bf16(
        ctypes.byref(dims), ctypes.byref(wst), _p(flat), ctypes.byref(outputs), _p(ws),
        ws.numel(), _stream()), "parrot_moe_experts_bf16")
    return out


def read_status(flat_tokens: int, cfg, device: torch.device) -> list[int]:
    """Device status word of the workspace used for ``flat_tokens`` (synchronises)."""
    dims = moe_dims(cfg, flat_tokens)
    ws = workspace(device, dims)
    buf = (ctypes.c_int * 4)()
    _lib.check(_lib.load().parrot_moe_read_status(_p(ws), ctypes.byref(dims), buf, _stream()),
               "parrot_moe_read_status")
    return list(buf)
