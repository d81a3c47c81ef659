"""Parrot XL inference model whose MoE block, RMSNorm and Block AttnRes run on B200 kernels.

Public surface = the reference's ``parrot`` package (``parrot/model.py``):
``ModelConfig``, ``Parrot.forward / prefill / decode_step / decode_next /
parameter_counts``, ``ModelOutput``, ``GenerationState`` and the cache
dataclasses, with the same module tree and ``state_dict`` keys, so
``Parrot(cfg).load_state_dict(reference.state_dict())`` is exact and
``torch.manual_seed(s); Parrot(cfg)`` draws the reference's seeded weights.

Backends: ``moe_backend="b200"`` and ``depth_backend="b200"`` are the only
values.  The MoE block (router, top-2, grouping, grouped SwiGLU experts,
shared expert, combine + residual), every RMSNorm and every depth mix run as
sm_100a kernels from ``libparrot_b200.so``; attention, the embedding and the
tied LM head stay PyTorch (SDPA / cuBLAS).  The backend is inference-only,
like the reference's Metal backends: call it under ``torch.inference_mode()``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch
from torch import Tensor, nn
from torch.nn import functional as F
from torch.nn.attention import SDPBackend, sdpa_kernel

from . import bridge

# Decode attends over a key length that grows by one every step.  The cuDNN
# SDPA backend builds an execution plan per new shape, so decode keeps to the
# shape-generic backends.
_DECODE_SDPA = [SDPBackend.FLASH_ATTENTION, SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]

_ROPE: dict[tuple, tuple[Tensor, Tensor]] = {}
_WINDOW_MASKS: dict[tuple, list[Tensor]] = {}


@dataclass(frozen=True)
class ModelConfig:
    """Hyper-parameters (``model.py:15-43``) plus the B200 backend selection."""
    vocab_size: int = 32768
    dim: int = 768
    n_layers: int = 16
    n_heads: int = 8
    n_kv_heads: int = 2
    head_dim: int = 96
    kv_latent_dim: int = 128
    global_every: int = 4
    window_size: int = 2048
    max_seq_len: int = 4096
    n_experts: int = 16
    top_k: int = 2
    expert_dim: int = 512
    shared_expert_dim: int = 256
    moe_backend: Literal["b200"] = "b200"
    depth_backend: Literal["b200"] = "b200"
    residual: Literal["attnres", "standard"] = "attnres"
    depth_block_size: int = 4
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6
    aux_loss_weight: float = 0.01
    collect_router_stats: bool = True
    checkpoint_modules: bool = False
    local_query_chunk: int = 256

    def __post_init__(self):
        # the reference's own checks (model.py:46-57, 81-82)
        for name in ("vocab_size", "dim", "n_layers", "n_heads", "n_kv_heads", "head_dim",
                     "kv_latent_dim", "global_every", "window_size", "max_seq_len",
                     "n_experts", "top_k", "expert_dim", "shared_expert_dim",
                     "depth_block_size", "local_query_chunk"):
            if getattr(self, name) <= 0:
                raise ValueError(f"{name} must be positive")
        if self.n_heads % self.n_kv_heads or self.head_dim % 2:
            raise ValueError("n_heads must divide by n_kv_heads; head_dim must be even")
        if self.top_k > self.n_experts:
            raise ValueError("top_k cannot exceed n_experts")
        if self.residual not in ("attnres", "standard"):
            raise ValueError("residual must be attnres or standard")
        if self.norm_eps <= 0 or self.rope_theta <= 0 or self.aux_loss_weight < 0:
            raise ValueError("Invalid norm_eps, rope_theta, or aux_loss_weight")
        # backend selection and the shapes the sm_100a kernels take
        # (the reference's per-backend checks: model.py:58-80)
        if self.moe_backend != "b200":
            raise ValueError("parrot_b200 implements moe_backend='b200' only")
        if self.depth_backend != "b200":
            raise ValueError("parrot_b200 implements depth_backend='b200' only")
        bridge.check_config(self)

    @property
    def depth_sources(self) -> int:
        """Most sources any depth mix sees (embedding + completed blocks + partial)."""
        return 1 + (2 * self.n_layers + self.depth_block_size - 1) // self.depth_block_size


@dataclass
class LocalKVCache:
    key: Tensor    # [batch, kv heads, max positions, head width], RoPE applied
    value: Tensor


@dataclass
class MLALatentCache:
    latent: Tensor  # [batch, max positions, latent width]


@dataclass
class GenerationState:
    layers: list[LocalKVCache | MLALatentCache]
    position: int
    batch_size: int
    # the same position as an int32 [1] device tensor: the decode kernels read
    # it there, so one captured decode step replays at every position
    position_device: Tensor | None = None


@dataclass
class ModelOutput:
    logits: Tensor
    loss: Tensor | None
    lm_loss: Tensor | None
    aux_loss: Tensor
    expert_utilization: Tensor


class RMSNorm(nn.Module):
    """RMSNorm on the B200 kernel (``model.py:109-127``)."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: Tensor) -> Tensor:
        return bridge.b200_rms_norm(self, x)


class DepthMix(nn.Module):
    """Block AttnRes (``model.py:130-164``): keys normalised, values raw block sums."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.query = nn.Parameter(torch.zeros(cfg.dim))
        self.norm = RMSNorm(cfg.dim, cfg.norm_eps)

    def forward(self, sources: list[Tensor]) -> Tensor:
        return bridge.b200_depth_mix(self, sources)

    def normalized(self, sources: list[Tensor], output_norm: RMSNorm,
                   pending_delta: Tensor | None = None, route=None):
        """``output_norm(self(sources))`` in one kernel; see ``bridge.b200_depth_mix_norm``
        (``route``: the MoE module this output feeds, routed in the same kernel)."""
        return bridge.b200_depth_mix_norm(self, sources, output_norm, pending_delta, route)


# decode steps of at most this many rows run their attention projections on
# parrot_linear_small (weights read ahead of the dependency wait); larger ones on cuBLAS
_SMALL_LINEAR_ROWS = 8


def _rope_tables(cfg: ModelConfig, device, dtype) -> tuple[Tensor, Tensor]:
    key = (device.type, device.index, dtype, cfg.max_seq_len, cfg.head_dim, cfg.rope_theta)
    hit = _ROPE.get(key)
    if hit is None:
        with torch.inference_mode(False):
            exponent = torch.arange(0, cfg.head_dim, 2, device=device).float() / cfg.head_dim
            angle = torch.arange(cfg.max_seq_len, device=device).float()[:, None] * \
                (cfg.rope_theta ** -exponent)
            hit = (angle.cos().to(dtype), angle.sin().to(dtype))
        _ROPE[key] = hit
    return hit


def _packed(module: nn.Module, attr: str, params: tuple[Tensor, ...]) -> Tensor:
    """Concatenated projection weights, rebuilt when any parameter changes."""
    version = tuple(bridge.param_key(p) for p in params)
    hit = module.__dict__.get(attr)
    if hit is None or hit[0] != version:
        hit = (version, torch.cat([p.detach() for p in params], 0).contiguous())
        module.__dict__[attr] = hit
    return hit[1]


class LocalGQA(nn.Module):
    """Sliding-window RoPE grouped-query attention (``model.py:167-328``), PyTorch SDPA."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.q = nn.Linear(cfg.dim, cfg.n_heads * cfg.head_dim, bias=False)
        self.k = nn.Linear(cfg.dim, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.v = nn.Linear(cfg.dim, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.out = nn.Linear(cfg.n_heads * cfg.head_dim, cfg.dim, bias=False)

    def _qkv(self, x: Tensor, start: int):
        """q, k (rotated) and v as [b, heads, t, head_dim] views of one projection."""
        c = self.cfg
        b, t, _ = x.shape
        if start + t > c.max_seq_len:
            raise ValueError("RoPE position exceeds max_seq_len")
        w = _packed(self, "_qkv_weight", (self.q.weight, self.k.weight, self.v.weight))
        qkv = F.linear(x, w)
        cos, sin = _rope_tables(c, x.device, x.dtype)
        bridge.b200_rope_(qkv, cos, sin, c.n_heads + c.n_kv_heads, c.head_dim, start)
        qw, kw = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
        q = qkv[..., :qw].view(b, t, c.n_heads, c.head_dim).transpose(1, 2)
        k = qkv[..., qw:qw + kw].view(b, t, c.n_kv_heads, c.head_dim).transpose(1, 2)
        v = qkv[..., qw + kw:].view(b, t, c.n_kv_heads, c.head_dim).transpose(1, 2)
        return q, k, v

    def prefill(self, x: Tensor):
        c = self.cfg
        b, t, _ = x.shape
        q, k, v = self._qkv(x, 0)
        if t <= c.window_size:
            # every key inside the window: plain causal attention
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        else:
            key = (x.device.type, x.device.index, t, c.window_size, c.local_query_chunk)
            masks = _WINDOW_MASKS.get(key)
            starts = list(range(0, t, c.local_query_chunk))
            if masks is None:
                masks = []
                for s in starts:
                    e = min(t, s + c.local_query_chunk)
                    lo = max(0, s - c.window_size + 1)
                    qi = torch.arange(s, e, device=x.device)[:, None]
                    ki = torch.arange(lo, e, device=x.device)[None, :]
                    masks.append((ki <= qi) & (ki > qi - c.window_size))
                _WINDOW_MASKS[key] = masks
            parts = []
            for s, m in zip(starts, masks):
                e = min(t, s + c.local_query_chunk)
                lo = max(0, s - c.window_size + 1)
                parts.append(F.scaled_dot_product_attention(
                    q[:, :, s:e], k[:, :, lo:e], v[:, :, lo:e], attn_mask=m, enable_gqa=True))
            y = torch.cat(parts, 2)
        return self.out(y.transpose(1, 2).reshape(b, t, -1)), k, v

    def forward(self, x: Tensor) -> Tensor:
        return self.prefill(x)[0]

    def decode(self, x: Tensor, cache: LocalKVCache, position: int,
               addend: Tensor | None = None, defer_sum: bool = False,
               position_device: Tensor | None = None) -> Tensor:
        if x.shape[1] != 1:
            raise ValueError("decode expects one model position")
        if defer_sum:
            raise RuntimeError("deferred attention reduction is not part of the b200 backend")
        c = self.cfg
        if position_device is not None:
            # device-position path: RoPE, cache append and attention read the
            # position from device memory (capturable)
            b = x.shape[0]
            w = _packed(self, "_qkv_weight", (self.q.weight, self.k.weight, self.v.weight))
            small = b <= _SMALL_LINEAR_ROWS
            qkv = bridge.b200_linear_small(x.view(b, -1), w, x.dtype) if small else F.linear(x, w)
            cos, sin = _rope_tables(c, x.device, x.dtype)
            flat = qkv.view(b, -1)
            qw, kw = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
            # RoPE of q and the new key happens inside the attention kernel
            y = bridge.b200_decode_attention(
                flat[:, :qw], flat[:, qw:qw + kw], flat[:, qw + kw:], cache.key, cache.value,
                position_device, c.n_heads, c.n_kv_heads, c.head_dim, c.window_size,
                c.head_dim ** -0.5, x.dtype, rope=(cos, sin))
            out = (bridge.b200_linear_small(y, self.out.weight, x.dtype).view(b, 1, -1) if small
                   else self.out(y.view(b, 1, -1)))
            return out if addend is None else addend + out
        q, k, v = self._qkv(x, position)
        cache.key[:, :, position:position + 1].copy_(k)
        cache.value[:, :, position:position + 1].copy_(v)
        lo = max(0, position - self.cfg.window_size + 1)
        with sdpa_kernel(_DECODE_SDPA):
            y = F.scaled_dot_product_attention(q, cache.key[:, :, lo:position + 1],
                                               cache.value[:, :, lo:position + 1],
                                               enable_gqa=True)
        out = self.out(y.transpose(1, 2).reshape(x.shape[0], 1, -1))
        return out if addend is None else addend + out


class GlobalMLA(nn.Module):
    """NoPE joint-latent attention (``model.py:331-432``), PyTorch SDPA."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        width = cfg.n_heads * cfg.head_dim
        self.q = nn.Linear(cfg.dim, width, bias=False)
        self.kv_down = nn.Linear(cfg.dim, cfg.kv_latent_dim, bias=False)
        self.k_up = nn.Linear(cfg.kv_latent_dim, width, bias=False)
        self.v_up = nn.Linear(cfg.kv_latent_dim, width, bias=False)
        self.out = nn.Linear(width, cfg.dim, bias=False)

    def prefill(self, x: Tensor):
        c = self.cfg
        b, t, _ = x.shape
        w = _packed(self, "_qkv_weight", (self.q.weight, self.kv_down.weight))
        q, latent = F.linear(x, w).split((c.n_heads * c.head_dim, c.kv_latent_dim), -1)
        kv = F.linear(latent, _packed(self, "_up_weight", (self.k_up.weight, self.v_up.weight)))
        k, v = kv.split(c.n_heads * c.head_dim, -1)

        def heads(y):
            return y.reshape(b, t, c.n_heads, c.head_dim).transpose(1, 2)

        y = F.scaled_dot_product_attention(heads(q), heads(k), heads(v), is_causal=True)
        return self.out(y.transpose(1, 2).reshape(b, t, -1)), latent.contiguous()

    def forward(self, x: Tensor) -> Tensor:
        return self.prefill(x)[0]

    def _absorbed(self) -> tuple[Tensor, Tensor]:
        """Latent-space query / output weights (``model.py:362-397``)."""
        c = self.cfg
        params = (self.q.weight, self.k_up.weight, self.v_up.weight, self.out.weight)
        version = tuple(bridge.param_key(p) for p in params)
        hit = self.__dict__.get("_absorbed_cache")
        if hit is None or hit[0] != version:
            wq = self.q.weight.detach().float().view(c.n_heads, c.head_dim, c.dim)
            wk = self.k_up.weight.detach().float().view(c.n_heads, c.head_dim, c.kv_latent_dim)
            wv = self.v_up.weight.detach().float().view(c.n_heads, c.head_dim, c.kv_latent_dim)
            wo = self.out.weight.detach().float().view(c.dim, c.n_heads, c.head_dim)
            aq = torch.einsum("hdl,hdm->hlm", wk, wq).reshape(c.n_heads * c.kv_latent_dim, c.dim)
            ao = torch.einsum("hdl,mhd->mhl", wv, wo).reshape(c.dim, c.n_heads * c.kv_latent_dim)
            dt = self.q.weight.dtype
            aq, ao = aq.to(dt).contiguous(), ao.to(dt).contiguous()
            # the fp32 forms the absorbed path multiplies with (model.py:420), kept
            # with the cache instead of converted on every decode step
            hit = (version, (aq, ao), (aq.float(), ao.float()))
            self.__dict__["_absorbed_cache"] = hit
        return hit[1]

    def _absorbed_f32(self) -> tuple[Tensor, Tensor]:
        """``_absorbed()`` as fp32 tensors (the bf16-rounded values, exactly)."""
        self._absorbed()
        return self.__dict__["_absorbed_cache"][2]

    def decode(self, x: Tensor, cache: MLALatentCache, position: int,
               addend: Tensor | None = None, defer_sum: bool = False,
               position_device: Tensor | None = None) -> Tensor:
        if x.shape[1] != 1:
            raise ValueError("decode expects one model position")
        if defer_sum:
            raise RuntimeError("deferred attention reduction is not part of the b200 backend")
        c = self.cfg
        b = x.shape[0]
        aq, ao = self._absorbed_f32()
        if position_device is not None:
            # absorbed latent attention at the device position (capturable):
            # fp32 query over the bf16 latent cache, fp32 context (model.py:417-432)
            small = b <= _SMALL_LINEAR_ROWS
            if small:
                xf = x.view(b, -1)
                latent = bridge.b200_linear_small(xf, self.kv_down.weight, x.dtype)
                q = bridge.b200_linear_small(xf, aq, torch.float32)  # x.float() is exact
            else:
                latent = self.kv_down(x).view(b, -1)
                q = F.linear(x.float(), aq).view(b, -1)
            ctx = bridge.b200_decode_attention(
                q, latent, None, cache.latent.unsqueeze(1), None, position_device, c.n_heads, 1,
                c.kv_latent_dim, 0, c.head_dim ** -0.5, torch.float32)
            out = (bridge.b200_linear_small(ctx, ao, x.dtype).view(b, 1, -1) if small
                   else F.linear(ctx.view(b, 1, -1), ao).to(x.dtype))
            return out if addend is None else addend + out
        cache.latent[:, position:position + 1].copy_(self.kv_down(x))
        seen = cache.latent[:, :position + 1]
        q = F.linear(x.float(), aq).view(b, 1, c.n_heads, c.kv_latent_dim).transpose(1, 2)
        # the absorbed query is fp32 (model.py:420); attend over the latents in fp32 too
        kv = seen[:, None].expand(-1, c.n_heads, -1, -1).float()
        with sdpa_kernel(_DECODE_SDPA):
            ctx = F.scaled_dot_product_attention(q, kv, kv, scale=c.head_dim ** -0.5)
        ctx = ctx.transpose(1, 2).reshape(b, 1, c.n_heads * c.kv_latent_dim)
        out = F.linear(ctx, ao).to(x.dtype)
        return out if addend is None else addend + out


class SwiGLU(nn.Module):
    """Expert parameters in ``nn.Linear`` layout (``model.py:435-448``)."""

    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.gate = nn.Linear(dim, hidden, bias=False)
        self.up = nn.Linear(dim, hidden, bias=False)
        self.down = nn.Linear(hidden, dim, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        return self.down(F.silu(self.gate(x)) * self.up(x))


class MoE(nn.Module):
    """Top-2 routed SwiGLU experts + shared expert on the B200 kernels (``model.py:463-607``).

    Parameters keep the reference's ``moe_backend="pytorch"`` layout; packed
    copies for the kernels are cached by ``bridge.pack_weights``.
    ``router_bias`` (not a parameter, default None) is a harness-only fp32
    logit offset used by the skewed-routing stress workload.
    """

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.router = nn.Linear(cfg.dim, cfg.n_experts, bias=False)
        self.experts = nn.ModuleList([SwiGLU(cfg.dim, cfg.expert_dim)
                                      for _ in range(cfg.n_experts)])
        self.shared = SwiGLU(cfg.dim, cfg.shared_expert_dim)
        self.router_bias: Tensor | None = None

    def forward(self, x: Tensor, addend: Tensor | None = None, *, defer_combine: bool = False):
        """``(out, aux, utilization)``; ``out`` includes ``addend`` when given.

        ``defer_combine``: ``out`` may be a ``bridge.PendingMoE`` whose
        combine the next depth mix performs.
        """
        flat = x.reshape(-1, x.shape[-1])
        if defer_combine:
            return bridge.b200_moe_deferred(self, flat, self.cfg.collect_router_stats, addend,
                                            x.shape)
        out, aux, util = bridge.b200_moe(self, flat, self.cfg.collect_router_stats, addend)
        return out.view_as(x), aux, util

    def inference(self, x: Tensor, *, direct: bool, addend: Tensor | None = None,
                  defer_sum: bool = False, defer_combine: bool = False):
        if defer_sum:
            raise ValueError("deferred MoE reduction is not part of the b200 backend")
        flat = x.reshape(-1, x.shape[-1])
        if defer_combine:
            return bridge.b200_moe_deferred(self, flat, False, addend, x.shape)[0]
        out, _, _ = bridge.b200_moe(self, flat, False, addend)
        return out.view_as(x)


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig, index: int):
        super().__init__()
        is_global = (index + 1) % cfg.global_every == 0
        self.attention = GlobalMLA(cfg) if is_global else LocalGQA(cfg)
        self.moe = MoE(cfg)
        self.attention_norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.moe_norm = RMSNorm(cfg.dim, cfg.norm_eps)

    def attend(self, x):
        return self.attention(self.attention_norm(x))

    def feedforward(self, x):
        return self.moe(self.moe_norm(x))

    def feedforward_inference(self, x, *, direct: bool):
        return self.moe.inference(self.moe_norm(x), direct=direct)


class _Residuals:
    """Block AttnRes bookkeeping (``model.py:680-705``) with one deferred add.

    ``pending`` holds an attention output not yet added to ``partial``; the
    next depth-mix kernel performs that add while it reads the sources.  The
    last source itself (``partial``, or the last completed block) may be a
    ``bridge.PendingMoE``: an MoE output whose combine the next depth mix
    performs.
    """

    def __init__(self, first: Tensor, block: int):
        self.completed = [first]
        self.partial: Tensor | None = None
        self.pending: Tensor | None = None
        self.block = block

    def sources(self) -> list[Tensor]:
        return self.completed + ([] if self.partial is None else [self.partial])

    def mix(self, depth: DepthMix, norm: RMSNorm, route=None) -> Tensor:
        """The normalised depth mix feeding the next module; ``route``: that
        module when it is an MoE block (its router runs in the same kernel)."""
        sources = self.sources()
        if isinstance(sources[-1], bridge.PendingMoE):
            out, resolved = depth.normalized(sources, norm)
            if self.partial is not None:
                self.partial = resolved
            else:
                self.completed[-1] = resolved
            return out
        if self.pending is None:
            return depth.normalized(sources, norm, route=route)
        out, resolved = depth.normalized(self.sources(), norm, self.pending, route=route)
        self.partial, self.pending = resolved, None
        return out

    def add_delta(self, delta: Tensor) -> None:
        if self.partial is None:
            self.partial = delta
        else:
            self.pending = delta

    def set_partial(self, value: Tensor) -> None:
        self.partial, self.pending = value, None

    def end_module(self, index: int) -> None:
        if (index + 1) % self.block == 0:
            if self.pending is not None:
                self.partial = self.partial + self.pending
                self.pending = None
            self.completed.append(self.partial)
            self.partial = None


class Parrot(nn.Module):
    """Parrot XL with the B200 MoE/depth backend (``model.py:638-937``)."""

    def __init__(self, cfg: ModelConfig = ModelConfig()):
        super().__init__()
        self.config = cfg
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.dim)
        self.blocks = nn.ModuleList([Block(cfg, i) for i in range(cfg.n_layers)])
        self.depth_mix = nn.ModuleList(
            [DepthMix(cfg) for _ in range(2 * cfg.n_layers + 1)]
            if cfg.residual == "attnres" else [])
        self.final_norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.apply(self._init_weights)

    @staticmethod
    def _init_weights(module):
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, std=0.02)

    def forward(self, input_ids: Tensor, labels: Tensor | None = None, *, bag_size: int = 1,
                supervised_logits_only: bool = False) -> ModelOutput:
        """Same contract as the reference ``Parrot.forward`` (``model.py:658-746``)."""
        cfg = self.config
        if input_ids.ndim != 2 or input_ids.numel() == 0:
            raise ValueError("input_ids must be a nonempty [batch, source_tokens] tensor")
        if not isinstance(bag_size, int) or bag_size < 1 or input_ids.shape[1] % bag_size:
            raise ValueError("source_tokens must be divisible by positive integer bag_size")
        b, source_len = input_ids.shape
        t = source_len // bag_size
        if t > cfg.max_seq_len:
            raise ValueError("Input exceeds max_seq_len model positions")
        if labels is not None and (labels.shape != input_ids.shape or t < 2):
            raise ValueError("labels must match input_ids and contain at least two model positions")
        if supervised_logits_only and labels is None:
            raise ValueError("supervised_logits_only requires labels")
        x = self.embedding(input_ids)
        if bag_size > 1:
            x = x.reshape(b, t, bag_size, -1).mean(2)
        aux_losses, utilization = [], []
        attnres = cfg.residual == "attnres"
        res = _Residuals(x, cfg.depth_block_size)
        index = 0
        for block in self.blocks:
            for is_moe in (False, True):
                norm = block.moe_norm if is_moe else block.attention_norm
                h = res.mix(self.depth_mix[index], norm, block.moe if is_moe else None) \
                    if attnres else norm(x)
                if is_moe:
                    base = res.partial if attnres else x
                    out, aux, usage = block.moe(h, addend=base, defer_combine=attnres)
                    if cfg.collect_router_stats:
                        aux_losses.append(aux)
                        utilization.append(usage)
                    if attnres:
                        res.set_partial(out)
                    else:
                        x = out
                else:
                    delta = block.attention(h)
                    if attnres:
                        res.add_delta(delta)
                    else:
                        x = x + delta
                if attnres:
                    res.end_module(index)
                index += 1
        if attnres:
            h = res.mix(self.depth_mix[-1], self.final_norm)
        else:
            h = self.final_norm(x)
        if supervised_logits_only:
            h = h[:, :-1]
        logits = F.linear(h, self.embedding.weight)
        if cfg.collect_router_stats:
            aux_loss = torch.stack(aux_losses).mean()
            expert_utilization = torch.stack(utilization)
        else:
            aux_loss = x.new_zeros((), dtype=torch.float32)
            expert_utilization = x.new_zeros((cfg.n_layers, cfg.n_experts), dtype=torch.float32)
        lm_loss = loss = None
        if labels is not None:
            targets = labels.reshape(b, t, bag_size)[:, 1:]
            scored = (logits if supervised_logits_only else logits[:, :-1]).float()
            valid = targets != -100
            picked = scored.gather(-1, targets.masked_fill(~valid, 0))
            lse = torch.logsumexp(scored, -1)
            numerator = (lse * valid.sum(-1) - (picked * valid).sum(-1)).sum()
            lm_loss = numerator / valid.sum().clamp_min(1)
            loss = lm_loss + cfg.aux_loss_weight * aux_loss
        return ModelOutput(logits, loss, lm_loss, aux_loss, expert_utilization)

    @torch.inference_mode()
    def prefill(self, input_ids: Tensor) -> tuple[Tensor, GenerationState]:
        """Prompt pass returning last-position logits and caches (``model.py:748-815``)."""
        cfg = self.config
        if self.training:
            raise RuntimeError("prefill requires model.eval()")
        if input_ids.ndim != 2 or input_ids.shape[1] < 1:
            raise ValueError("input_ids must be nonempty [batch, positions]")
        b, t = input_ids.shape
        if t > cfg.max_seq_len:
            raise ValueError("Prompt exceeds max_seq_len")
        x = self.embedding(input_ids)
        attnres = cfg.residual == "attnres"
        res = _Residuals(x, cfg.depth_block_size)
        caches: list[LocalKVCache | MLALatentCache] = []
        index = 0
        for block in self.blocks:
            h = res.mix(self.depth_mix[index], block.attention_norm) if attnres \
                else block.attention_norm(x)
            if isinstance(block.attention, LocalGQA):
                delta, k, v = block.attention.prefill(h)
                kc = torch.empty((b, cfg.n_kv_heads, cfg.max_seq_len, cfg.head_dim),
                                 device=k.device, dtype=k.dtype)
                vc = torch.empty_like(kc)
                kc[:, :, :t].copy_(k)
                vc[:, :, :t].copy_(v)
                caches.append(LocalKVCache(kc, vc))
            else:
                delta, latent = block.attention.prefill(h)
                lc = torch.empty((b, cfg.max_seq_len, cfg.kv_latent_dim),
                                 device=latent.device, dtype=latent.dtype)
                lc[:, :t].copy_(latent)
                caches.append(MLALatentCache(lc))
            if attnres:
                res.add_delta(delta)
                res.end_module(index)
            else:
                x = x + delta
            index += 1
            h = res.mix(self.depth_mix[index], block.moe_norm, block.moe) if attnres \
                else block.moe_norm(x)
            out = block.moe.inference(h, direct=False, addend=res.partial if attnres else x,
                                      defer_combine=attnres)
            if attnres:
                res.set_partial(out)
                res.end_module(index)
            else:
                x = out
            index += 1
        h = res.mix(self.depth_mix[-1], self.final_norm) if attnres else self.final_norm(x)
        logits = F.linear(h[:, -1:], self.embedding.weight)
        position = torch.full((1,), t, device=logits.device, dtype=torch.int32)
        return logits, GenerationState(caches, t, b, position)

    @torch.inference_mode()
    def decode_step(self, input_ids: Tensor, state: GenerationState, *,
                    _next_token_only: bool = False) -> tuple[Tensor, GenerationState]:
        """Append one token to a generation state (``model.py:817-925``)."""
        cfg = self.config
        if self.training:
            raise RuntimeError("decode_step requires model.eval()")
        if input_ids.shape != (state.batch_size, 1):
            raise ValueError("decode_step input must be [cached batch, 1]")
        if state.position >= cfg.max_seq_len:
            raise ValueError("Generation state has reached max_seq_len")
        if len(state.layers) != cfg.n_layers:
            raise ValueError("Generation state does not match model depth")
        x = self.embedding(input_ids)
        attnres = cfg.residual == "attnres"
        res = _Residuals(x, cfg.depth_block_size)
        index = 0
        for layer, block in enumerate(self.blocks):
            cache = state.layers[layer]
            h = res.mix(self.depth_mix[index], block.attention_norm) if attnres \
                else block.attention_norm(x)
            if isinstance(block.attention, LocalGQA):
                if not isinstance(cache, LocalKVCache):
                    raise ValueError("Local attention received an MLA cache")
            elif not isinstance(cache, MLALatentCache):
                raise ValueError("MLA attention received a local cache")
            # the residual add is left to the next depth mix (attnres), as in forward
            delta = block.attention.decode(h, cache, state.position,
                                           position_device=state.position_device)
            if attnres:
                res.add_delta(delta)
                res.end_module(index)
            else:
                x = x + delta
            index += 1
            h = res.mix(self.depth_mix[index], block.moe_norm, block.moe) if attnres \
                else block.moe_norm(x)
            out = block.moe.inference(h, direct=True, addend=res.partial if attnres else x,
                                      defer_combine=attnres)
            if attnres:
                res.set_partial(out)
                res.end_module(index)
            else:
                x = out
            index += 1
        h = res.mix(self.depth_mix[-1], self.final_norm) if attnres else self.final_norm(x)
        if _next_token_only:
            # the projection and the argmax in one pass, no logits (model.py:927-931)
            output = bridge.b200_vocab_argmax(h, self.embedding.weight)
        else:
            output = F.linear(h, self.embedding.weight)
        state.position += 1
        if state.position_device is not None:
            state.position_device.add_(1)
        return output, state

    @torch.inference_mode()
    def decode_next(self, input_ids: Tensor, state: GenerationState):
        """Append one token and return the next greedy token (``model.py:927-931``)."""
        return self.decode_step(input_ids, state, _next_token_only=True)

    def capture_decode(self, state: GenerationState, next_token_only: bool = False):
        """CUDA-graph replay of ``decode_step`` (or ``decode_next``) on ``state``.

        Returns a ``graphs.GraphedDecode``; each call appends one token to
        ``state`` (whose caches and device position the graph captured).
        """
        from .graphs import GraphedDecode
        return GraphedDecode(self, state, next_token_only)

    def capture(self, batch: int, source_len: int, **forward_kwargs):
        """CUDA-graph replay of ``forward`` for one input shape.

        Returns a ``graphs.GraphedForward``; calling it with ``[batch,
        source_len]`` ids (host or device) runs the captured forward.
        """
        from .graphs import GraphedForward
        return GraphedForward(self, batch, source_len, **forward_kwargs)

    def parameter_counts(self) -> dict[str, int]:
        total = sum(p.numel() for p in self.parameters())
        inactive = (self.config.n_layers * (self.config.n_experts - self.config.top_k)
                    * 3 * self.config.dim * self.config.expert_dim)
        return {"total": total, "active_per_token": total - inactive}
