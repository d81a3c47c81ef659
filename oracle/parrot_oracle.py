"""CPU oracle for the Parrot XL MoE block and its companions.

TEST INFRASTRUCTURE ONLY.  This module restates, in plain PyTorch, the
reference's ``moe_backend="pytorch"`` / ``depth_backend="pytorch"`` algorithm
(jkpdino/parrot-h200-worker, ``parrot/model.py``).  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it, and only as the checker or the timed CPU baseline.  The product
package ``parrot_b200`` never imports it and has no CPU fallback.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference package
itself in the build container and freezes its outputs under ``tests/golden``;
``tests/test_oracle_golden.py`` checks this module against those fixtures.

The module tree (attribute names, registration order, parameter shapes) is
the same as the reference's so that ``torch.manual_seed(s); OracleParrot(cfg)``
draws exactly the reference's seeded weights and ``state_dict`` keys match
(``model.py:109-164, 167-174, 337-345, 435-441, 463-503, 610-617, 638-656``).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
from torch import Tensor, nn
from torch.nn import functional as F


# ---------------------------------------------------------------------------
# configuration (model.py:15-82, pytorch backends only)
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class OracleConfig:
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
    residual: str = "attnres"
    depth_block_size: int = 4
    rope_theta: float = 10000.0
    norm_eps: float = 1e-6
    aux_loss_weight: float = 0.01
    collect_router_stats: bool = True
    local_query_chunk: int = 256


def tiny_config(**overrides) -> OracleConfig:
    """Frozen stand-in for the reference's missing ``example.py --tiny``."""
    base = dict(vocab_size=32768, dim=128, n_layers=4, n_heads=4, n_kv_heads=2,
                head_dim=32, kv_latent_dim=32, n_experts=8, top_k=2,
                expert_dim=128, shared_expert_dim=64, window_size=128,
                max_seq_len=512)
    base.update(overrides)
    return OracleConfig(**base)


# ---------------------------------------------------------------------------
# grouping contract (model.py:547-548 order; metal_moe.py:388-391 capacity)
# ---------------------------------------------------------------------------
def expert_capacity(assignments: int, n_experts: int) -> int:
    """Per-expert slot count: twice the balanced load, rounded up to 8, >= 8.

    Follows ``metal_moe.py:388-391``.
    """
    balanced = (2 * assignments + n_experts - 1) // n_experts
    return max(8, (balanced + 7) // 8 * 8)


@dataclass
class Grouping:
    counts: "list[int]"          # assignments per expert
    slots: "list[int]"           # [A] rank of assignment a within its expert
    capacity: int
    order: "list[list[int]]" = field(default_factory=list)  # per expert: assignment ids


def group_assignments(indices, n_experts: int, capacity: int | None = None) -> Grouping:
    """Stable counting sort of top-k assignments by expert.

    ``indices`` is ``[T, k]``.  Assignment ``a = t * k + j``.  Within one
    expert, assignments are ranked in ascending ``a`` — the order
    ``torch.where(indices == e)`` yields (``model.py:548``).  Slots at or past
    ``capacity`` are the exact overflow path (``moe_bf16.metal:678-777``).
    """
    import numpy as np
    flat = np.asarray(indices).reshape(-1).astype(np.int64)
    a_total = flat.shape[0]
    if capacity is None:
        capacity = expert_capacity(a_total, n_experts)
    counts = np.zeros(n_experts, dtype=np.int64)
    slots = np.empty(a_total, dtype=np.int64)
    order: list[list[int]] = [[] for _ in range(n_experts)]
    for a in range(a_total):
        e = int(flat[a])
        slots[a] = counts[e]
        counts[e] += 1
        order[e].append(a)
    return Grouping(counts.tolist(), slots.tolist(), capacity, order)


def grouped_rows(grouping: Grouping, indices) -> "list[int]":
    """Row of each assignment in the [E*C + A, d] grouped buffer.

    In-capacity slots land at ``e*C + slot``; overflow slots are packed per
    expert after the capacity region, experts in ascending order.
    """
    import numpy as np
    flat = np.asarray(indices).reshape(-1).astype(np.int64)
    n_experts = len(grouping.counts)
    cap = grouping.capacity
    overflow_base = np.zeros(n_experts + 1, dtype=np.int64)
    for e in range(n_experts):
        overflow_base[e + 1] = overflow_base[e] + max(grouping.counts[e] - cap, 0)
    rows = []
    for a, e in enumerate(flat.tolist()):
        s = grouping.slots[a]
        if s < cap:
            rows.append(e * cap + s)
        else:
            rows.append(n_experts * cap + int(overflow_base[e]) + s - cap)
    return rows


# ---------------------------------------------------------------------------
# modules
# ---------------------------------------------------------------------------
class RMSNorm(nn.Module):
    """``model.py:109-127``: fp32 statistics, one rounding to the input dtype."""

    def __init__(self, dim: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x: Tensor) -> Tensor:
        h = x.float()
        inv = torch.rsqrt(h.square().mean(-1, keepdim=True) + self.eps)
        return ((h * inv) * self.weight.float()).to(x.dtype)


class DepthMix(nn.Module):
    """Block AttnRes mixing, ``model.py:130-164`` (pytorch path :149-155)."""

    def __init__(self, cfg: OracleConfig):
        super().__init__()
        self.cfg = cfg
        self.query = nn.Parameter(torch.zeros(cfg.dim))
        self.norm = RMSNorm(cfg.dim, cfg.norm_eps)

    def forward(self, sources: list[Tensor]) -> Tensor:
        stacked = torch.stack(sources, 0)
        keys = F.rms_norm(stacked, (self.cfg.dim,), self.norm.weight, self.norm.eps)
        logits = (keys.float() * self.query.float()).sum(-1)
        alpha = logits.softmax(0).to(stacked.dtype)
        return (alpha[..., None] * stacked).sum(0)

    def normalized(self, sources: list[Tensor], output_norm: RMSNorm) -> Tensor:
        return output_norm(self(sources))


def _rope_tables(cfg: OracleConfig, device, dtype):
    """fp32 angles, cast to the activation dtype (``model.py:176-204``)."""
    half = torch.arange(0, cfg.head_dim, 2, device=device).float() / cfg.head_dim
    inv_freq = cfg.rope_theta ** (-half)
    pos = torch.arange(cfg.max_seq_len, device=device).float()
    ang = pos[:, None] * inv_freq
    return ang.cos().to(dtype), ang.sin().to(dtype)


def _apply_rope(cfg: OracleConfig, x: Tensor, start: int) -> Tensor:
    """Interleaved-pair rotation (``model.py:206-216``)."""
    cos, sin = _rope_tables(cfg, x.device, x.dtype)
    stop = start + x.shape[-2]
    if stop > cfg.max_seq_len:
        raise ValueError("RoPE position exceeds max_seq_len")
    c, s = cos[start:stop], sin[start:stop]
    ev, od = x[..., 0::2], x[..., 1::2]
    return torch.stack((ev * c - od * s, ev * s + od * c), -1).flatten(-2)


class LocalGQA(nn.Module):
    """Sliding-window RoPE GQA (``model.py:167-328``)."""

    def __init__(self, cfg: OracleConfig):
        super().__init__()
        self.cfg = cfg
        self.q = nn.Linear(cfg.dim, cfg.n_heads * cfg.head_dim, bias=False)
        self.k = nn.Linear(cfg.dim, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.v = nn.Linear(cfg.dim, cfg.n_kv_heads * cfg.head_dim, bias=False)
        self.out = nn.Linear(cfg.n_heads * cfg.head_dim, cfg.dim, bias=False)

    def _heads(self, y: Tensor, n: int) -> Tensor:
        b, t, _ = y.shape
        return y.view(b, t, n, self.cfg.head_dim).transpose(1, 2)

    def prefill(self, x: Tensor):
        c = self.cfg
        b, t, _ = x.shape
        q = _apply_rope(c, self._heads(self.q(x), c.n_heads), 0)
        k = _apply_rope(c, self._heads(self.k(x), c.n_kv_heads), 0)
        v = self._heads(self.v(x), c.n_kv_heads)
        if t <= c.window_size and t <= c.local_query_chunk:
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
        else:
            # query chunks attend to the last window_size keys (model.py:274-294)
            parts = []
            for start in range(0, t, c.local_query_chunk):
                stop = min(t, start + c.local_query_chunk)
                lo = max(0, start - c.window_size + 1)
                qi = torch.arange(start, stop, device=x.device)[:, None]
                ki = torch.arange(lo, stop, device=x.device)[None, :]
                mask = (ki <= qi) & (ki > qi - c.window_size)
                parts.append(F.scaled_dot_product_attention(
                    q[:, :, start:stop], k[:, :, lo:stop], v[:, :, lo:stop],
                    attn_mask=mask, enable_gqa=True))
            y = torch.cat(parts, 2)
        y = y.transpose(1, 2).reshape(b, t, -1)
        return self.out(y), k, v

    def forward(self, x: Tensor) -> Tensor:
        return self.prefill(x)[0]

    def decode(self, x: Tensor, cache: "OracleKV", position: int, addend=None):
        """One position against the cached window (``model.py:303-328``)."""
        c = self.cfg
        b = x.shape[0]
        w = torch.cat([self.q.weight, self.k.weight, self.v.weight], 0)
        qkv = F.linear(x, w)
        qw, kw = c.n_heads * c.head_dim, c.n_kv_heads * c.head_dim
        ql, kl, vl = qkv.split((qw, kw, kw), -1)
        q = _apply_rope(c, ql.view(b, 1, c.n_heads, c.head_dim).transpose(1, 2), position)
        k = _apply_rope(c, kl.view(b, 1, c.n_kv_heads, c.head_dim).transpose(1, 2), position)
        v = vl.view(b, 1, c.n_kv_heads, c.head_dim).transpose(1, 2)
        cache.key[:, :, position:position + 1].copy_(k)
        cache.value[:, :, position:position + 1].copy_(v)
        lo = max(0, position - c.window_size + 1)
        y = F.scaled_dot_product_attention(
            q, cache.key[:, :, lo:position + 1], cache.value[:, :, lo:position + 1],
            enable_gqa=True)
        out = self.out(y.transpose(1, 2).reshape(b, 1, -1))
        return out if addend is None else addend + out


class GlobalMLA(nn.Module):
    """NoPE latent attention (``model.py:331-432``)."""

    def __init__(self, cfg: OracleConfig):
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

        def split(y):
            return y.view(b, t, c.n_heads, c.head_dim).transpose(1, 2)

        latent = self.kv_down(x)
        y = F.scaled_dot_product_attention(
            split(self.q(x)), split(self.k_up(latent)), split(self.v_up(latent)),
            is_causal=True)
        return self.out(y.transpose(1, 2).reshape(b, t, -1)), latent

    def forward(self, x: Tensor) -> Tensor:
        return self.prefill(x)[0]

    def _absorbed(self):
        """Query/output absorption of the latent up-projections (``model.py:362-397``)."""
        c = self.cfg
        wq = self.q.weight.float().view(c.n_heads, c.head_dim, c.dim)
        wk = self.k_up.weight.float().view(c.n_heads, c.head_dim, c.kv_latent_dim)
        wv = self.v_up.weight.float().view(c.n_heads, c.head_dim, c.kv_latent_dim)
        wo = self.out.weight.float().view(c.dim, c.n_heads, c.head_dim).permute(1, 2, 0)
        aq = torch.einsum("hdl,hdm->hlm", wk, wq).reshape(
            c.n_heads * c.kv_latent_dim, c.dim).to(self.q.weight.dtype)
        ao = torch.einsum("hdl,hdm->hlm", wv, wo).permute(2, 0, 1).reshape(
            c.dim, c.n_heads * c.kv_latent_dim).to(self.q.weight.dtype)
        return aq, ao

    def decode(self, x: Tensor, cache: "OracleLatent", position: int, addend=None):
        c = self.cfg
        b = x.shape[0]
        aq, ao = self._absorbed()
        cache.latent[:, position:position + 1].copy_(self.kv_down(x))
        seen = cache.latent[:, :position + 1]
        ql = F.linear(x.float(), aq.float()).view(b, 1, c.n_heads, c.kv_latent_dim).transpose(1, 2)
        kv = seen[:, None].expand(-1, c.n_heads, -1, -1)
        ctx = F.scaled_dot_product_attention(ql, kv, kv, scale=c.head_dim ** -0.5)
        ctx = ctx.transpose(1, 2).reshape(b, 1, c.n_heads * c.kv_latent_dim)
        out = F.linear(ctx, ao.float()).to(x.dtype)
        return out if addend is None else addend + out


class SwiGLU(nn.Module):
    """``down(silu(gate x) * up x)`` (``model.py:435-448``)."""

    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.gate = nn.Linear(dim, hidden, bias=False)
        self.up = nn.Linear(dim, hidden, bias=False)
        self.down = nn.Linear(hidden, dim, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        return self.down(F.silu(self.gate(x)) * self.up(x))


@dataclass
class RouterTrace:
    """What the MoE router decided, for bit-exact selection/grouping checks."""
    logits: Tensor        # [T, E] fp32
    probabilities: Tensor  # [T, E] fp32
    weights: Tensor       # [T, k] fp32
    indices: Tensor       # [T, k] int64


def route(x_flat: Tensor, router_weight: Tensor, top_k: int) -> RouterTrace:
    """fp32 router, softmax, top-k, renormalise (``model.py:521-527``)."""
    logits = F.linear(x_flat.float(), router_weight.float())
    probs = logits.softmax(-1)
    w, idx = probs.topk(top_k, dim=-1)
    w = w / w.sum(-1, keepdim=True)
    return RouterTrace(logits, probs, w, idx)


class MoE(nn.Module):
    """Router + routed SwiGLU experts + shared expert (``model.py:463-607``)."""

    def __init__(self, cfg: OracleConfig):
        super().__init__()
        self.cfg = cfg
        self.router = nn.Linear(cfg.dim, cfg.n_experts, bias=False)
        self.experts = nn.ModuleList(
            [SwiGLU(cfg.dim, cfg.expert_dim) for _ in range(cfg.n_experts)])
        self.shared = SwiGLU(cfg.dim, cfg.shared_expert_dim)
        self.last_trace: RouterTrace | None = None
        self.router_bias: Tensor | None = None  # test-only logit offset (Zipf stress)

    def forward(self, x: Tensor):
        flat = x.reshape(-1, x.shape[-1])
        logits = F.linear(flat.float(), self.router.weight.float())
        if self.router_bias is not None:
            logits = logits + self.router_bias.float()
        probs = logits.softmax(-1)
        w, idx = probs.topk(self.cfg.top_k, dim=-1)
        w = w / w.sum(-1, keepdim=True)
        self.last_trace = RouterTrace(logits, probs, w, idx)
        out = self.shared(flat)
        # experts in id order; rows ascending (model.py:547-551)
        for e, expert in enumerate(self.experts):
            tok, lane = torch.where(idx == e)
            if tok.numel():
                y = expert(flat[tok]) * w[tok, lane, None].to(out.dtype)
                out = out.index_add(0, tok, y)
        if not self.cfg.collect_router_stats:
            return out.view_as(x), None, None
        counts = torch.zeros(self.cfg.n_experts, dtype=torch.float32, device=x.device)
        counts.scatter_add_(0, idx.flatten(), torch.ones(idx.numel(), device=x.device))
        util = counts / idx.numel()
        aux = self.cfg.n_experts * (util * probs.mean(0)).sum()
        return out.view_as(x), aux, util

    def inference(self, x: Tensor, addend: Tensor | None = None) -> Tensor:
        out = self.forward(x)[0]
        return out if addend is None else addend + out


class Block(nn.Module):
    def __init__(self, cfg: OracleConfig, index: int):
        super().__init__()
        is_global = (index + 1) % cfg.global_every == 0
        self.attention = GlobalMLA(cfg) if is_global else LocalGQA(cfg)
        self.moe = MoE(cfg)
        self.attention_norm = RMSNorm(cfg.dim, cfg.norm_eps)
        self.moe_norm = RMSNorm(cfg.dim, cfg.norm_eps)


@dataclass
class OracleKV:
    key: Tensor
    value: Tensor


@dataclass
class OracleLatent:
    latent: Tensor


@dataclass
class OracleState:
    layers: list
    position: int
    batch_size: int


@dataclass
class OracleOutput:
    logits: Tensor
    loss: Tensor | None
    lm_loss: Tensor | None
    aux_loss: Tensor
    expert_utilization: Tensor


class OracleParrot(nn.Module):
    """Whole-model oracle (``model.py:638-937``, pytorch backends)."""

    def __init__(self, cfg: OracleConfig = OracleConfig()):
        super().__init__()
        self.config = cfg
        self.embedding = nn.Embedding(cfg.vocab_size, cfg.dim)
        self.blocks = nn.ModuleList([Block(cfg, i) for i in range(cfg.n_layers)])
        self.depth_mix = nn.ModuleList(
            [DepthMix(cfg) for _ in range(2 * cfg.n_layers + 1)]
            if cfg.residual == "attnres" else [])
        self.final_norm = RMSNorm(cfg.dim, cfg.norm_eps)
        for m in self.modules_post_order():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, std=0.02)

    def modules_post_order(self):
        """Children before parents, like ``nn.Module.apply`` (``model.py:651``)."""
        out = []

        def walk(m):
            for child in m.children():
                walk(child)
            out.append(m)
        walk(self)
        return out

    # -- attnres bookkeeping shared by forward / prefill / decode ----------
    def _sources(self, completed, partial):
        return completed + ([] if partial is None else [partial])

    def _accumulate(self, index, completed, partial, delta):
        partial = delta if partial is None else partial + delta
        if (index + 1) % self.config.depth_block_size == 0:
            completed.append(partial)
            partial = None
        return completed, partial

    def forward(self, input_ids: Tensor, labels: Tensor | None = None, *,
                bag_size: int = 1, supervised_logits_only: bool = False) -> OracleOutput:
        cfg = self.config
        b, n_src = input_ids.shape
        t = n_src // bag_size
        x = self.embedding(input_ids).reshape(b, t, bag_size, -1).mean(2)
        completed, partial = [x], None
        aux_all, util_all = [], []
        index = 0
        for block in self.blocks:
            for is_moe in (False, True):
                if cfg.residual == "attnres":
                    h = self.depth_mix[index](self._sources(completed, partial))
                else:
                    h = x
                if is_moe:
                    delta, aux, util = block.moe(block.moe_norm(h))
                    if cfg.collect_router_stats:
                        aux_all.append(aux)
                        util_all.append(util)
                else:
                    delta = block.attention(block.attention_norm(h))
                if cfg.residual == "attnres":
                    completed, partial = self._accumulate(index, completed, partial, delta)
                else:
                    x = x + delta
                index += 1
        if cfg.residual == "attnres":
            x = self.depth_mix[-1](self._sources(completed, partial))
        head_in = x[:, :-1] if supervised_logits_only else x
        logits = F.linear(self.final_norm(head_in), self.embedding.weight)
        if cfg.collect_router_stats:
            aux_loss = torch.stack(aux_all).mean()
            utilization = torch.stack(util_all)
        else:
            aux_loss = x.new_zeros((), dtype=torch.float32)
            utilization = x.new_zeros((cfg.n_layers, cfg.n_experts), dtype=torch.float32)
        lm_loss = loss = None
        if labels is not None:
            targets = labels.reshape(b, t, bag_size)[:, 1:]
            scored = (logits if supervised_logits_only else logits[:, :-1]).float()
            valid = targets != -100
            picked = scored.gather(-1, targets.masked_fill(~valid, 0))
            lse = torch.logsumexp(scored, -1)
            num = (lse * valid.sum(-1) - (picked * valid).sum(-1)).sum()
            lm_loss = num / valid.sum().clamp_min(1)
            loss = lm_loss + cfg.aux_loss_weight * aux_loss
        return OracleOutput(logits, loss, lm_loss, aux_loss, utilization)

    @torch.inference_mode()
    def prefill(self, input_ids: Tensor):
        """``model.py:748-815``."""
        cfg = self.config
        b, t = input_ids.shape
        x = self.embedding(input_ids)
        completed, partial = [x], None
        caches = []
        index = 0
        for block in self.blocks:
            h = self.depth_mix[index].normalized(self._sources(completed, partial),
                                                  block.attention_norm)
            if isinstance(block.attention, LocalGQA):
                delta, k, v = block.attention.prefill(h)
                kc = torch.empty((b, cfg.n_kv_heads, cfg.max_seq_len, cfg.head_dim),
                                 dtype=k.dtype, device=k.device)
                vc = torch.empty_like(kc)
                kc[:, :, :t].copy_(k)
                vc[:, :, :t].copy_(v)
                caches.append(OracleKV(kc, vc))
            else:
                delta, lat = block.attention.prefill(h)
                lc = torch.empty((b, cfg.max_seq_len, cfg.kv_latent_dim),
                                 dtype=lat.dtype, device=lat.device)
                lc[:, :t].copy_(lat)
                caches.append(OracleLatent(lc))
            completed, partial = self._accumulate(index, completed, partial, delta)
            index += 1
            h = self.depth_mix[index](self._sources(completed, partial))
            delta = block.moe.inference(block.moe_norm(h))
            completed, partial = self._accumulate(index, completed, partial, delta)
            index += 1
        x = self.depth_mix[-1](self._sources(completed, partial))
        logits = F.linear(self.final_norm(x[:, -1:]), self.embedding.weight)
        return logits, OracleState(caches, t, b)

    @torch.inference_mode()
    def decode_step(self, input_ids: Tensor, state: OracleState):
        """``model.py:817-925`` (non-deferred path)."""
        x = self.embedding(input_ids)
        completed, partial = [x], None
        index = 0
        for li, block in enumerate(self.blocks):
            h = self.depth_mix[index].normalized(self._sources(completed, partial),
                                                  block.attention_norm)
            delta = block.attention.decode(h, state.layers[li], state.position, addend=partial)
            partial = delta
            if (index + 1) % self.config.depth_block_size == 0:
                completed.append(partial)
                partial = None
            index += 1
            h = self.depth_mix[index].normalized(self._sources(completed, partial),
                                                  block.moe_norm)
            partial = block.moe.inference(h, addend=partial)
            if (index + 1) % self.config.depth_block_size == 0:
                completed.append(partial)
                partial = None
            index += 1
        h = self.depth_mix[-1].normalized(self._sources(completed, partial), self.final_norm)
        logits = F.linear(h, self.embedding.weight)
        state.position += 1
        return logits, state


def oracle_threads() -> int:
    """Host threads the CPU baseline uses."""
    import os
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


__all__ = [
    "OracleConfig", "OracleParrot", "MoE", "RMSNorm", "DepthMix", "SwiGLU",
    "LocalGQA", "GlobalMLA", "route", "RouterTrace", "tiny_config",
    "expert_capacity", "group_assignments", "grouped_rows", "Grouping",
    "oracle_threads",
    "OracleKV", "OracleLatent", "OracleState", "OracleOutput",
]

