"""The reference's Block AttnRes decoder, restated as the caller of this operator.

This is the model the reference uses to measure what the operator costs inside
a real training step (``src/switchyard/model.py``): a decoder-only Transformer
whose residual stream is either the ordinary PreNorm sum (``"standard"``) or
Block AttnRes over the depth axis, evaluated either by the framework
formulation (``"attnres"``, the control) or by this package's kernels
(``"switchyard"``). Configuration fields, parameter names, the source schedule
and the arena are the reference's, so a reference checkpoint (its
``state_dict``) loads unchanged and the golden fixtures made from the
reference model pin this one (``tests/golden/make_decoder_golden.py``).

The structure (arXiv:2603.15031 as the reference reads it,
``model.py:27-57``): every Transformer layer holds two sublayers (attention,
SwiGLU), each preceded by its own Block AttnRes site (a pseudo-query ``w`` and
an RMSNorm gain ``g``); the ``2 * n_layers`` sublayers form ``n_blocks``
contiguous blocks. Sublayer ``i`` of block ``n`` attends over the completed
block representations ``blocks[0..n]`` (``blocks[0]`` is the embedding) plus,
except for a block's first sublayer, the block's running partial sum; the
site's output replaces the residual input; a final site over all blocks feeds
the LM head.

What is specific to this package (the B200 side of the integration):

* **Arena** (``sources="arena"``, ``model.py:340-369``): one ``[n_blocks + 1,
  B, T, D]`` buffer per forward holds every site's sources as one contiguous
  run, so the kernels read them in place. The running partial is staged into
  its slot by :func:`switchyard.stage_partial` -- the add and the arena write in
  one kernel instead of an add and a copy.
* **Fused site** (:class:`_ArenaSite`): in ``"switchyard"`` mode the arena's
  autograd Function launches the forward kernel on an alias of the arena and,
  in backward, restores the partial's slot, launches the backward kernel and
  the gain-split dw reduction (``dw = dq * g`` and ``dg = dq * w`` in the same
  launch) and hands each source its ``dv`` slice. No inner autograd graph, no
  ``w * g`` kernels. The reference's ``_ArenaAttnRes`` runs the operator under
  ``enable_grad`` and replays ``torch.autograd.grad`` instead; the framework
  mode here does the same, since its operator is made of autograd ops.
* ``sources="stack"`` (``torch.stack`` of the sources at every site) is kept,
  as in the reference, so the two can be compared.

This module is a caller of the operator used to measure it (step time, DDP
scaling); it is not part of the operator's API.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _sy_torch
from .arena import stage_partial
from .triton_op import DEFAULT_EPS, _BlockAttnResTriton, _forward

__all__ = [
    "DecoderConfig",
    "Decoder",
    "RESIDUAL_MODES",
    "SOURCE_MODES",
    "source_count_schedule",
    "slab_copies",
    "folded_form",
]

RESIDUAL_MODES = ("standard", "attnres", "switchyard")
SOURCE_MODES = ("arena", "stack")


@dataclass
class DecoderConfig:
    """Shape and structure (the reference's ``ModelConfig``, ``model.py:150-202``).

    The defaults are the 1.3 B benchmark model: 24 layers, hidden
    2048, 16 heads, SwiGLU 5632, 8 blocks, vocabulary 32000 (the reference's
    own default is 32768).
    """

    vocab_size: int = 32000
    d_model: int = 2048
    n_layers: int = 24
    n_heads: int = 16
    d_ff: int = 5632
    n_blocks: int = 8
    max_seq_len: int = 4096
    rope_theta: float = 10000.0
    norm_eps: float = DEFAULT_EPS
    tie_embeddings: bool = True
    residual: str = "switchyard"
    sources: str = "arena"

    def __post_init__(self) -> None:
        if self.residual not in RESIDUAL_MODES:
            raise ValueError(f"residual must be one of {RESIDUAL_MODES}, got {self.residual!r}")
        if self.sources not in SOURCE_MODES:
            raise ValueError(f"sources must be one of {SOURCE_MODES}, got {self.sources!r}")
        if self.d_model % self.n_heads:
            raise ValueError(f"d_model {self.d_model} not divisible by n_heads {self.n_heads}")
        if (2 * self.n_layers) % self.n_blocks:
            raise ValueError(
                f"n_blocks {self.n_blocks} must divide the sublayer count {2 * self.n_layers}")

    @property
    def n_sublayers(self) -> int:
        return 2 * self.n_layers

    @property
    def block_size(self) -> int:
        return self.n_sublayers // self.n_blocks

    @property
    def head_dim(self) -> int:
        return self.d_model // self.n_heads

    @property
    def uses_attnres(self) -> bool:
        return self.residual != "standard"


def source_count_schedule(n_sublayers: int, n_blocks: int) -> list[int]:
    """Sources per site in order, the readout site last (``model.py:205-219``):
    sublayer ``i`` of block ``i // block_size`` sees the ``i // block_size + 1``
    completed blocks plus the partial unless it opens its block."""
    size = n_sublayers // n_blocks
    per_sublayer = [i // size + 1 + (i % size != 0) for i in range(n_sublayers)]
    return per_sublayer + [n_blocks + 1]


def slab_copies(n_sublayers: int, n_blocks: int, sources: str) -> int:
    """``[B, T, D]`` slabs written to assemble the sources in one forward
    (``model.py:222-235``): every site's stack, or, with the arena, the
    embedding plus one partial per sublayer."""
    if sources == "stack":
        return sum(source_count_schedule(n_sublayers, n_blocks))
    return n_sublayers + 1


def folded_form(v: torch.Tensor, q: torch.Tensor, eps: float = DEFAULT_EPS) -> torch.Tensor:
    """The framework formulation the reference's ``"attnres"`` mode uses as
    its control (``src/switchyard/baselines.py:64-73``): the logits fold the
    inverse RMS in after the dot product, so ``k`` is never materialised.
    Autograd ops only (any device); not this package's operator."""
    scores = torch.einsum("d,nbtd->nbt", q, v) * torch.rsqrt(v.pow(2).mean(-1) + eps)
    return torch.einsum("nbt,nbtd->btd", scores.softmax(0), v)


# ---------------------------------------------------------------------------
# the standard pieces (identical in the three modes)
# ---------------------------------------------------------------------------


class RMSNorm(nn.Module):
    """``x * rsqrt(mean(x^2) + eps)`` (statistics in fp32) times a gain."""

    def __init__(self, d: int, eps: float) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        inv = torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + self.eps)
        return x * inv.to(x.dtype) * self.weight


def rope_tables(max_seq_len: int, head_dim: int, theta: float):
    """cos/sin of the rotary angles ``t * theta^(-2i/head_dim)``, fp32."""
    inv_freq = 1.0 / theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim)
    ang = torch.arange(max_seq_len, dtype=torch.float32)[:, None] * inv_freq[None, :]
    return ang.cos(), ang.sin()


def rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotary embedding of ``x [B, H, T, hd]`` on its two halves, in fp32."""
    a, b = x.float().chunk(2, dim=-1)
    c, s = cos[: x.shape[-2]], sin[: x.shape[-2]]
    return torch.cat([a * c - b * s, b * c + a * s], dim=-1).to(x.dtype)


class CausalSelfAttention(nn.Module):
    def __init__(self, cfg: DecoderConfig) -> None:
        super().__init__()
        self.n_heads, self.head_dim = cfg.n_heads, cfg.head_dim
        d = cfg.d_model
        self.q_proj = nn.Linear(d, d, bias=False)
        self.k_proj = nn.Linear(d, d, bias=False)
        self.v_proj = nn.Linear(d, d, bias=False)
        self.o_proj = nn.Linear(d, d, bias=False)

    def forward(self, x: torch.Tensor, rope) -> torch.Tensor:
        b, t, d = x.shape

        def heads(y):
            return y.view(b, t, self.n_heads, self.head_dim).transpose(1, 2)

        q = rotate(heads(self.q_proj(x)), *rope)
        k = rotate(heads(self.k_proj(x)), *rope)
        y = F.scaled_dot_product_attention(q, k, heads(self.v_proj(x)), is_causal=True)
        return self.o_proj(y.transpose(1, 2).reshape(b, t, d))


class SwiGLU(nn.Module):
    def __init__(self, cfg: DecoderConfig) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(cfg.d_model, cfg.d_ff, bias=False)
        self.up_proj = nn.Linear(cfg.d_model, cfg.d_ff, bias=False)
        self.down_proj = nn.Linear(cfg.d_ff, cfg.d_model, bias=False)

    def forward(self, x: torch.Tensor, rope=None) -> torch.Tensor:
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class Sublayer(nn.Module):
    def __init__(self, norm: RMSNorm, op: nn.Module) -> None:
        super().__init__()
        self.norm = norm
        self.op = op

    def forward(self, x: torch.Tensor, rope) -> torch.Tensor:
        return self.op(self.norm(x), rope)


class AttnResSite(nn.Module):
    """One site's parameters: the zero-initialised pseudo-query ``w`` (uniform
    attention at initialisation) and the RMSNorm gain ``g``; the operator
    consumes ``w * g`` (the reference's ``BlockAttnRes``,
    ``src/switchyard/reference.py:149-183``)."""

    def __init__(self, d_model: int) -> None:
        super().__init__()
        self.w = nn.Parameter(torch.zeros(d_model))
        self.g = nn.Parameter(torch.ones(d_model))


# ---------------------------------------------------------------------------
# the arena
# ---------------------------------------------------------------------------


def arena_alias(arena: torch.Tensor, n_src: int) -> torch.Tensor:
    """``arena[:n_src]`` as a tensor with its own autograd version counter
    (``set_`` onto the arena's storage): later writes to other slots do not
    invalidate it (``model.py:325-337``)."""
    out = torch.empty(0, dtype=arena.dtype, device=arena.device)
    out.set_(arena.untyped_storage(), arena.storage_offset(), (n_src, *arena.shape[1:]),
             arena.stride())
    return out


class _ArenaSite(torch.autograd.Function):
    """A Block AttnRes site over ``arena[:n_src]`` whose gradients go to the
    live source tensors (the inputs after ``eps``; they are inputs only so
    autograd accumulates into them).

    The partial's slot is rewritten by later sublayers, so it is saved and
    restored into the arena before the backward reads the sources; the graph
    orders site ``i + 1``'s backward before site ``i``'s, so every site finds
    its own bytes (the reasoning of ``model.py:87-110``).
    """

    @staticmethod
    def forward(ctx, w, g, arena, n_src, has_partial, eps, fused, *sources):
        v = arena_alias(arena, n_src)
        if fused:
            q = (w * g).contiguous()
            _, q, out, stats, _ = _forward(v, q, eps)
            ctx.save_for_backward(q, stats, w, g, *sources[-1:] if has_partial else ())
        else:
            with torch.enable_grad():
                vv = v.requires_grad_(True)
                ww = w.detach().requires_grad_(True)
                gg = g.detach().requires_grad_(True)
                out = folded_form(vv, ww * gg, eps)
            ctx.inner = (vv, ww, gg, out)
            ctx.save_for_backward(*sources[-1:] if has_partial else ())
            out = out.detach()
        ctx.arena, ctx.n_src, ctx.has_partial, ctx.eps, ctx.fused = arena, n_src, has_partial, eps, fused
        return out

    @staticmethod
    def backward(ctx, grad_out):
        saved = ctx.saved_tensors
        if ctx.has_partial:
            with torch.no_grad():
                ctx.arena[ctx.n_src - 1].copy_(saved[-1])
        if ctx.fused:
            q, stats, w, g = saved[:4]
            v = arena_alias(ctx.arena, ctx.n_src)
            # one extension call: backward kernel, then the gain-split reduction
            dv, dw, dg = _sy_torch.backward_gain(v, q, stats, grad_out, w, g, float(ctx.eps),
                                                 True, True)
        else:
            vv, ww, gg, out = ctx.inner
            ctx.inner = None
            dv, dw, dg = torch.autograd.grad(out, (vv, ww, gg), grad_out)
        return (dw, dg, None, None, None, None, None, *(dv[j] for j in range(ctx.n_src)))


# ---------------------------------------------------------------------------
# the model
# ---------------------------------------------------------------------------


class Decoder(nn.Module):
    """Decoder-only Transformer with a switchable residual mechanism (the
    reference's ``Transformer``, ``model.py:377-568``)."""

    def __init__(self, cfg: DecoderConfig) -> None:
        super().__init__()
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        ops = [op for _ in range(cfg.n_layers) for op in (CausalSelfAttention(cfg), SwiGLU(cfg))]
        self.sublayers = nn.ModuleList(Sublayer(RMSNorm(cfg.d_model, cfg.norm_eps), op) for op in ops)
        self.attn_res = (nn.ModuleList(AttnResSite(cfg.d_model) for _ in range(cfg.n_sublayers + 1))
                         if cfg.uses_attnres else None)
        self.final_norm = RMSNorm(cfg.d_model, cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        if cfg.tie_embeddings:
            self.lm_head.weight = self.embed.weight
        cos, sin = rope_tables(cfg.max_seq_len, cfg.head_dim, cfg.rope_theta)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        # N(0, 0.02) for every projection and the embedding, the residual
        # projections scaled by 1/sqrt(2 * n_layers) (model.py:410-442)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, mean=0.0, std=0.02)
        with torch.no_grad():
            for sub in self.sublayers:
                proj = sub.op.o_proj if isinstance(sub.op, CausalSelfAttention) else sub.op.down_proj
                proj.weight.mul_(1.0 / math.sqrt(2 * cfg.n_layers))
        self.last_source_counts: list[int] = []

    def forward(self, idx: torch.Tensor, targets: torch.Tensor | None = None):
        """``idx [B, T]`` -> logits ``[B, T, V]``, or ``(logits, loss)``."""
        t = idx.shape[1]
        if t > self.cfg.max_seq_len:
            raise ValueError(f"sequence length {t} exceeds max_seq_len {self.cfg.max_seq_len}")
        rope = (self.rope_cos[:t], self.rope_sin[:t])
        x0 = self.embed(idx)
        h = self._attnres_stream(x0, rope) if self.cfg.uses_attnres else self._standard(x0, rope)
        logits = self.lm_head(self.final_norm(h))
        if targets is None:
            return logits
        return logits, F.cross_entropy(logits.float().flatten(0, 1), targets.flatten())

    def _standard(self, x, rope):
        for sub in self.sublayers:
            x = x + sub(x, rope)
        self.last_source_counts = []
        return x

    def _attnres_stream(self, x0, rope):
        cfg = self.cfg
        arena = None
        if cfg.sources == "arena":
            # one per forward: a second forward before backward keeps its own
            arena = torch.empty(cfg.n_blocks + 1, *x0.shape, device=x0.device, dtype=x0.dtype)
            with torch.no_grad():
                arena[0].copy_(x0)
        fused_stage = arena is not None and cfg.residual == "switchyard"
        blocks, partial, counts = [x0], None, []
        for i, sub in enumerate(self.sublayers):
            if i and i % cfg.block_size == 0:
                blocks.append(partial)  # the partial a block ends with is its representation
                partial = None
            sources = blocks if partial is None else [*blocks, partial]
            counts.append(len(sources))
            out = sub(self._site(i, arena, sources, partial is not None), rope)
            if partial is None:
                partial = out
                if arena is not None:
                    with torch.no_grad():
                        arena[len(blocks)].copy_(out)
            elif fused_stage:
                partial = stage_partial(partial, out, arena[len(blocks)])
            else:
                partial = partial + out
                if arena is not None:
                    with torch.no_grad():
                        arena[len(blocks)].copy_(partial)
        blocks.append(partial)
        counts.append(len(blocks))
        self.last_source_counts = counts
        return self._site(cfg.n_sublayers, arena, blocks, False)

    def _site(self, i, arena, sources, has_partial):
        site = self.attn_res[i]
        eps = self.cfg.norm_eps
        fused = self.cfg.residual == "switchyard"
        if arena is not None:
            return _ArenaSite.apply(site.w, site.g, arena, len(sources), has_partial, eps, fused,
                                    *sources)
        v = torch.stack(sources, 0)
        if fused:
            if site.w.dtype == site.g.dtype:
                return _BlockAttnResTriton.apply(v, site.w, eps, site.g)
            return _BlockAttnResTriton.apply(v, site.w * site.g, eps)
        return folded_form(v, site.w * site.g, eps)
