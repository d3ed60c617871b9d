"""The energy network E(z; x) and its latent descent: the caller of the attention path.

This restates the parts of the reference's model code that drive the hot path, with the same shapes, dtypes and
call semantics, so the benchmark exercises the sm_100a attention exactly as the reference's training and evaluation
loops do:

* ``rms_norm`` / ``CastedLinear`` / ``CastedEmbedding`` / ``SwiGLU`` / 2D RoPE: ``models/layers.py:37-132``;
* ``EnergyAttention``: qkv projection, 2D RoPE, per-head temperature ``exp(log_logit_scale)``, attention on
  ``[B, H, N, D]`` views, o projection (``models/attention.py:181-242``); post-norm block
  (``models/attention.py:248-266``);
* ``ScalarEnergy`` = sum over cells of a per-cell head on top of the blocks (``models/energy.py:190-216``);
* ``EnergyDescent.forward``: one microstep ``z <- sphere(rms_norm(z) + sigma * eps - alpha * dE/dv)`` with
  ``create_graph`` in graded (training) microsteps (``models/energy.py:219-222``, ``:285-350``);
* ``descend`` runs a segment of microsteps; ``lowest_energy_pick`` keeps the lowest-energy sample of each input
  (``evaluators/protocol.py:10-12``).

The attention is ``ebr_b200.fused_attn.fused_attention`` unless a caller injects another callable with the same
signature (the CPU baseline of the benchmark injects the oracle there); there is no backend registry or fallback.

``EnergyConfig.layers`` picks how the layers around the attention run: ``"fused"`` (CUDA: the kernels of
``ebr_b200.layers`` -- the 2D-RoPE split / merge, residual + rms_norm, the SwiGLU activation, and the pointwise ops of
inference microsteps) or ``"eager"`` (plain torch ops, the reference's ``rope_impl: eager`` code; the CPU model and
the parity yardstick). As in the reference (``models/attention.py:215-242``), the per-head temperature is folded into
the RoPE split only outside the graded window, where log_logit_scale needs no gradient.
"""

from __future__ import annotations

import contextlib
import math
import threading
from dataclasses import dataclass
from typing import Callable

import torch
import torch.nn.functional as F
from torch import nn

from ebr_b200 import layers as fl
from ebr_b200.fused_attn import fused_attention

RMS_NORM_EPS = 1e-5
ROPE_THETA = 10000.0

AttentionFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def _fused(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return fused_attention(q, k, v, scale=q.shape[-1] ** -0.5)


_window = threading.local()


@contextlib.contextmanager
def second_order_window(enabled: bool):
    """Mark the energy evaluations inside as graded (their dE/dz is differentiated again), thread-locally
    (``models/attention.py:22-37``)."""
    prev = getattr(_window, "graded", False)
    _window.graded = enabled
    try:
        yield
    finally:
        _window.graded = prev


def second_order_required() -> bool:
    return getattr(_window, "graded", False)


# ------------------------------------------------------------------------------------------------------------ layers


def trunc_normal_(t: torch.Tensor, std: float = 1.0, lower: float = -2.0, upper: float = 2.0) -> torch.Tensor:
    """Normal truncated to [lower, upper] standard deviations, rescaled to standard deviation ``std``."""
    with torch.no_grad():
        if std == 0:
            return t.zero_()
        sqrt2 = math.sqrt(2.0)
        a, b = math.erf(lower / sqrt2), math.erf(upper / sqrt2)
        z = (b - a) / 2.0
        c = (2.0 * math.pi) ** -0.5
        pdf_u, pdf_l = c * math.exp(-0.5 * lower**2), c * math.exp(-0.5 * upper**2)
        comp_std = std / math.sqrt(1.0 - (upper * pdf_u - lower * pdf_l) / z - ((pdf_u - pdf_l) / z) ** 2)
        t.uniform_(a, b).erfinv_().mul_(sqrt2 * comp_std).clip_(lower * comp_std, upper * comp_std)
        return t


def rms_norm(x: torch.Tensor, eps: float = RMS_NORM_EPS) -> torch.Tensor:
    """Unit RMS over the last dim, computed in float32, returned in the input dtype."""
    dtype = x.dtype
    x = x.to(torch.float32)
    return (x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps)).to(dtype)


class CastedLinear(nn.Module):
    """Linear layer with float32 weights cast to the input dtype at use."""

    def __init__(self, fan_in: int, fan_out: int, bias: bool) -> None:
        super().__init__()
        self.weight = nn.Parameter(trunc_normal_(torch.empty(fan_out, fan_in), std=fan_in**-0.5))
        self.bias = nn.Parameter(torch.zeros(fan_out)) if bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b = self.bias.to(x.dtype) if self.bias is not None else None
        return F.linear(x, self.weight.to(x.dtype), b)


class CastedEmbedding(nn.Module):
    def __init__(self, num: int, dim: int, init_std: float, cast_to: torch.dtype) -> None:
        super().__init__()
        self.cast_to = cast_to
        self.weight = nn.Parameter(trunc_normal_(torch.empty(num, dim), std=init_std))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        return F.embedding(ids, self.weight.to(self.cast_to))


class SwiGLU(nn.Module):
    def __init__(self, hidden: int, expansion: float, fused: bool = False) -> None:
        super().__init__()
        inter = round(expansion * hidden * 2 / 3)
        inter = -(inter // -256) * 256
        self.gate_up = CastedLinear(hidden, 2 * inter, bias=False)
        self.down = CastedLinear(inter, hidden, bias=False)
        self.fused = fused

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.fused:
            return self.down(fl.gate_up_swiglu(x, self.gate_up.weight.to(x.dtype)))
        gate, up = self.gate_up(x).chunk(2, dim=-1)
        return self.down(F.silu(gate) * up)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2 :]
    return torch.cat((-x2, x1), dim=-1)


class Rope2D(nn.Module):
    """2D RoPE over a height x width board: the first half of each head's channels rotates with the row, the second
    half with the column."""

    def __init__(self, head_dim: int, height: int, width: int, base: float = ROPE_THETA) -> None:
        super().__init__()
        half = head_dim // 2
        inv = 1.0 / (base ** (torch.arange(0, half, 2, dtype=torch.float32) / half))
        rows = torch.outer(torch.arange(height, dtype=torch.float32), inv)
        cols = torch.outer(torch.arange(width, dtype=torch.float32), inv)
        rows, cols = torch.cat((rows, rows), -1), torch.cat((cols, cols), -1)
        self.height, self.width = height, width
        self.register_buffer("cos_h", rows.cos(), persistent=False)
        self.register_buffer("sin_h", rows.sin(), persistent=False)
        self.register_buffer("cos_w", cols.cos(), persistent=False)
        self.register_buffer("sin_w", cols.sin(), persistent=False)
        # The same angles as [height * width, D] tables for the fused split (sign of rotate_half folded into sin).
        cos_t, sin_t = fl.rotary_tables(self.cos_h, self.sin_h, self.cos_w, self.sin_w)
        self.register_buffer("cos_table", cos_t, persistent=False)
        self.register_buffer("sin_table", sin_t, persistent=False)

    def apply(self, q: torch.Tensor, k: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """q, k: [B, N, heads, D] with N = height * width."""
        ch, sh = self.cos_h[None, :, None, None, :], self.sin_h[None, :, None, None, :]
        cw, sw = self.cos_w[None, None, :, None, :], self.sin_w[None, None, :, None, :]

        def rot(x: torch.Tensor) -> torch.Tensor:
            b, n, heads, d = x.shape
            g = x.reshape(b, self.height, self.width, heads, d).to(ch.dtype)
            r, c = g[..., : d // 2], g[..., d // 2 :]
            r = r * ch + _rotate_half(r) * sh
            c = c * cw + _rotate_half(c) * sw
            return torch.cat([r, c], -1).to(x.dtype).reshape(b, n, heads, d)

        return rot(q), rot(k)


# ------------------------------------------------------------------------------------------------------------ blocks


class EnergyAttention(nn.Module):
    def __init__(self, hidden: int, heads: int, attention: AttentionFn | None = None, fused: bool = False) -> None:
        super().__init__()
        self.heads, self.head_dim = heads, hidden // heads
        self.qkv = CastedLinear(hidden, 3 * hidden, bias=False)
        self.o = CastedLinear(hidden, hidden, bias=False)
        self.log_logit_scale = nn.Parameter(torch.zeros(heads))
        self.attention = attention or _fused
        self.fused = fused

    def forward(self, rope: Rope2D, x: torch.Tensor) -> torch.Tensor:
        b, n, _ = x.shape
        h, d = self.heads, self.head_dim
        temperature_applied = False
        if self.fused:
            # One kernel: the projection GEMM with split + 2D RoPE + head-major layout (+ the temperature outside the
            # graded window) as its epilogue.
            qscale = None
            if not second_order_required():
                qscale = self.log_logit_scale.detach().exp().to(x.dtype)
                temperature_applied = True
            q, k, v = fl.qkv_rope_split(x, self.qkv.weight.to(x.dtype), rope.cos_table, rope.sin_table, h, qscale)
        else:
            q, k, v = self.qkv(x).split([h * d] * 3, dim=-1)
            q, k, v = q.view(b, n, h, d), k.view(b, n, h, d), v.view(b, n, h, d)
            q, k = rope.apply(q, k)
            q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if not temperature_applied:
            q = q * self.log_logit_scale.exp().to(q.dtype).view(1, -1, 1, 1)
        y = self.attention(q, k, v)
        if self.fused:
            # The projection reads the head-major attention output directly (no transpose copy).
            return fl.o_proj(y, self.o.weight.to(y.dtype))
        return self.o(y.transpose(1, 2).reshape(b, n, h * d))


class Block(nn.Module):
    def __init__(self, hidden: int, heads: int, expansion: float, attention: AttentionFn | None = None,
                 fused: bool = False) -> None:  # fmt: skip
        super().__init__()
        self.attn = EnergyAttention(hidden, heads, attention, fused)
        self.mlp = SwiGLU(hidden, expansion, fused)
        self.fused = fused

    def forward(self, rope: Rope2D, x: torch.Tensor) -> torch.Tensor:
        if self.fused:
            x = fl.add_rms_norm(x, self.attn(rope, x), RMS_NORM_EPS)
            return fl.add_rms_norm(x, self.mlp(x), RMS_NORM_EPS)
        x = rms_norm(x + self.attn(rope, x))
        return rms_norm(x + self.mlp(x))


class ScalarEnergy(nn.Module):
    """E(z, x): blocks over z + x, then the sum over cells of a per-cell scalar head. Returns [B] float32."""

    def __init__(self, hidden: int, heads: int, layers: int, expansion: float, softplus: bool,
                 attention: AttentionFn | None = None, fused: bool = False) -> None:  # fmt: skip
        super().__init__()
        self.blocks = nn.ModuleList(Block(hidden, heads, expansion, attention, fused) for _ in range(layers))
        self.head_hidden = CastedLinear(hidden, hidden, bias=True)
        self.head_out = CastedLinear(hidden, 1, bias=False)
        self.softplus = softplus

    def forward(self, z: torch.Tensor, x: torch.Tensor, rope: Rope2D) -> torch.Tensor:
        h = z + x
        for blk in self.blocks:
            h = blk(rope, h)
        raw = self.head_out(F.silu(self.head_hidden(h)))
        if self.softplus:
            raw = F.softplus(raw.to(torch.float32))
        return raw.to(torch.float32).squeeze(-1).sum(dim=1)


def sphere(z: torch.Tensor, eps: float = RMS_NORM_EPS) -> torch.Tensor:
    """Rescale each row (the whole board) to unit RMS, in float32."""
    rms = z.to(torch.float32).square().mean(dim=(1, 2), keepdim=True).sqrt().clamp_min(eps)
    return (z.to(torch.float32) / rms).to(z.dtype)


# ------------------------------------------------------------------------------------------------------------ model


@dataclass
class EnergyConfig:
    """The benchmark architecture: 4 layers, hidden 512, 8 heads x 64, SwiGLU 4x."""

    board_height: int = 9
    board_width: int = 9
    vocab_size: int = 10
    hidden_size: int = 512
    num_heads: int = 8
    num_layers: int = 4
    expansion: float = 4.0
    forward_dtype: torch.dtype = torch.bfloat16
    softplus: bool = False
    step_size: float = 250.0
    noise_scale: float = 0.05
    init_std: float = 1.0
    layers: str = "fused"  # "fused" (CUDA kernels around the attention) or "eager" (torch ops; CPU)

    @property
    def seq_len(self) -> int:
        return self.board_height * self.board_width


class EnergyReasoner(nn.Module):
    """Token embedding + energy + one descent microstep (``models/energy.py:264-319``, ``:447-490``)."""

    def __init__(self, cfg: EnergyConfig, attention: AttentionFn | None = None) -> None:
        super().__init__()
        self.cfg = cfg
        self.embed_scale = math.sqrt(cfg.hidden_size)
        self.embed = CastedEmbedding(cfg.vocab_size, cfg.hidden_size, 1.0 / self.embed_scale, cfg.forward_dtype)
        self.lm_head = CastedLinear(cfg.hidden_size, cfg.vocab_size, bias=False)
        self.rope = Rope2D(cfg.hidden_size // cfg.num_heads, cfg.board_height, cfg.board_width)
        if cfg.layers not in ("fused", "eager"):
            raise ValueError(f"EnergyConfig.layers must be 'fused' or 'eager', got {cfg.layers!r}")
        self.fused = cfg.layers == "fused"
        self.energy = ScalarEnergy(cfg.hidden_size, cfg.num_heads, cfg.num_layers, cfg.expansion, cfg.softplus,
                                   attention, self.fused)  # fmt: skip

    def input_embeddings(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.embed_scale * self.embed(tokens.to(torch.int32))

    def fresh_states(self, rows: int, device, generator: torch.Generator | None = None) -> torch.Tensor:
        shape = (rows, self.cfg.seq_len, self.cfg.hidden_size)
        z = torch.empty(shape, device=device, dtype=torch.float32)
        if generator is None:
            trunc_normal_(z, std=self.cfg.init_std)
        else:
            z.normal_(generator=generator).clamp_(-2.0, 2.0)
        return z.to(self.cfg.forward_dtype)

    def energy_and_grad(self, v: torch.Tensor, x: torch.Tensor, create_graph: bool):
        """E(v, x) per row and dE/dv (``_energy_gradient``, ``models/energy.py:345-350``)."""
        with torch.enable_grad(), second_order_window(create_graph):
            if not v.requires_grad:
                v = v.detach().requires_grad_(True)
            e = self.energy(v, x, self.rope)
            (g,) = torch.autograd.grad(e.sum(), v, create_graph=create_graph)
        return e, g, v

    def microstep(self, z: torch.Tensor, x: torch.Tensor, *, graded: bool, noise: torch.Tensor | None = None,
                  sigma: float | None = None, alpha: float | torch.Tensor | None = None):  # fmt: skip
        """One descent microstep from ``z``; returns (z_next, E(v) per row)."""
        cfg = self.cfg
        sigma = cfg.noise_scale if sigma is None else sigma
        step = cfg.step_size if alpha is None else alpha
        if self.fused and not graded and not torch.is_tensor(step):
            # Inference microstep: v = rms_norm(z) + noise and z' = sphere(v - alpha g) as fused kernels.
            if noise is not None:
                v = fl.noisy_point(z, noise, 1.0, RMS_NORM_EPS)
            elif sigma:
                v = fl.noisy_point(z, torch.randn_like(z), float(sigma), RMS_NORM_EPS)
            else:
                v = fl.noisy_point(z, None, 0.0, RMS_NORM_EPS)
            e, g, v = self.energy_and_grad(v, x, create_graph=False)
            return fl.step_and_project(v.detach(), g, float(step), RMS_NORM_EPS), e.detach()
        v = rms_norm(z)
        if noise is not None:
            v = v + noise.to(v.dtype)
        elif sigma:
            v = v + torch.randn_like(v) * sigma
        e, g, v = self.energy_and_grad(v, x, create_graph=graded)
        z_next = sphere(v - step * g)
        return (z_next, e) if graded else (z_next.detach(), e.detach())

    def decode(self, z: torch.Tensor) -> torch.Tensor:
        return self.lm_head(z)


@torch.no_grad()
def lowest_energy_pick(energy: torch.Tensor, samples: int) -> torch.Tensor:
    """energy [inputs * samples] (an input's samples contiguous) -> index of each input's lowest-energy sample."""
    return energy.view(-1, samples).argmin(dim=1)


def descend(model: EnergyReasoner, z: torch.Tensor, x: torch.Tensor, steps: int, *, sigma: float | None = None,
            noises: list[torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:  # fmt: skip
    """``steps`` no-graph microsteps (inference: forward + first-order dE/dz each). Returns (z, last energies)."""
    e = None
    for t in range(steps):
        z, e = model.microstep(z, x, graded=False, sigma=sigma, noise=None if noises is None else noises[t])
    return z, e


def train_step_loss(model: EnergyReasoner, z: torch.Tensor, x: torch.Tensor, labels: torch.Tensor,
                    prefix: int, graded: int, alpha: torch.Tensor | None = None) -> torch.Tensor:  # fmt: skip
    """A training segment: ``prefix`` no-graph microsteps, then ``graded`` microsteps with ``create_graph=True``
    (double backward through the attention), and cross-entropy of the decoded endpoint against ``labels``."""
    for _ in range(prefix):
        z, _ = model.microstep(z, x, graded=False, alpha=alpha)
    for _ in range(graded):
        z, _ = model.microstep(z, x, graded=True, alpha=alpha)
    logits = model.decode(rms_norm(z)).float()
    return F.cross_entropy(logits.flatten(0, 1), labels.flatten().long())
