"""CPU restatement of the reference's energy network and descent microstep.

TEST INFRASTRUCTURE ONLY: the parity tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg are the
only callers. The product network is ``ebr_b200.energy.LatentEnergyNet``; nothing in ``ebr_b200`` imports this file.

It evaluates, with plain torch ops, the reference's eager path (``rope_impl: broadcast``, no compilation) on a state
dict in the reference's own names (``models/energy.py`` ``InnerNetwork.state_dict()``):

* embedding: ``sqrt(hidden) * embedding[tokens]`` in the compute dtype (``models/energy.py:508-509``, ``:494-496``);
* block: qkv projection, 2D RoPE on q and k, per-head temperature ``q * exp(log_logit_scale)``, attention on
  ``[B, H, N, D]``, o projection, post-norm residual, SwiGLU MLP, post-norm residual (``models/attention.py:215-242``,
  ``:264-266``; ``models/layers.py:37-42``, ``:74-84``, ``:91-132``);
* energy: sum over cells of ``w2 . silu(W1 h + b1)``, softplus per cell for the non-negative head
  (``models/energy.py:190-216``);
* microstep: ``z' = sphere(rms_norm(z) + noise - alpha dE/dv)`` (``models/energy.py:219-241``, ``:285-319``).

``spec`` is a dict with ``board`` (height, width), ``hidden``, ``heads``, ``layers`` and ``softplus`` (the format of
``tests/golden/energy_case.py``). Pinned by ``tests/test_energy_cpu.py`` against the reference's own outputs in
``tests/golden/layers_golden.npz``.
"""

from __future__ import annotations

import math
from typing import Callable

import torch
import torch.nn.functional as F

EPS = 1e-5
ROPE_BASE = 10000.0


def math_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Plain softmax attention, float32 softmax for 16-bit inputs (the reference's ``math`` backend,
    ``models/attention.py:49-54``); differentiable to any order."""
    ct = torch.float32 if q.dtype in (torch.bfloat16, torch.float16) else q.dtype
    s = torch.matmul(q.to(ct), k.to(ct).transpose(-1, -2)) * q.shape[-1] ** -0.5
    return torch.matmul(s.softmax(dim=-1), v.to(ct)).to(q.dtype)


def math_attention64(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """The same in float64, rounded back to the input type: the accuracy yardstick for 16-bit attentions."""
    s = torch.matmul(q.double(), k.double().transpose(-1, -2)) * q.shape[-1] ** -0.5
    return torch.matmul(s.softmax(dim=-1), v.double()).to(q.dtype)


def rms_norm(x: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)).to(x.dtype)


def sphere(z: torch.Tensor, eps: float = EPS) -> torch.Tensor:
    zf = z.float()
    return (zf / zf.square().mean(dim=(1, 2), keepdim=True).sqrt().clamp_min(eps)).to(z.dtype)


def rope_tables(spec: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """[H * W, D] cos / sin of the 2D rotation: channel pair i of the first half turns by row * f_i, of the second
    half by column * f_i, f_i = 1 / base^(2i / (D / 2)) (evaluated in that form, as the reference does, so the tables
    agree to the last bit); sin carries the sign of the rotate-half partner."""
    hh, ww = spec["board"]
    d = spec["hidden"] // spec["heads"]
    half = d // 2
    f = 1.0 / (ROPE_BASE ** (torch.arange(0, half, 2, dtype=torch.float32) / half))
    rows = torch.arange(hh, dtype=torch.float32).repeat_interleave(ww)
    cols = torch.arange(ww, dtype=torch.float32).repeat(hh)
    ang = torch.cat([torch.outer(rows, f).repeat(1, 2), torch.outer(cols, f).repeat(1, 2)], dim=-1)
    sign = torch.ones(d)
    sign[: d // 4] = -1.0
    sign[d // 2 : d // 2 + d // 4] = -1.0
    return ang.cos(), ang.sin() * sign


def quarter_swap(t: torch.Tensor) -> torch.Tensor:
    """(a, b, c, d) -> (b, a, d, c) over the quarters of the last dim."""
    s = t.shape
    return t.reshape(*s[:-1], 2, 2, s[-1] // 4).flip(-2).reshape(s)


def rotate(t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """2D RoPE of ``t`` [B, N, heads, D] in float32 with the [N, D] tables, rounded back to t's dtype."""
    c, s = cos.to(t.device)[None, :, None, :], sin.to(t.device)[None, :, None, :]
    tf = t.float()
    return (tf * c + quarter_swap(tf) * s).to(t.dtype)


def _w(state: dict, name: str, dt: torch.dtype) -> torch.Tensor:
    return state[name].to(dt)


def embed(state: dict, spec: dict, tokens: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return F.embedding(tokens.to(torch.int32), _w(state, "embed_tokens.embedding_weight", dtype)) * math.sqrt(
        spec["hidden"]
    )


def energy(state: dict, spec: dict, v: torch.Tensor, x: torch.Tensor,
           attention: Callable = math_attention) -> torch.Tensor:  # fmt: skip
    """E(v; x) per row, float32 [B]."""
    dt = v.dtype
    b, n, c = v.shape
    heads = spec["heads"]
    d = c // heads
    cos, sin = rope_tables(spec)
    h = v + x
    for i in range(spec["layers"]):
        p = f"level.energy.layers.{i}."
        q, k, vv = F.linear(h, _w(state, p + "self_attn.qkv_proj.weight", dt)).split([c, c, c], dim=-1)
        q, k, vv = q.view(b, n, heads, d), k.view(b, n, heads, d), vv.view(b, n, heads, d)
        q, k = rotate(q, cos, sin), rotate(k, cos, sin)
        q, k, vv = q.transpose(1, 2), k.transpose(1, 2), vv.transpose(1, 2)
        q = q * state[p + "self_attn.log_logit_scale"].exp().to(dt).view(1, -1, 1, 1)
        y = attention(q, k, vv).transpose(1, 2).reshape(b, n, c)
        h = rms_norm(h + F.linear(y, _w(state, p + "self_attn.o_proj.weight", dt)))
        gate, up = F.linear(h, _w(state, p + "mlp.gate_up_proj.weight", dt)).chunk(2, dim=-1)
        h = rms_norm(h + F.linear(F.silu(gate) * up, _w(state, p + "mlp.down_proj.weight", dt)))
    hp = "level.energy.energy_head."
    cell = F.linear(F.silu(F.linear(h, _w(state, hp + "hidden.weight", dt), _w(state, hp + "hidden.bias", dt))),
                    _w(state, hp + "output.weight", dt))  # fmt: skip
    if spec["softplus"]:
        cell = F.softplus(cell.float())
    return cell.float().squeeze(-1).sum(dim=1)


def energy_and_grad(state, spec, v, x, attention=math_attention, create_graph: bool = False):
    """(E, dE/dv)."""
    with torch.enable_grad():
        v = v if v.requires_grad else v.detach().requires_grad_(True)
        e = energy(state, spec, v, x, attention)
        (g,) = torch.autograd.grad(e.sum(), v, create_graph=create_graph)
    return (e if create_graph else e.detach()), g


def microstep(state, spec, z, x, noise=None, alpha: float = 250.0, attention=math_attention):
    """One descent microstep with replayed noise (or none); returns (z', E at v)."""
    v = rms_norm(z)
    if noise is not None:
        v = v + noise.to(v.dtype)
    e, g = energy_and_grad(state, spec, v, x, attention)
    return sphere(v - alpha * g).detach(), e.detach()


class _ReferenceRounding(torch.autograd.Function):
    """Softmax attention with the rounding choices of the reference's GPU kernels
    (``models/fused_attn/triton_kernels.py:576-586``): P rounded to the input type before the P V product, P and dS
    rounded before the backward's products, float32 elsewhere. First order only (enough for dE/dz)."""

    @staticmethod
    def forward(ctx, q, k, v):
        sc = q.shape[-1] ** -0.5
        s = q.float() @ k.float().transpose(-1, -2) * sc
        m = s.amax(-1, keepdim=True)
        p = torch.exp(s - m)
        den = p.sum(-1, keepdim=True)
        o = ((p.to(q.dtype).float() @ v.float()) / den).to(q.dtype)
        ctx.save_for_backward(q, k, v, o, m + torch.log(den))
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        sc = q.shape[-1] ** -0.5
        qf, kf, vf, dof = q.float(), k.float(), v.float(), do.to(q.dtype).float()
        p = torch.exp(qf @ kf.transpose(-1, -2) * sc - lse)
        dv = p.to(q.dtype).float().transpose(-1, -2) @ dof
        dp = dof @ vf.transpose(-1, -2)
        ds = (p * (dp - (dof * o.float()).sum(-1, keepdim=True))).to(q.dtype).float()
        return (ds @ kf * sc).to(q.dtype), (ds.transpose(-1, -2) @ qf * sc).to(q.dtype), dv.to(q.dtype)


def reference_rounding_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    return _ReferenceRounding.apply(q, k, v)
