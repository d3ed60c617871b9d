"""CPU restatement of the reference's dense 2D-RoPE split and merge (``models/fused_attn/rope_split.py:31-67``).

TEST INFRASTRUCTURE ONLY: the GPU layer tests use it as the yardstick of the RoPE kernels on inputs too large to
store; ``tests/test_oracle.py`` pins it bit for bit against the reference's own outputs
(``tests/golden/layers_golden.npz``).

* ``split(qkv, cos, sin, heads, qscale)``: ``qkv`` [B, N, 3 H D] -> q, k, v [B, H, N, D]; q and k rotated in float32
  (float64 for float64 input) with ``t * cos + quarter_swap(t) * sin`` and rounded to the input type, then q times
  the per-head temperature (a second rounding), as the reference does.
* ``merge(dq, dk, dv, cos, sin, qscale)``: the adjoint, ``[B, N, 3 H D]``.
"""

from __future__ import annotations

import torch


def _compute_type(t: torch.Tensor) -> torch.dtype:
    return torch.float64 if t.dtype == torch.float64 else torch.float32


def quarter_swap(x: torch.Tensor) -> torch.Tensor:
    """(a, b, c, d) -> (b, a, d, c) over the quarters of the last dim."""
    s = x.shape
    return x.reshape(*s[:-1], 2, 2, s[-1] // 4).flip(-2).reshape(s)


def split(qkv, cos, sin, heads: int, qscale=None):
    b, n, c3 = qkv.shape
    d = c3 // (3 * heads)
    ct = _compute_type(qkv)
    parts = qkv.view(b, n, 3, heads, d)
    c, s = cos.to(qkv.device, ct)[None, :, None, :], sin.to(qkv.device, ct)[None, :, None, :]
    turn = lambda t: (t.to(ct) * c + quarter_swap(t.to(ct)) * s).to(qkv.dtype)
    q, k, v = turn(parts[:, :, 0]), turn(parts[:, :, 1]), parts[:, :, 2]
    if qscale is not None and qscale.numel():
        q = (q.to(ct) * qscale.to(qkv.device, ct).view(1, 1, -1, 1)).to(qkv.dtype)
    return tuple(t.transpose(1, 2).contiguous() for t in (q, k, v))


def merge(dq, dk, dv, cos, sin, qscale=None):
    b, h, n, d = dq.shape
    ct = _compute_type(dq)
    c, s = cos.to(dq.device, ct)[None, None], sin.to(dq.device, ct)[None, None]
    adj = lambda g: (g.to(ct) * c + quarter_swap(g.to(ct) * s)).to(dq.dtype)
    if qscale is not None and qscale.numel():
        dq = (dq.to(ct) * qscale.to(dq.device, ct).view(1, -1, 1, 1)).to(dq.dtype)
    out = torch.stack([adj(dq), adj(dk), dv.to(dq.dtype)], dim=2)  # [B, H, 3, N, D]
    return out.permute(0, 3, 2, 1, 4).reshape(b, n, 3 * h * d)
