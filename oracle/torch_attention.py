"""The oracle as a differentiable torch attention callable (CPU), for the benchmark's CPU baseline and CPU tests.

TEST INFRASTRUCTURE ONLY (see ``oracle/attention.py``). ``oracle_attention(q, k, v)`` has the signature of the
product's ``fused_attention`` call in the energy network and chains the oracle's forward, backward and double
backward exactly as the reference's autograd Functions chain its ops (``models/fused_attn/ops.py:131-175``): it is
the reference's CPU path (dense math, float32) restated on numpy.
"""

from __future__ import annotations

import numpy as np
import torch

from oracle import attention as oracle


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.contiguous().numpy()


def _t(a: np.ndarray, like: torch.Tensor) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(like.dtype)


class _OracleBwd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, o, lse, do, scale):
        ctx.save_for_backward(q, k, v, o, lse, do)
        ctx.scale = scale
        dq, dk, dv = oracle.attn_bwd(_np(q), _np(k), _np(v), _np(o), _np(lse), _np(do), scale)
        return _t(dq, q), _t(dk, q), _t(dv, q)

    @staticmethod
    def backward(ctx, gq, gk, gv):
        q, k, v, o, lse, do = ctx.saved_tensors
        g = lambda x: None if x is None else _np(x)
        hs = oracle.attn_bwd_bwd(_np(q), _np(k), _np(v), _np(o), _np(lse), _np(do), None, g(gq), g(gk), g(gv),
                                 ctx.scale)  # fmt: skip
        hq, hk, hv, hdo = (_t(h, q) for h in hs)
        return hq, hk, hv, None, None, hdo, None


class _OracleAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale):
        o, lse = oracle.attn_fwd(_np(q), _np(k), _np(v), scale)
        o_t, lse_t = _t(o, q), torch.from_numpy(lse)
        ctx.save_for_backward(q, k, v, o_t, lse_t)
        ctx.scale = scale
        ctx.mark_non_differentiable(lse_t)
        return o_t, lse_t

    @staticmethod
    def backward(ctx, do, dlse):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = _OracleBwd.apply(q, k, v, o, lse, do.to(q.dtype), ctx.scale)
        return dq, dk, dv, None


def oracle_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    o, _ = _OracleAttn.apply(q, k, v, q.shape[-1] ** -0.5)
    return o
