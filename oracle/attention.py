"""CPU oracle for the fused second-order attention path.

TEST INFRASTRUCTURE ONLY. This module is the checker the parity tests, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` compare against or time. Nothing in the product package
(``ebr_b200``) imports it, and the product path never falls back to it.

It is a numpy restatement of the reference's dense attention math, ``models/fused_attn/reference.py`` in
wwillchen/ebr, function by function:

* ``attn_fwd``        follows ``reference.py:32-36`` (with ``_probs`` at ``:23-29``);
* ``_first_backward`` follows ``reference.py:39-47`` (D = rowsum(dO * O) from the *stored* O, ``:44-45``);
* ``attn_bwd``        follows ``reference.py:50-58``;
* ``attn_bwd_bwd``    follows ``reference.py:61-91`` (the closed-form second-order formula);
* ``default_scale`` / ``lse_dtype_for`` follow ``reference.py:18-20`` and ``:13-15``.

Compute dtype: float32 for every input dtype except float64, which stays float64 (``reference.py:9-10``). Inputs are
numpy arrays of shape ``[B, H, N, D]`` (bfloat16 tensors are passed in already widened to float32, which is exact).
The outputs are returned in the compute dtype; rounding them to the caller's storage dtype is the caller's business.

Parity pinning: ``tests/golden/make_golden.py`` runs the real reference (imported from its source tree in the build
container) on seeded inputs and commits its outputs under ``tests/golden/``; ``tests/test_oracle.py`` checks this
module against them.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "attn_bwd",
    "attn_bwd_bwd",
    "attn_fwd",
    "compute_dtype",
    "default_scale",
    "lse_dtype_for",
    "max_rel",
]


def compute_dtype(x: np.ndarray) -> type:
    """float64 stays float64, everything else computes in float32 (``reference.py:9-10``)."""
    return np.float64 if x.dtype == np.float64 else np.float32


def lse_dtype_for(x: np.ndarray) -> type:
    """The row logsumexp is float32, float64 for float64 inputs (``reference.py:13-15``)."""
    return compute_dtype(x)


def default_scale(head_dim: int, scale: float | None = None) -> float:
    """``D ** -0.5`` unless given (``reference.py:18-20``)."""
    return float(head_dim**-0.5) if scale is None else float(scale)


def _t(x: np.ndarray) -> np.ndarray:
    return np.swapaxes(x, -1, -2)


def _scalar(scale: float, ct: type):
    # torch multiplies a float32 tensor by a python float in float32: the scale is rounded to the compute dtype once.
    return ct(scale)


def _logsumexp(s: np.ndarray) -> np.ndarray:
    if s.shape[-1] == 0:
        return np.full(s.shape[:-1], -np.inf, dtype=s.dtype)
    m = s.max(-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0).astype(s.dtype)
    return (np.log(np.exp(s - m).sum(-1, keepdims=True)) + m)[..., 0]


def _probs(q, k, scale, lse=None):
    """P = exp(scale * Q K^T - lse) and the natural-log row logsumexp (``reference.py:23-29``)."""
    ct = compute_dtype(q)
    s = np.matmul(q.astype(ct), _t(k.astype(ct))) * _scalar(scale, ct)
    if lse is None:
        lse = _logsumexp(s)
    p = np.exp(s - lse.astype(ct)[..., None])
    return p, lse


def attn_fwd(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> tuple[np.ndarray, np.ndarray]:
    """O = softmax(scale Q K^T) V and the row logsumexp (``reference.py:32-36``)."""
    ct = compute_dtype(q)
    p, lse = _probs(q, k, scale)
    o = np.matmul(p, v.astype(ct))
    return o.astype(ct), lse.astype(lse_dtype_for(q))


def _first_backward(q, k, v, o, lse, do, scale):
    """P, dP = dO V^T, D = rowsum(dO * O) with the stored O, dS = P (dP - D) (``reference.py:39-47``)."""
    ct = compute_dtype(q)
    p, _ = _probs(q, k, scale, lse)
    dof, vf = do.astype(ct), v.astype(ct)
    dp = np.matmul(dof, _t(vf))
    d = (dof * o.astype(ct)).sum(-1, keepdims=True)
    ds = p * (dp - d)
    return p, dp, d, ds


def attn_bwd(q, k, v, o, lse, do, scale: float) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(dQ, dK, dV) of <dO, O> (``reference.py:50-58``)."""
    ct = compute_dtype(q)
    sc = _scalar(scale, ct)
    p, _, _, ds = _first_backward(q, k, v, o, lse, do, scale)
    dq = np.matmul(ds, k.astype(ct)) * sc
    dk = np.matmul(_t(ds), q.astype(ct)) * sc
    dv = np.matmul(_t(p), do.astype(ct))
    return dq.astype(ct), dk.astype(ct), dv.astype(ct)


def attn_bwd_bwd(q, k, v, o, lse, do, dq, gq, gk, gv, scale: float):
    """(hQ, hK, hV, hdO): total derivative of <gQ,dQ> + <gK,dK> + <gV,dV> w.r.t. (Q, K, V, dO).

    Follows ``reference.py:61-91``. ``dq`` is accepted for the op contract and not read (``reference.py:74``); a
    ``None`` cotangent is zeros.
    """
    del dq
    ct = compute_dtype(q)
    sc = _scalar(scale, ct)
    z = lambda g: np.zeros(q.shape, ct) if g is None else g.astype(ct)
    qf, kf, vf, dof = q.astype(ct), k.astype(ct), v.astype(ct), do.astype(ct)
    gqf, gkf, gvf = z(gq), z(gk), z(gv)
    p, dp, d, ds = _first_backward(q, k, v, o, lse, do, scale)

    g = (np.matmul(gqf, _t(kf)) + np.matmul(qf, _t(gkf))) * sc
    r = np.matmul(dof, _t(gvf))
    e = (p * g).sum(-1, keepdims=True)
    a = p * (g - e)
    gp = (dp - d) * g - e * dp + r
    gs = p * (gp - (p * gp).sum(-1, keepdims=True))

    hq = (np.matmul(gs, kf) + np.matmul(ds, gkf)) * sc
    hk = (np.matmul(_t(gs), qf) + np.matmul(_t(ds), gqf)) * sc
    hv = np.matmul(_t(a), dof)
    hdo = np.matmul(a, vf) + np.matmul(p, gvf)
    return hq.astype(ct), hk.astype(ct), hv.astype(ct), hdo.astype(ct)


def max_rel(a: np.ndarray, ref: np.ndarray) -> float:
    """The reference's error metric, ``max|a - ref| / max|ref|`` (``models/attention.py:156-161``)."""
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if ref.size == 0:
        return 0.0
    return float(np.abs(a - ref).max() / max(np.abs(ref).max(), 1e-12))
