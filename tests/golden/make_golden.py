"""Generate the golden vectors of the attention path from the REAL reference implementation.

Run in the build container, where the reference source tree is mounted::

    EBR_REFERENCE=/path/to/ebr python tests/golden/make_golden.py

It imports ``models.fused_attn`` from the reference tree (CPU: the dense ``reference.py`` path, the same math the
reference's Triton kernels are checked against), runs the three ops and the double-differentiable
``fused_attention`` on seeded inputs, and writes ``tests/golden/attn_golden.npz``. The GPU box never runs this script;
the tests only read the committed ``.npz``.

Cases
-----
* ``cfg1``: BASELINE config 1. fp32, B=4, L=81, H=8, D=64, ``torch.manual_seed(0)``, drawn in the order q, k, v
  ~ N(0,1)/8, dO ~ N(0,1), R ~ N(0,1). O, then (dQ, dK, dV) with ``create_graph=True``, then the gradient of
  sum(dQ * R) w.r.t. (Q, K, V). Too large to store whole: the inputs are re-drawn from the seed by the tests (their
  checksums are stored), the outputs are stored as 4096 fixed random entries each plus per-(b, h) sums.
* small cases stored whole: N=1, 17, 33 and 100 with D in {16, 64, 128}, fp32 / fp64 / bf16 (bf16 stored as its
  uint16 bit pattern), including the op-level ``attn_bwd_bwd`` with all three cotangents and with ``gk = gv = None``.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SUBSAMPLE = 4096


def _import_reference():
    root = os.environ.get("EBR_REFERENCE")
    if not root:
        raise SystemExit("set EBR_REFERENCE to the reference source tree")
    os.environ["EBR_FUSED_ATTN_IMPL"] = "reference"
    sys.path.insert(0, root)
    from models.fused_attn import fused_attention, reference  # noqa: E402

    return fused_attention, reference


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def cfg1_inputs() -> dict[str, torch.Tensor]:
    """BASELINE config 1 inputs, drawn exactly as the config states (also used by the tests)."""
    torch.manual_seed(0)
    shape = (4, 8, 81, 64)
    q = torch.randn(shape) / 8
    k = torch.randn(shape) / 8
    v = torch.randn(shape) / 8
    do = torch.randn(shape)
    r = torch.randn(shape)
    return {"q": q, "k": k, "v": v, "do": do, "r": r}


def cfg1_subsample_index(numel: int) -> np.ndarray:
    return np.random.default_rng(20251201).choice(numel, size=SUBSAMPLE, replace=False)


def main() -> None:
    fused_attention, reference = _import_reference()
    out: dict[str, np.ndarray] = {}

    # ---- cfg1 ------------------------------------------------------------------------------------------------
    x = cfg1_inputs()
    q, k, v = (x[n].clone().requires_grad_(True) for n in ("q", "k", "v"))
    o = fused_attention(q, k, v)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), grad_outputs=x["do"], create_graph=True)
    hq, hk, hv = torch.autograd.grad((dq * x["r"]).sum(), (q, k, v))
    _, lse = reference.attn_fwd(x["q"], x["k"], x["v"], 0.125)
    idx = cfg1_subsample_index(o.numel())
    out["cfg1/index"] = idx
    for name, t in x.items():
        out[f"cfg1/in_sum/{name}"] = np.array([t.double().sum().item(), t.double().abs().sum().item()])
    for name, t in {"o": o, "dq": dq, "dk": dk, "dv": dv, "hq": hq, "hk": hk, "hv": hv}.items():
        flat = t.detach().reshape(-1)
        out[f"cfg1/{name}/sample"] = flat[idx].numpy()
        out[f"cfg1/{name}/bh_sum"] = t.detach().double().sum(dim=(2, 3)).numpy()
    out["cfg1/lse/sample"] = lse.reshape(-1)[np.unique(idx // 64)].numpy()
    out["cfg1/lse/rows"] = np.unique(idx // 64)

    # ---- small whole cases ---------------------------------------------------------------------------------------
    cases = [
        ("n1_d64_f32", (1, 1, 1, 64), torch.float32),
        ("n17_d16_f64", (1, 2, 17, 16), torch.float64),
        ("n33_d64_f32", (1, 2, 33, 64), torch.float32),
        ("n81_d64_bf16", (1, 1, 81, 64), torch.bfloat16),
        ("n100_d128_bf16", (1, 1, 100, 128), torch.bfloat16),
        ("n100_d64_bf16", (1, 1, 100, 64), torch.bfloat16),
    ]
    for name, shape, dtype in cases:
        gen = torch.Generator().manual_seed(sum(map(ord, name)))
        draw = lambda s=1.0: (torch.randn(shape, generator=gen, dtype=torch.float64) * s).to(dtype)
        q, k, v = draw(0.5), draw(0.5), draw(0.5)
        do, gq, gk, gv = draw(), draw(), draw(), draw()
        scale = shape[-1] ** -0.5
        o, lse = reference.attn_fwd(q, k, v, scale)
        dq, dk, dv = reference.attn_bwd(q, k, v, o, lse, do, scale)
        hq, hk, hv, hdo = reference.attn_bwd_bwd(q, k, v, o, lse, do, dq, gq, gk, gv, scale)
        zero = torch.zeros_like(q)
        hq0, hk0, hv0, hdo0 = reference.attn_bwd_bwd(q, k, v, o, lse, do, dq, gq, zero, zero, scale)
        tensors = dict(
            q=q, k=k, v=v, do=do, gq=gq, gk=gk, gv=gv, o=o, lse=lse, dq=dq, dk=dk, dv=dv,
            hq=hq, hk=hk, hv=hv, hdo=hdo, hq0=hq0, hk0=hk0, hv0=hv0, hdo0=hdo0,
        )  # fmt: skip
        for tname, t in tensors.items():
            out[f"{name}/{tname}"] = _np(t)
        out[f"{name}/meta"] = np.array([str(dtype).replace("torch.", ""), repr(scale)])

    np.savez_compressed(HERE / "attn_golden.npz", **out)
    print(f"wrote {HERE / 'attn_golden.npz'} ({(HERE / 'attn_golden.npz').stat().st_size} bytes, {len(out)} arrays)")


if __name__ == "__main__":
    main()
