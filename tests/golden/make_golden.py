"""Generate the golden vectors of the attention path from the REAL reference implementation.

Run in the build container, where the reference source tree is mounted::

    EBR_REFERENCE=/path/to/ebr python tests/golden/make_golden.py

It imports ``models.fused_attn`` from the reference tree (CPU: the dense ``reference.py`` path, the same math the
reference's Triton kernels are checked against), runs the three ops and the double-differentiable
``fused_attention`` on seeded inputs, and writes ``tests/golden/attn_golden.npz``. The GPU box never runs this script;
the tests only read the committed ``.npz``.

Cases
-----
* ``cfg1``: the benchmark's fp32 parity case, B=4, L=81, H=8, D=64, ``torch.manual_seed(0)``, drawn in the order q, k, v
  ~ N(0,1)/8, dO ~ N(0,1), R ~ N(0,1). O, then (dQ, dK, dV) with ``create_graph=True``, then the gradient of
  sum(dQ * R) w.r.t. (Q, K, V). Too large to store whole: the inputs are re-drawn from the seed by the tests (their
  checksums are stored), the outputs are stored as 4096 fixed random entries each plus per-(b, h) sums.
* small cases stored whole: N=1, 17, 33 and 100 with D in {16, 64, 128}, fp32 / fp64 / bf16 (bf16 stored as its
  uint16 bit pattern), including the op-level ``attn_bwd_bwd`` with all three cotangents and with ``gk = gv = None``.

It also writes ``tests/golden/layers_golden.npz``:

* ``rope/<case>``: the reference's dense 2D-RoPE split and merge (``models/fused_attn/rope_split.py`` ``ref_split`` /
  ``ref_merge``) on its own ``RotaryTable2D`` tables (``models/layers.py:149-172``), bf16 / fp16 / fp32, with and
  without the per-head temperature.
* ``energy/<case>/<dtype>``: the reference's ``InnerNetwork`` (``models/energy.py``) with the seeded weights of
  ``energy_case.py`` loaded into it, eager math attention, broadcast RoPE: the energies E(v, x) at v = rms_norm(z),
  dE/dv, one ``EnergyDescent`` microstep with replayed noise (eval step size), and for the small case the second-order
  probe of the reference's compiled-gradient check (``models/energy.py:386-434``): d<dE/dv, u>/dv and
  d<dE/dv, u>/dtheta. Large outputs are stored as sampled entries plus per-cell norms.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
SUBSAMPLE = 4096
if str(HERE) not in sys.path:
    sys.path.insert(0, str(HERE))

from energy_case import CASES, SAMPLE, STEP_SIZE, checksum, make_inputs, make_params  # noqa: E402


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
    """The fp32 parity case's inputs, drawn in the stated order (also used by the tests)."""
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

    layers: dict[str, np.ndarray] = {}
    rope_fixtures(layers)
    energy_fixtures(layers)
    np.savez_compressed(HERE / "layers_golden.npz", **layers)
    size = (HERE / "layers_golden.npz").stat().st_size
    print(f"wrote {HERE / 'layers_golden.npz'} ({size} bytes, {len(layers)} arrays)")


ROPE_CASES = [
    # name, batch, board (height, width), heads, head_dim, dtype, with temperature
    ("b2_3x4_h2_d64_bf16_q", 2, (3, 4), 2, 64, torch.bfloat16, True),
    ("b1_9x9_h2_d64_bf16", 1, (9, 9), 2, 64, torch.bfloat16, False),
    ("b1_5x5_h2_d128_fp16_q", 1, (5, 5), 2, 128, torch.float16, True),
    ("b2_3x3_h2_d32_f32_q", 2, (3, 3), 2, 32, torch.float32, True),
]


def rope_fixtures(out: dict[str, np.ndarray]) -> None:
    from models.fused_attn.rope_split import ref_merge, ref_split
    from models.layers import RotaryTable2D

    for name, b, (hh, ww), heads, d, dtype, with_q in ROPE_CASES:
        gen = torch.Generator().manual_seed(sum(map(ord, name)))
        n = hh * ww
        table = RotaryTable2D(d, hh, ww)
        cos, sin = table.cos_table, table.sin_table
        qkv = torch.randn(b, n, 3 * heads * d, generator=gen).to(dtype)
        qscale = (torch.rand(heads, generator=gen) + 0.5).to(dtype) if with_q else None
        q, k, v = ref_split(qkv, cos, sin, heads, qscale)
        dq, dk, dv = (torch.randn(b, heads, n, d, generator=gen).to(dtype) for _ in range(3))
        g = ref_merge(dq, dk, dv, cos, sin, qscale)
        arrays = dict(qkv=qkv, cos=cos, sin=sin, q=q, k=k, v=v, dq=dq, dk=dk, dv=dv, g=g)
        if qscale is not None:
            arrays["qscale"] = qscale
        for t_name, t in arrays.items():
            out[f"rope/{name}/{t_name}"] = _np16(t)
        out[f"rope/{name}/meta"] = np.array([str(dtype).replace("torch.", ""), str(heads)])


def _np16(t: torch.Tensor) -> np.ndarray:
    """bf16 as its uint16 bits, fp16 as float16, the rest as is."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def reference_config(ref_energy, case: dict, dtype: str):
    """The reference's EnergyConfig for a golden case: eager math attention, broadcast RoPE, no compilation."""
    hh, ww = case["board"]
    return ref_energy.EnergyConfig(
        seq_len=hh * ww, vocab_size=case["vocab"], num_layers=case["layers"], hidden_size=case["hidden"],
        expansion=case["expansion"], num_heads=case["heads"], board_height=hh, board_width=ww, forward_dtype=dtype,
        energy_cell_activation="softplus" if case["softplus"] else "linear", attn_backend="math",
        attn_nograd_backend="math", cycles=16, grad_cycles=7, randomize_min_cycles=16, reset_cycles_low=7,
        reset_cycles_high=16, halt_max_steps=16, halt_exploration_prob=0.0, step_size=STEP_SIZE, step_size_low=200.0,
        step_size_high=250.0, init_std=1.0, noise_scale=0.05, noise_cosine=False, noise_settle_hot=0.4,
        microstep_ce=0.5, microstep_ce_ramp=1.0, convergence_threshold=0.75, convergence_temperature=0.05,
        convergence_window=2, explore_k=1, energy_compile=False,
    )  # fmt: skip


def energy_fixtures(out: dict[str, np.ndarray]) -> None:
    import models.energy as ref_energy

    for cname, case in CASES.items():
        params = make_params(case)
        inputs = make_inputs(case)
        out[f"energy/{cname}/param_checksum"] = np.array([checksum(params)])
        out[f"energy/{cname}/input_checksum"] = np.array([checksum({k: v.double() for k, v in inputs.items()})])
        for dtype_name in ("float32", "bfloat16"):
            dtype = getattr(torch, dtype_name)
            torch.manual_seed(0)
            net = ref_energy.InnerNetwork(reference_config(ref_energy, case, dtype_name))
            missing, unexpected = net.load_state_dict(params, strict=False)
            assert not unexpected and all("rotary" in m for m in missing), (missing, unexpected)
            net.eval()
            key = f"energy/{cname}/{dtype_name}"
            cos_sin = net.cos_sin()
            with torch.no_grad():
                x = net.input_embeddings(inputs["tokens"])
            z = inputs["z"].to(dtype)
            level = net.level
            v = level.normalize_descent_state(z).detach().requires_grad_(True)
            e = level.energy(v, x, cos_sin)
            (g,) = torch.autograd.grad(e.sum(), v)
            z_next = level(z, x, cos_sin, noise=inputs["noise"])
            idx = np.random.default_rng(7).choice(g.numel(), size=min(SAMPLE, g.numel()), replace=False)
            out[f"{key}/index"] = idx.astype(np.int32)
            out[f"{key}/energy"] = e.detach().double().numpy()
            out[f"{key}/grad/sample"] = g.detach().float().reshape(-1)[idx].numpy()
            out[f"{key}/grad/cell_norm"] = g.detach().double().norm(dim=-1).numpy()
            out[f"{key}/z_next/sample"] = z_next.detach().float().reshape(-1)[idx].numpy()
            out[f"{key}/z_next/cell_norm"] = z_next.detach().double().norm(dim=-1).numpy()
            if cname == "small16":
                second_order_fixture(out, key, net, v.detach(), x, inputs["u"].to(dtype))


def second_order_fixture(out, key, net, v0, x, u) -> None:
    """d<dE/dv, u>/dv and d<dE/dv, u>/dtheta through the reference's graded energy gradient (create_graph=True)."""
    level = net.level
    v = v0.clone().requires_grad_(True)
    params = [p for _, p in level.energy.named_parameters()]
    names = [n for n, _ in level.energy.named_parameters()]
    g = level._energy_gradient(v, x, net.cos_sin(), create_graph=True)
    hz, *ht = torch.autograd.grad((g * u).sum(), [v] + params)
    out[f"{key}/hz"] = hz.detach().float().numpy()
    rng = np.random.default_rng(11)
    for name, t in zip(names, ht):
        flat = t.detach().double().reshape(-1)
        sel = rng.choice(flat.numel(), size=min(512, flat.numel()), replace=False)
        out[f"{key}/htheta/{name}/index"] = sel.astype(np.int32)
        out[f"{key}/htheta/{name}/sample"] = flat[sel].float().numpy()
        out[f"{key}/htheta/{name}/norm"] = np.array([float(flat.norm())])


if __name__ == "__main__":
    main()
