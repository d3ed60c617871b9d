"""Seeded weights and inputs of the energy-network golden cases, shared by ``make_golden.py`` (which runs the
reference's own ``InnerNetwork`` on them in the build container) and the tests (which regenerate them on any machine,
CPU or GPU box, so only the reference's outputs are stored).

Weights are keyed by the reference's state-dict names (``models/energy.py`` ``InnerNetwork``: ``embed_tokens``,
``lm_head``, ``level.energy.layers.<i>.{self_attn,mlp}.*``, ``level.energy.energy_head.*``) and drawn from one
``torch.Generator`` in a fixed order, scaled like the reference's initialisation (fan-in 1/sqrt scaling), with a
non-zero per-head temperature and bias so every parameter of the path is exercised.
"""

from __future__ import annotations

import math

import torch

CASES: dict[str, dict] = {
    # the benchmark architecture on a 9 x 9 board: 4 layers, hidden 512, 8 heads x 64, SwiGLU 4x (width 1536)
    "bench81": dict(board=(9, 9), vocab=10, hidden=512, heads=8, layers=4, expansion=4.0, softplus=False, rows=2,
                    seed=101),  # fmt: skip
    # a one-layer 4 x 4 case with the softplus cell head, small enough for the second-order probe
    "small16": dict(board=(4, 4), vocab=6, hidden=256, heads=4, layers=1, expansion=4.0, softplus=True, rows=2,
                    seed=202),  # fmt: skip
}


def mlp_width(hidden: int, expansion: float) -> int:
    """SwiGLU width: 2/3 of ``expansion * hidden``, rounded up to a multiple of 256 (``models/layers.py:74-80``)."""
    width = round(expansion * hidden * 2 / 3)
    return (width + 255) // 256 * 256


def param_shapes(case: dict) -> dict[str, tuple[int, ...]]:
    """Reference state-dict name -> shape, in the fixed draw order."""
    c, v, heads = case["hidden"], case["vocab"], case["heads"]
    w = mlp_width(c, case["expansion"])
    out: dict[str, tuple[int, ...]] = {"embed_tokens.embedding_weight": (v, c), "lm_head.weight": (v, c)}
    for i in range(case["layers"]):
        p = f"level.energy.layers.{i}."
        out[p + "self_attn.log_logit_scale"] = (heads,)
        out[p + "self_attn.qkv_proj.weight"] = (3 * c, c)
        out[p + "self_attn.o_proj.weight"] = (c, c)
        out[p + "mlp.gate_up_proj.weight"] = (2 * w, c)
        out[p + "mlp.down_proj.weight"] = (c, w)
    out["level.energy.energy_head.hidden.weight"] = (c, c)
    out["level.energy.energy_head.hidden.bias"] = (c,)
    out["level.energy.energy_head.output.weight"] = (1, c)
    return out


def make_params(case: dict) -> dict[str, torch.Tensor]:
    """float32 weights keyed by the reference's state-dict names."""
    g = torch.Generator().manual_seed(case["seed"])
    out = {}
    for name, shape in param_shapes(case).items():
        x = torch.randn(shape, generator=g, dtype=torch.float32)
        if name.endswith("embedding_weight"):
            x = x / math.sqrt(case["hidden"])
        elif name.endswith("log_logit_scale"):
            x = x * 0.2
        elif name.endswith(".bias"):
            x = x * 0.1
        else:
            x = x / math.sqrt(shape[1])
        out[name] = x.contiguous()
    return out


def make_inputs(case: dict) -> dict[str, torch.Tensor]:
    """Tokens [rows, L] (int64), latent z, noise and a probe direction u ([rows, L, hidden], float32)."""
    g = torch.Generator().manual_seed(case["seed"] + 1)
    rows, (h, w), c = case["rows"], case["board"], case["hidden"]
    n = h * w
    tokens = torch.randint(0, case["vocab"], (rows, n), generator=g)
    z = torch.randn(rows, n, c, generator=g).clamp_(-2.0, 2.0)
    noise = torch.randn(rows, n, c, generator=g) * 0.05
    u = torch.randn(rows, n, c, generator=g)
    return {"tokens": tokens, "z": z, "noise": noise, "u": u}


def checksum(tensors: dict[str, torch.Tensor]) -> float:
    """Order-independent float64 checksum that detects a drifted generator."""
    return float(sum(t.double().abs().sum().item() + 0.5 * t.double().sum().item() for t in tensors.values()))


STEP_SIZE = 250.0  # the microstep fixture's alpha (the reference's eval step size, config/arch/ebr.yaml)
SAMPLE = 8192  # sampled entries stored per large output
