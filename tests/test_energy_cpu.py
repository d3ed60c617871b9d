"""The CPU restatement of the reference's energy network (``oracle/energy.py``) against the reference's own outputs
(``tests/golden/layers_golden.npz``, written by ``tests/golden/make_golden.py`` from ``models/energy.py``), and the
product network's translation to and from the reference's state-dict names.

The restatement is the yardstick of the GPU network tests and the CPU baseline, so it is pinned here first: energies,
dE/dv, one descent microstep and the second-order probe of the reference's compiled-gradient check, in float32 and
bf16, on the benchmark architecture and on a small softplus-head case."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import energy as oe
from tests.golden.energy_case import CASES, STEP_SIZE, checksum, make_inputs, make_params

DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16}


def _inputs(golden, cname):
    case = CASES[cname]
    params, inputs = make_params(case), make_inputs(case)
    assert np.isclose(checksum(params), golden[f"energy/{cname}/param_checksum"][0], rtol=1e-12)
    assert np.isclose(checksum({k: v.double() for k, v in inputs.items()}),
                      golden[f"energy/{cname}/input_checksum"][0], rtol=1e-12)  # fmt: skip
    return case, params, inputs


def _maxrel(a: np.ndarray, r: np.ndarray) -> float:
    return float(np.abs(a - r).max() / np.abs(r).max())


@pytest.mark.parametrize("dtype_name", list(DTYPES))
@pytest.mark.parametrize("cname", list(CASES))
def test_oracle_energy_matches_reference(layers_golden, cname, dtype_name):
    g_ = layers_golden
    case, params, inputs = _inputs(g_, cname)
    dt = DTYPES[dtype_name]
    key = f"energy/{cname}/{dtype_name}"
    x = oe.embed(params, case, inputs["tokens"], dt)
    z = inputs["z"].to(dt)
    v = oe.rms_norm(z)
    e, g = oe.energy_and_grad(params, case, v, x)
    idx = g_[f"{key}/index"]
    # The restatement runs the reference's torch ops in the reference's order: equal to the last bit in this
    # container (the tolerance only absorbs a different CPU's matmul kernels).
    tol = 1e-6
    assert _maxrel(e.double().numpy(), g_[f"{key}/energy"]) <= tol
    assert _maxrel(g.float().reshape(-1).numpy()[idx], g_[f"{key}/grad/sample"]) <= tol
    assert _maxrel(g.double().norm(dim=-1).numpy(), g_[f"{key}/grad/cell_norm"]) <= tol
    z_next, _ = oe.microstep(params, case, z, x, noise=inputs["noise"], alpha=STEP_SIZE)
    assert _maxrel(z_next.float().reshape(-1).numpy()[idx], g_[f"{key}/z_next/sample"]) <= tol
    assert _maxrel(z_next.double().norm(dim=-1).numpy(), g_[f"{key}/z_next/cell_norm"]) <= tol


@pytest.mark.parametrize("dtype_name", list(DTYPES))
def test_oracle_second_order_matches_reference(layers_golden, dtype_name):
    """d<dE/dv, u>/dv and d<dE/dv, u>/dtheta (the probe of models/energy.py:386-434) on the small case."""
    g_ = layers_golden
    case, params, inputs = _inputs(g_, "small16")
    dt = DTYPES[dtype_name]
    key = f"energy/small16/{dtype_name}"
    state = {n: p.clone().requires_grad_(True) for n, p in params.items()}
    x = oe.embed(state, case, inputs["tokens"], dt).detach()
    v = oe.rms_norm(inputs["z"].to(dt)).detach().requires_grad_(True)
    _, g = oe.energy_and_grad(state, case, v, x, create_graph=True)
    names = [n for n in state if n.startswith("level.energy.")]
    hz, *ht = torch.autograd.grad((g * inputs["u"].to(dt)).sum(), [v] + [state[n] for n in names])
    tol = 1e-6
    assert _maxrel(hz.float().numpy(), g_[f"{key}/hz"]) <= tol
    for n, t in zip(names, ht):
        rel = n[len("level.energy."):]  # the fixture names parameters relative to ScalarEnergy
        idx = g_[f"{key}/htheta/{rel}/index"]
        assert _maxrel(t.float().reshape(-1).numpy()[idx], g_[f"{key}/htheta/{rel}/sample"]) <= tol, n


def test_oracle_rope_matches_reference(layers_golden):
    """The restatement's 2D-RoPE tables and rotation equal the reference's ref_split (rope_split.py:31-47) bit for bit;
    the GPU RoPE kernels are then checked against the same fixtures."""
    g_ = layers_golden
    for name in sorted({k.split("/")[1] for k in g_.files if k.startswith("rope/")}):
        meta = g_[f"rope/{name}/meta"]
        heads = int(meta[1])
        cos, sin = g_[f"rope/{name}/cos"], g_[f"rope/{name}/sin"]
        n, d = cos.shape
        board = {12: (3, 4), 81: (9, 9), 25: (5, 5), 9: (3, 3)}[n]
        ocos, osin = oe.rope_tables({"board": board, "hidden": heads * d, "heads": heads})
        assert np.array_equal(ocos.numpy(), cos) and np.array_equal(osin.numpy(), sin), name


def test_product_network_reference_names_round_trip():
    """LatentEnergyNet takes the reference's state dict and gives it back unchanged (weights only; no compute)."""
    from ebr_b200.energy import LatentEnergyNet, NetShape

    case = CASES["small16"]
    params = make_params(case)
    net = LatentEnergyNet(NetShape(board=case["board"], vocab=case["vocab"], hidden=case["hidden"],
                                   heads=case["heads"], layers=case["layers"], cell_softplus=case["softplus"]))  # fmt: skip
    net.load_reference_state(params)
    back = net.reference_state()
    assert set(back) == set(params)
    assert all(torch.equal(back[k], params[k]) for k in params)
    with pytest.raises(KeyError):
        net.load_reference_state({k: v for k, v in params.items() if "down_proj" not in k})


def test_product_rope_tables_match_reference(layers_golden):
    """The product network's RoPE tables are the reference's RotaryTable2D tables bit for bit."""
    from ebr_b200.energy import NetShape, rope_tables

    cos, sin = rope_tables(NetShape(board=(9, 9), hidden=128, heads=2))
    assert np.array_equal(cos.numpy(), layers_golden["rope/b1_9x9_h2_d64_bf16/cos"])
    assert np.array_equal(sin.numpy(), layers_golden["rope/b1_9x9_h2_d64_bf16/sin"])
