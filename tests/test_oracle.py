"""The CPU oracle against the reference's own outputs (golden vectors made by ``tests/golden/make_golden.py``)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oracle
from tests.conftest import GOLDEN_CASES, bf16_round, golden_case

TOL = {"float64": 1e-12, "float32": 2e-6}


def _err(got: np.ndarray, want: np.ndarray) -> float:
    """max|got - want| over max(max|want|, 1): max-rel, with outputs that are zero up to rounding (N = 1 gives
    dQ = dK = 0 exactly in real arithmetic) measured against the unit scale of the inputs."""
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1.0)) if want.size else 0.0


def _close(got: np.ndarray, want: np.ndarray, dtype: str) -> float:
    if dtype == "bfloat16":
        # The reference rounds its float32 result to bf16; the oracle result rounded the same way may land one ulp
        # away where the two float32 sums differ in their last bits.
        err = _err(bf16_round(got), want)
        assert err <= 2.0**-7, err
        return err
    err = _err(got, want)
    assert err <= TOL[dtype], err
    return err


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_matches_reference_golden(golden, name):
    c = golden_case(golden, name)
    dt, scale = c["_dtype"], c["_scale"]
    q, k, v, do, gq, gk, gv = (c[n] for n in ("q", "k", "v", "do", "gq", "gk", "gv"))
    o, lse = oracle.attn_fwd(q, k, v, scale)
    _close(o, c["o"], dt)
    assert oracle.max_rel(lse, c["lse"]) <= (1e-12 if dt == "float64" else 2e-6)
    # The backward passes take the reference's stored (rounded) O, as the op contract does.
    dq, dk, dv = oracle.attn_bwd(q, k, v, c["o"], c["lse"], do, scale)
    for got, want in ((dq, c["dq"]), (dk, c["dk"]), (dv, c["dv"])):
        _close(got, want, dt)
    hs = oracle.attn_bwd_bwd(q, k, v, c["o"], c["lse"], do, c["dq"], gq, gk, gv, scale)
    for got, want in zip(hs, (c["hq"], c["hk"], c["hv"], c["hdo"])):
        _close(got, want, dt)
    hs0 = oracle.attn_bwd_bwd(q, k, v, c["o"], c["lse"], do, c["dq"], gq, None, None, scale)
    for got, want in zip(hs0, (c["hq0"], c["hk0"], c["hv0"], c["hdo0"])):
        _close(got, want, dt)


def cfg1_inputs():
    torch.manual_seed(0)
    shape = (4, 8, 81, 64)
    q = torch.randn(shape) / 8
    k = torch.randn(shape) / 8
    v = torch.randn(shape) / 8
    do = torch.randn(shape)
    r = torch.randn(shape)
    return {n: t.numpy() for n, t in dict(q=q, k=k, v=v, do=do, r=r).items()}


def test_oracle_cfg1_against_reference_autograd(golden):
    """The fp32 B=4, L=81, H=8, D=64 case: O, first-order grads, and grad of sum(dQ * R) through the reference's
    autograd chain."""
    x = cfg1_inputs()
    for name, arr in x.items():
        want = golden[f"cfg1/in_sum/{name}"]
        got = np.array([arr.astype(np.float64).sum(), np.abs(arr.astype(np.float64)).sum()])
        np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-9)
    idx = golden["cfg1/index"]
    o, lse = oracle.attn_fwd(x["q"], x["k"], x["v"], 0.125)
    dq, dk, dv = oracle.attn_bwd(x["q"], x["k"], x["v"], o, lse, x["do"], 0.125)
    hq, hk, hv, _ = oracle.attn_bwd_bwd(x["q"], x["k"], x["v"], o, lse, x["do"], dq, x["r"], None, None, 0.125)
    for name, t in dict(o=o, dq=dq, dk=dk, dv=dv, hq=hq, hk=hk, hv=hv).items():
        assert oracle.max_rel(t.reshape(-1)[idx], golden[f"cfg1/{name}/sample"]) < 1e-5, name
        np.testing.assert_allclose(
            t.astype(np.float64).sum(axis=(2, 3)), golden[f"cfg1/{name}/bh_sum"], rtol=1e-4, atol=1e-5
        )
    rows = golden["cfg1/lse/rows"]
    assert oracle.max_rel(lse.reshape(-1)[rows], golden["cfg1/lse/sample"]) < 1e-6


def test_oracle_empty_and_single():
    z = np.zeros((2, 3, 0, 64), np.float32)
    o, lse = oracle.attn_fwd(z, z, z, 0.125)
    assert o.shape == z.shape and lse.shape == (2, 3, 0)
    q = np.random.default_rng(0).standard_normal((1, 1, 1, 8)).astype(np.float32)
    o, lse = oracle.attn_fwd(q, q, q, 0.3)
    np.testing.assert_allclose(o, q, rtol=1e-6)  # one key: P = 1
    assert abs(lse[0, 0, 0] - 0.3 * float((q * q).sum())) < 1e-5


def test_max_rel_metric():
    assert oracle.max_rel(np.array([1.0, 2.0]), np.array([1.0, 2.0])) == 0.0
    assert abs(oracle.max_rel(np.array([1.1, 2.0]), np.array([1.0, 2.0])) - 0.05) < 1e-12


def test_rope_restatement_matches_reference_fixtures(layers_golden):
    """oracle/rope.py (the GPU RoPE tests' yardstick) reproduces the reference's ref_split / ref_merge bit for bit."""
    import torch

    from oracle.rope import merge, split

    g_ = layers_golden

    def load(key):
        a = g_[key]
        if a.dtype == np.uint16:
            return torch.from_numpy(a.astype(np.int32)).to(torch.int16).view(torch.bfloat16)
        return torch.from_numpy(a)

    names = sorted({k.split("/")[1] for k in g_.files if k.startswith("rope/")})
    assert len(names) == 4
    for name in names:
        heads = int(g_[f"rope/{name}/meta"][1])
        t = {k: load(f"rope/{name}/{k}") for k in ("qkv", "cos", "sin", "q", "k", "v", "dq", "dk", "dv", "g")}
        qs = load(f"rope/{name}/qscale") if f"rope/{name}/qscale" in g_.files else None
        for a, r in zip(split(t["qkv"], t["cos"], t["sin"], heads, qs), (t["q"], t["k"], t["v"])):
            assert torch.equal(a, r), name
        assert torch.equal(merge(t["dq"], t["dk"], t["dv"], t["cos"], t["sin"], qs), t["g"]), name
