"""GPU parity of the sm_100a attention kernels against the CPU oracle (numpy restatement of reference.py).

Tolerances (forward within 2e-3 max-rel of an fp32 reference, first- and second-order gradients
within 1e-2). max-rel is the reference's metric, max|a - r| / max|r| (models/attention.py:156-161), against the oracle
run in fp32 on the same rounded inputs.

* fp16 I/O: the forward is asserted at 2e-3 max-rel with no allowance at all. fp16's own rounding of O is at most
  2^-11 of the largest element, so this bar shows the kernels' arithmetic error directly; the bf16 and fp16 calls run
  the same kernel templates (the element type only changes the conversions at load and store).
* bf16 I/O: rounding O to bf16 alone moves an element by up to 2^-9 of its value, i.e. up to 3.9e-3 of max|O| when
  the largest element sits at the bottom of its binade, so a plain 2e-3 bar against the unrounded reference is not
  reachable by ANY bf16-output kernel (the reference's Triton kernels included). The bf16 forward is therefore
  asserted at 2e-3 beyond each element's own half-ulp, and the plain max-rel is reported in the message.
* Gradients: 1e-2 beyond the half-ulp of the output type. float32 calls (IEEE CUDA-core kernels) within 1e-4, float64
  within 1e-10.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oracle

pytestmark = pytest.mark.gpu

if torch.cuda.is_available():
    from ebr_b200 import _native, fused_attn
    from ebr_b200.build import build

    build()

DEV = "cuda"
FWD_TOL = 2e-3
GRAD_TOL = 1e-2
TOL32, TOL64 = 1e-4, 1e-10
HALF_ULP = {torch.bfloat16: 2.0**-8, torch.float16: 2.0**-11}


def _np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype in (torch.bfloat16, torch.float16):
        t = t.float()
    return t.numpy()


def _maxrel(a, r) -> float:
    return oracle.max_rel(_np(a) if isinstance(a, torch.Tensor) else a, r)


def check_out(got: torch.Tensor, ref: np.ndarray, dtype, tol16: float, what: str, ulps: float = 0.5,
              floor: float = 1e-3) -> float:
    """Assert ``got`` (device) matches the oracle's ``ref``; returns the plain max-rel for the log.

    ``ulps``: 16-bit rounding allowance on top of the tolerance, in units of the type's ulp (0.5 against an unrounded
    reference, 1 against a reference rounded to the same type). ``floor``: smallest max|ref| used as the denominator,
    so outputs that are zero up to rounding (N = 1 gives dQ = dK = 0) are measured on the inputs' unit scale.
    """
    g = _np(got).astype(np.float64)
    r = ref.astype(np.float64)
    assert np.isfinite(g).all(), f"{what}: non-finite output"
    denom = max(np.abs(r).max(), floor) if r.size else 1.0
    plain = float(np.abs(g - r).max() / denom) if r.size else 0.0
    if dtype == torch.float16 and tol16 == FWD_TOL and ulps == 0.5:
        assert plain <= FWD_TOL, f"{what}: fp16 plain max-rel {plain:.3e} > {FWD_TOL}"
    elif dtype in HALF_ULP:
        allow = 2 * ulps * HALF_ULP[dtype]
        err = float(np.maximum(np.abs(g - r) - allow * np.abs(r), 0).max() / denom) if r.size else 0.0
        assert err <= tol16, f"{what}: {err:.3e} (plain max-rel {plain:.3e}) > {tol16}"
    else:
        tol = TOL64 if dtype == torch.float64 else TOL32
        assert plain <= tol, f"{what}: max-rel {plain:.3e} > {tol}"
    return plain


def make_inputs(B, H, N, D, dtype, seed=0, layout="contiguous"):
    """q, k, v (scaled like projected activations), dO, gQ, gK, gV on the device, seeded."""
    g = torch.Generator().manual_seed(seed)
    draw = lambda s=1.0: torch.randn(B, H, N, D, generator=g, dtype=torch.float64) * s
    q, k, v = draw(0.5), draw(0.5), draw(0.5)
    do, gq, gk, gv = draw(), draw(), draw(), draw()
    if layout == "qkv":
        # q / k / v as head-major views of one [B, N, 3 H D] projection, as EnergyAttention produces them.
        qkv = torch.cat([t.transpose(1, 2).reshape(B, N, H * D) for t in (q, k, v)], dim=-1)
        qkv = qkv.to(dtype).to(DEV)
        q, k, v = (x.view(B, N, H, D).transpose(1, 2) for x in qkv.split(H * D, dim=-1))
    elif layout == "odd":
        # token stride D + 8 elements keeps 16-byte rows; D + 1 does not (CUDA-core kernels take those).
        def pad(t):
            big = torch.zeros(B, H, N, D + 1, dtype=torch.float64)
            big[..., :D] = t
            return big.to(dtype).to(DEV)[..., :D]

        q, k, v = pad(q), pad(k), pad(v)
    else:
        q, k, v = (t.to(dtype).to(DEV) for t in (q, k, v))
    do, gq, gk, gv = (t.to(dtype).to(DEV) for t in (do, gq, gk, gv))
    return q, k, v, do, gq, gk, gv


SHAPES_16 = [
    (2, 3, 81, 64),  # cfg2-like slice count, ragged N
    (1, 2, 17, 64),
    (1, 1, 1, 64),
    (2, 2, 64, 64),
    (2, 2, 128, 64),
    (1, 2, 100, 64),
    (1, 2, 100, 128),
    (1, 2, 81, 128),
    (1, 2, 256, 64),
    (1, 1, 300, 128),
    (1, 1, 900, 64),
    # N > 128 edges of the paired forward and the multi-buffered backward: a second query tile of one row and a last
    # key step of one key (129), an odd tile count with a ragged 64-key step of more than 32 keys (191), exact
    # multiples of 64 and 128 (320, 384 at D = 128), several items per CTA across the grid (1000 keys, 16 slices).
    (1, 2, 129, 64),
    (1, 2, 191, 128),
    (2, 1, 320, 64),
    (1, 2, 384, 128),
    (2, 8, 1000, 64),
    # the kernel sweep's long and D = 128 shapes: L = 2048 at both head dims, D = 128 at L = 256 and 900
    (1, 1, 2048, 64),
    (1, 1, 2048, 128),
    (1, 1, 900, 128),
    (1, 2, 256, 128),
]


def run_all(q, k, v, do, gq, gk, gv, scale):
    o, lse = torch.ops.ebr_fused.attn_fwd(q, k, v, scale)
    dq, dk, dv = torch.ops.ebr_fused.attn_bwd(q, k, v, o, lse, do, scale)
    hs = torch.ops.ebr_fused.attn_bwd_bwd(q, k, v, o, lse, do, dq, gq, gk, gv, scale)
    torch.cuda.synchronize()
    _native.device_status()
    return o, lse, (dq, dk, dv), hs


def oracle_all(q, k, v, do, gq, gk, gv, o, lse, scale):
    """Oracle on the same (rounded) inputs; the backward passes take the kernel's stored o / lse, as the op chain
    does (the reference's ops pass the forward's outputs along)."""
    n = lambda t: _np(t).astype(np.float64 if t.dtype == torch.float64 else np.float32)
    Q, K, V, DO, GQ, GK, GV = map(n, (q, k, v, do, gq, gk, gv))
    O, LSE = oracle.attn_fwd(Q, K, V, scale)
    On, Ln = n(o), _np(lse)
    grads = oracle.attn_bwd(Q, K, V, On, Ln, DO, scale)
    hs = oracle.attn_bwd_bwd(Q, K, V, On, Ln, DO, None, GQ, GK, GV, scale)
    return O, LSE, grads, hs


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", SHAPES_16, ids=lambda s: "x".join(map(str, s)))
def test_parity_16bit(shape, dtype):
    B, H, N, D = shape
    scale = D**-0.5
    q, k, v, do, gq, gk, gv = make_inputs(B, H, N, D, dtype, seed=N * 7 + D)
    o, lse, grads, hs = run_all(q, k, v, do, gq, gk, gv, scale)
    O, LSE, G, HS = oracle_all(q, k, v, do, gq, gk, gv, o, lse, scale)
    check_out(o, O, dtype, FWD_TOL, "o")
    assert _maxrel(lse, LSE) < 1e-5
    for name, got, ref in zip(("dq", "dk", "dv"), grads, G):
        check_out(got, ref, dtype, GRAD_TOL, name)
    for name, got, ref in zip(("hq", "hk", "hv", "hdo"), hs, HS):
        check_out(got, ref, dtype, GRAD_TOL, name)


# Short-sequence packing: floor(128 / N) slices per 128-row tile, slice counts that do not divide evenly (the last
# tile is partial), and strided views whose slices are not at a uniform stride (the tile then packs a divisor of H).
PACKED = [
    ((3, 8, 17, 64), "contiguous"),   # 7 slices per tile, 24 slices: 4 tiles, the last with 3
    ((2, 5, 33, 64), "contiguous"),   # 3 per tile, 10 slices
    ((1, 5, 64, 64), "contiguous"),   # 2 per tile, 5 slices
    ((3, 3, 40, 128), "contiguous"),  # 3 per tile at D = 128, 9 slices
    ((2, 8, 17, 64), "qkv"),          # strided views: 4 heads (a divisor of 8) of one batch row per tile
    ((2, 6, 33, 64), "qkv"),          # 3 heads per tile
    ((37, 3, 100, 64), "contiguous"),  # one slice per tile, many tiles per CTA
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape,layout", PACKED, ids=lambda x: "x".join(map(str, x)) if isinstance(x, tuple) else x)
def test_parity_short_packed(shape, layout, dtype):
    B, H, N, D = shape
    scale = D**-0.5
    q, k, v, do, gq, gk, gv = make_inputs(B, H, N, D, dtype, seed=N * 3 + H, layout=layout)
    o, lse, grads, hs = run_all(q, k, v, do, gq, gk, gv, scale)
    O, LSE, G, HS = oracle_all(q, k, v, do, gq, gk, gv, o, lse, scale)
    check_out(o, O, dtype, FWD_TOL, "o")
    assert _maxrel(lse, LSE) < 1e-5
    for name, got, ref in zip(("dq", "dk", "dv", "hq", "hk", "hv", "hdo"), (*grads, *hs), (*G, *HS)):
        check_out(got, ref, dtype, GRAD_TOL, name)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_parity_growing_logits(dtype):
    """Logits that grow from one key tile to the next, differently per row, so the forward's lazy rescale of O runs
    for some rows of a warp and not others (unit-scale random inputs never trigger it)."""
    B, H, N, D = 2, 2, 900, 64
    q, k, v, do, gq, gk, gv = make_inputs(B, H, N, D, dtype, seed=77)
    g = torch.Generator().manual_seed(78)
    row_scale = (torch.rand(B, H, N, 1, generator=g) * 3.0 + 0.5).to(DEV)
    key_scale = torch.ones(1, 1, N, 1, device=DEV)
    key_scale[:, :, 384:] = 2.5
    key_scale[:, :, 768:] = 5.0
    q = (q.float() * row_scale * (1.0 if dtype == torch.bfloat16 else 0.5)).to(dtype)
    k = (k.float() * key_scale).to(dtype)
    o, lse, grads, hs = run_all(q, k, v, do, gq, gk, gv, D**-0.5)
    O, LSE, G, HS = oracle_all(q, k, v, do, gq, gk, gv, o, lse, D**-0.5)
    check_out(o, O, dtype, FWD_TOL, "o")
    assert _maxrel(lse, LSE) < 1e-5
    for got, ref in zip(grads, G):
        check_out(got, ref, dtype, GRAD_TOL, "grad")


@pytest.mark.parametrize("D", [64, 128])
def test_parity_forward_v_scale(D):
    """V whose magnitude changes across the key tiles of one slice and leaves fp16's range at both ends, each head
    judged on its own scale (a P V product carried in a 16-bit format with one fixed scale would lose these):
    h0: |v| rising 4x per 64-key tile up to 4^7 and falling back; h1: the first 200 keys' v all zero;
    h2: v x 3e5 (above fp16's largest finite 65504); h3: v x 1e-6 (fp16 subnormal)."""
    B, H, N = 1, 4, 900
    dtype = torch.bfloat16
    q, k, v, do, gq, gk, gv = make_inputs(B, H, N, D, dtype, seed=900 + D)
    tile = torch.arange(N, device=DEV) // 64
    f = torch.ones(H, N, device=DEV)
    f[0] = 4.0 ** torch.minimum(tile, 14 - tile).clamp(min=0).float()
    f[1, :200] = 0.0
    f[2] = 3e5
    f[3] = 1e-6
    v = (v.float() * f[None, :, :, None]).to(dtype)
    o, lse = torch.ops.ebr_fused.attn_fwd(q, k, v, D**-0.5)
    torch.cuda.synchronize()
    _native.device_status()
    n = lambda t: _np(t).astype(np.float32)
    O, LSE = oracle.attn_fwd(n(q), n(k), n(v), D**-0.5)
    for h in range(H):
        check_out(o[:, h], O[:, h], dtype, FWD_TOL, f"o head {h}", floor=0.0)
    assert _maxrel(lse, LSE) < 1e-5


@pytest.mark.parametrize("layout", ["qkv", "odd"])
def test_parity_strided_operands(layout):
    B, H, N, D = 2, 4, 81, 64
    dtype = torch.bfloat16
    q, k, v, do, gq, gk, gv = make_inputs(B, H, N, D, dtype, seed=3, layout=layout)
    assert not q.is_contiguous()
    assert fused_attn.uses_tensor_cores(q, k, v) == (layout == "qkv")
    o, lse, grads, hs = run_all(q, k, v, do, gq, gk, gv, D**-0.5)
    O, LSE, G, HS = oracle_all(q, k, v, do, gq, gk, gv, o, lse, D**-0.5)
    check_out(o, O, dtype, FWD_TOL, "o")
    for got, ref in zip((*grads, *hs), (*G, *HS)):
        check_out(got, ref, dtype, GRAD_TOL, "grad")


@pytest.mark.parametrize("dtype,shape", [
    (torch.float32, (2, 3, 81, 64)),
    (torch.float32, (1, 2, 33, 16)),
    (torch.float32, (1, 1, 300, 128)),
    (torch.float64, (1, 2, 17, 16)),
    (torch.float64, (1, 1, 130, 64)),
    (torch.bfloat16, (1, 2, 40, 32)),  # D = 32: CUDA-core kernels
])  # fmt: skip
def test_parity_cuda_core_kernels(dtype, shape):
    B, H, N, D = shape
    q, k, v, do, gq, gk, gv = make_inputs(B, H, N, D, dtype, seed=11)
    o, lse, grads, hs = run_all(q, k, v, do, gq, gk, gv, D**-0.5)
    O, LSE, G, HS = oracle_all(q, k, v, do, gq, gk, gv, o, lse, D**-0.5)
    tol16 = GRAD_TOL
    check_out(o, O, dtype, FWD_TOL, "o")
    for got, ref in zip((*grads, *hs), (*G, *HS)):
        check_out(got, ref, dtype, tol16, "grad")


def test_golden_cases_on_device(golden):
    """The committed reference outputs, reproduced by the kernels on the same inputs."""
    from tests.conftest import GOLDEN_CASES, golden_case

    tdt = {"float32": torch.float32, "float64": torch.float64, "bfloat16": torch.bfloat16}
    for name in GOLDEN_CASES:
        c = golden_case(golden, name)
        dtype = tdt[c["_dtype"]]
        dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dtype).to(DEV)
        q, k, v, do, gq, gk, gv = (dev(c[n]) for n in ("q", "k", "v", "do", "gq", "gk", "gv"))
        o, lse, grads, hs = run_all(q, k, v, do, gq, gk, gv, c["_scale"])
        # The golden outputs are already rounded to the input type: allow one ulp of rounding difference.
        check_out(o, c["o"], dtype, FWD_TOL, f"{name}/o", ulps=1.0)
        for n_, got in zip(("dq", "dk", "dv"), grads):
            check_out(got, c[n_], dtype, GRAD_TOL, f"{name}/{n_}", ulps=1.0)
        for n_, got in zip(("hq", "hk", "hv", "hdo"), hs):
            check_out(got, c[n_], dtype, GRAD_TOL, f"{name}/{n_}", ulps=1.0)


def test_cfg1_golden_on_device(golden):
    """BASELINE config 1 through the op chain on the device (fp32, B=4, L=81, H=8, D=64, seed 0: O, then dQ/dK/dV
    with create_graph=True, then the gradient of sum(dQ * R)), against the reference's own outputs stored in the
    golden file: 4096 sampled entries of every output and its per-(b, h) sums. The inputs are redrawn from the seed
    and checked against the stored checksums first."""
    from tests.golden.make_golden import cfg1_inputs

    x = cfg1_inputs()
    for name, t in x.items():
        assert np.allclose(golden[f"cfg1/in_sum/{name}"], [t.double().sum().item(), t.double().abs().sum().item()],
                           rtol=1e-12, atol=1e-9), name  # fmt: skip
    q, k, v = (x[n].to(DEV).requires_grad_(True) for n in ("q", "k", "v"))
    o = fused_attn.fused_attention(q, k, v)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), grad_outputs=x["do"].to(DEV), create_graph=True)
    hq, hk, hv = torch.autograd.grad((dq * x["r"].to(DEV)).sum(), (q, k, v))
    torch.cuda.synchronize()
    _native.device_status()
    idx = golden["cfg1/index"]
    for name, t in {"o": o, "dq": dq, "dk": dk, "dv": dv, "hq": hq, "hk": hk, "hv": hv}.items():
        got = t.detach().double().cpu()
        ref = golden[f"cfg1/{name}/sample"].astype(np.float64)
        err = float(np.abs(got.reshape(-1).numpy()[idx] - ref).max() / np.abs(ref).max())
        assert err <= TOL32, f"cfg1 {name}: sampled max-rel {err:.3e}"
        sums = got.sum(dim=(2, 3)).numpy()
        ref_sums = golden[f"cfg1/{name}/bh_sum"]
        scale = max(np.abs(ref_sums).max(), float(got.abs().sum(dim=(2, 3)).max()) * 1e-3)
        assert np.abs(sums - ref_sums).max() <= 1e-4 * scale, f"cfg1 {name}: per-(b, h) sums"


@pytest.mark.parametrize("shape", [(2, 2, 81, 64), (1, 2, 300, 64), (1, 2, 200, 128)], ids=str)
@pytest.mark.parametrize("null", ["gk_gv", "gq", "gq_gk_gv"])
def test_zero_cotangents_through_c_abi(shape, null):
    """NULL cotangents at the C ABI equal explicit zeros (the reference expands a zero row, triton_kernels.py:868-873),
    for the single-tile and the tiled double-backward kernels."""
    import ctypes

    B, H, N, D = shape
    q, k, v, do, gq, gk, gv = make_inputs(B, H, N, D, torch.bfloat16, seed=5)
    scale = D**-0.5
    o, lse = torch.ops.ebr_fused.attn_fwd(q, k, v, scale)
    dq, _, _ = torch.ops.ebr_fused.attn_bwd(q, k, v, o, lse, do, scale)
    z = torch.zeros_like(q)
    nulls = set(null.split("_"))
    g = {n: (z if n in nulls else t) for n, t in (("gq", gq), ("gk", gk), ("gv", gv))}
    ref = torch.ops.ebr_fused.attn_bwd_bwd(q, k, v, o, lse, do, dq, g["gq"], g["gk"], g["gv"], scale)
    outs = [torch.empty_like(q) for _ in range(4)]
    lib = _native.lib()
    nbytes = lib.ebr_attn_bwd_bwd_scratch_bytes(_native.BFLOAT16, B, H, N, D)
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    op = lambda t: _native.Operand(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))
    ops = [op(t) for t in (q, k, v, do)]
    gops = {n: (None if n in nulls else op(t)) for n, t in (("gq", gq), ("gk", gk), ("gv", gv))}
    r = ctypes.byref
    rr = lambda x: None if x is None else r(x)
    st = lib.ebr_attn_bwd_bwd(_native.BFLOAT16, B, H, N, D, scale, r(ops[0]), r(ops[1]), r(ops[2]), o.data_ptr(),
                              lse.data_ptr(), r(ops[3]), dq.data_ptr(), rr(gops["gq"]), rr(gops["gk"]), rr(gops["gv"]),
                              *[t.data_ptr() for t in outs], scratch.data_ptr(), nbytes,
                              torch.cuda.current_stream().cuda_stream)  # fmt: skip
    assert st == 0
    torch.cuda.synchronize()
    for a, b in zip(outs, ref):
        # Skipped zero products leave the same sums; allow the last-bit differences of a different summation order.
        assert _maxrel(a, _np(b)) <= 1e-2


def test_autograd_second_order_matches_oracle():
    """fused_attention with create_graph=True, then the gradient of <dQ, R> (bf16 and fp32)."""
    for dtype in (torch.bfloat16, torch.float32):
        B, H, N, D = 4, 8, 81, 64
        q0, k0, v0, do, r, _, _ = make_inputs(B, H, N, D, dtype, seed=0)
        q, k, v = (t.detach().clone().requires_grad_(True) for t in (q0, k0, v0))
        o = fused_attn.fused_attention(q, k, v)
        dq, dk, dv = torch.autograd.grad(o, (q, k, v), grad_outputs=do, create_graph=True)
        hq, hk, hv = torch.autograd.grad((dq * r).sum(), (q, k, v))
        n = lambda t: _np(t).astype(np.float32)
        Q, K, V, DO, R = map(n, (q0, k0, v0, do, r))
        O, L = oracle.attn_fwd(Q, K, V, 0.125)
        On = n(o)
        G = oracle.attn_bwd(Q, K, V, On, L, DO, 0.125)
        HS = oracle.attn_bwd_bwd(Q, K, V, On, L, DO, None, R, None, None, 0.125)
        check_out(o, O, dtype, FWD_TOL, "o")
        for got, ref in zip((dq, dk, dv, hq, hk, hv), (*G, *HS[:3])):
            check_out(got, ref, dtype, GRAD_TOL, "autograd")


def test_deterministic():
    q, k, v, do, gq, gk, gv = make_inputs(3, 4, 100, 64, torch.bfloat16, seed=9)
    a = run_all(q, k, v, do, gq, gk, gv, 0.125)
    b = run_all(q, k, v, do, gq, gk, gv, 0.125)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    for x, y in zip((*a[2], *a[3]), (*b[2], *b[3])):
        assert torch.equal(x, y)


def test_compiled_func_grad_smoke():
    """torch.compile(torch.func.grad(...)) traces the ops as opaque nodes (the reference's energy_compile path)."""
    q, k, v, *_ = make_inputs(2, 2, 81, 64, torch.bfloat16, seed=1)

    def energy(x):
        return fused_attn.fused_attention(x, k, v).float().square().sum()

    eager = torch.func.grad(energy)(q)
    compiled = torch.compile(torch.func.grad(energy), backend="aot_eager")(q)
    assert torch.equal(eager, compiled)


def test_large_batch_slices():
    """Many (b, h) slices in one launch (grid x = B * H), cfg2-sized head count."""
    B, H, N, D = 96, 8, 81, 64
    q, k, v, do, gq, gk, gv = make_inputs(B, H, N, D, torch.bfloat16, seed=21)
    o, lse, grads, hs = run_all(q, k, v, do, gq, gk, gv, 0.125)
    sel = slice(90, 96)
    sub = lambda t: t[sel]
    O, LSE, G, HS = oracle_all(*(sub(t) for t in (q, k, v, do, gq, gk, gv)), sub(o), sub(lse), 0.125)
    check_out(sub(o), O, torch.bfloat16, FWD_TOL, "o")
    for got, ref in zip((*grads, *hs), (*G, *HS)):
        check_out(sub(got), ref, torch.bfloat16, GRAD_TOL, "grad")
