"""The fused kernels around the attention (include/ebr_layers.h) on the B200, against the reference:

* 2D-RoPE split / merge: bit-exact against the reference's own ``ref_split`` / ``ref_merge`` outputs (the fixtures
  of ``tests/golden/make_golden.py``, models/fused_attn/rope_split.py:31-67) and, on larger and strided inputs,
  against the oracle's restatement of them (``oracle/rope.py``, itself pinned bit for bit to those fixtures) and the
  oracle's broadcast rotation (models/layers.py:115-131), in bf16 / fp16 / fp32 / fp64, with and without the per-head
  temperature; the merge is the split's adjoint (<split(x), y> = <x, merge(y)>) and autograd passes gradcheck and
  gradgradcheck in float64;
* residual + rms_norm, SwiGLU activation, the descent point and step: equal to the eager ops up to the order of the
  row sums (at most one unit in the last place of the I/O type, on a small fraction of elements), first derivatives
  within 1e-2 max-rel of float64 autograd, second derivatives (create_graph) matching the eager ops' own;
* the energy network with fused layers against the oracle's eager restatement of the reference network (same fused
  attention): dE/dz within the network's bf16 noise floor (the deviation that swapping fp32 for fp64 inside the
  attention already causes).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"
DTYPES = [torch.bfloat16, torch.float16, torch.float32, torch.float64]


def _tables(h=9, w=9, d=64):
    """The reference's RotaryTable2D tables ([H * W, D] cos, sign-folded sin) on the device."""
    from oracle.energy import rope_tables

    cos, sin = rope_tables({"board": (h, w), "hidden": d, "heads": 1})
    return cos.to(DEV), sin.to(DEV)


def quarter_swap(x):
    from oracle.rope import quarter_swap as qs

    return qs(x)


def ref_split(qkv, cos, sin, heads, qscale=None):
    from oracle.rope import split

    return split(qkv, cos, sin, heads, qscale)


def ref_merge(dq, dk, dv, cos, sin, qscale=None):
    from oracle.rope import merge

    return merge(dq, dk, dv, cos, sin, qscale)


def test_rope_kernels_reproduce_reference_fixtures(layers_golden):
    """The split and merge kernels on the reference's own inputs reproduce its outputs bit for bit."""
    import numpy as np

    from ebr_b200.layers import rope_merge_op, rope_split_op

    g_ = layers_golden

    def load(key, dtype):
        a = g_[key]
        if a.dtype == np.uint16:
            return torch.from_numpy(a.astype(np.int32)).to(torch.int16).view(torch.bfloat16).to(DEV)
        return torch.from_numpy(a).to(DEV)

    for name in sorted({k.split("/")[1] for k in g_.files if k.startswith("rope/")}):
        meta = g_[f"rope/{name}/meta"]
        dtype, heads = getattr(torch, str(meta[0])), int(meta[1])
        t = {k: load(f"rope/{name}/{k}", dtype) for k in ("qkv", "cos", "sin", "q", "k", "v", "dq", "dk", "dv", "g")}
        qs = load(f"rope/{name}/qscale", dtype) if f"rope/{name}/qscale" in g_.files else torch.zeros(0, device=DEV)
        got = rope_split_op(t["qkv"], t["cos"], t["sin"], qs, heads)
        for a, r in zip(got, (t["q"], t["k"], t["v"])):
            assert a.dtype == r.dtype and torch.equal(a, r), name
        assert torch.equal(rope_merge_op(t["dq"], t["dk"], t["dv"], t["cos"], t["sin"], qs), t["g"]), name


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("with_scale", [False, True])
def test_rope_split_and_merge_bit_exact(dtype, with_scale):
    from ebr_b200.layers import rope_merge_op, rope_split_op

    cos, sin = _tables()
    g = torch.Generator(device="cpu").manual_seed(3)
    b, n, h, d = 3, 81, 8, 64
    qkv = torch.randn(b, n, 3 * h * d, generator=g).to(DEV, dtype)
    qs = (torch.rand(h, generator=g) + 0.5).to(dtype).to(DEV) if with_scale else None
    empty = torch.zeros(0, device=DEV)
    got = rope_split_op(qkv, cos, sin, qs if with_scale else empty, h)
    for a, r in zip(got, ref_split(qkv, cos, sin, h, qs)):
        assert torch.equal(a, r)
    dq, dk, dv = (torch.randn(b, h, n, d, generator=g).to(DEV, dtype) for _ in range(3))
    out = rope_merge_op(dq, dk, dv, cos, sin, qs if with_scale else empty)
    assert torch.equal(out, ref_merge(dq, dk, dv, cos, sin, qs))


def test_rope_split_matches_the_eager_apply_rope_path():
    """The [N, D] tables with folded signs give exactly the eager split + apply_rope + transpose (+ temperature)."""
    from ebr_b200.layers import rope_split

    from oracle.energy import rotate

    cos, sin = _tables()
    g = torch.Generator(device="cpu").manual_seed(4)
    b, n, h, d = 2, 81, 8, 64
    qkv = torch.randn(b, n, 3 * h * d, generator=g).to(DEV, torch.bfloat16)
    temp = (torch.randn(h, generator=g) * 0.1).to(DEV).exp().to(torch.bfloat16)
    q, k, v = qkv.split([h * d] * 3, dim=-1)
    q, k = rotate(q.reshape(b, n, h, d), cos, sin), rotate(k.reshape(b, n, h, d), cos, sin)
    q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.reshape(b, n, h, d).transpose(1, 2)
    q = q * temp.view(1, -1, 1, 1)
    fq, fk, fv = rope_split(qkv, cos, sin, h, temp)
    assert torch.equal(fq, q) and torch.equal(fk, k) and torch.equal(fv, v)


def test_rope_strided_qkv_and_odd_head_dim():
    from ebr_b200.layers import rope_merge_op, rope_split_op

    g = torch.Generator(device="cpu").manual_seed(5)
    for d in (64, 20):  # vector path; D % 32 != 0 takes the one-element path
        cos, sin = _tables(3, 5, d)
        b, n, h = 2, 15, 3
        big = torch.randn(b, n, 3 * h * d + 8, generator=g).to(DEV, torch.bfloat16)
        qkv = big[..., : 3 * h * d]  # token stride 3 h d + 8
        empty = torch.zeros(0, device=DEV)
        for a, r in zip(rope_split_op(qkv, cos, sin, empty, h), ref_split(qkv.contiguous(), cos, sin, h)):
            assert torch.equal(a, r)
        dq = torch.randn(b, n, h, d, generator=g).to(DEV, torch.bfloat16).transpose(1, 2)  # strided [B, H, N, D]
        dk, dv = dq.contiguous(), dq * 2
        assert torch.equal(rope_merge_op(dq, dk, dv, cos, sin, empty), ref_merge(dq, dk, dv, cos, sin))


def test_rope_merge_is_the_adjoint_and_autograd_is_exact():
    from ebr_b200.layers import rope_merge_op, rope_split, rope_split_op

    cos, sin = _tables(3, 4, 16)
    g = torch.Generator(device="cpu").manual_seed(6)
    b, n, h, d = 2, 12, 2, 16
    qkv = torch.randn(b, n, 3 * h * d, generator=g, dtype=torch.float64).to(DEV)
    ys = [torch.randn(b, h, n, d, generator=g, dtype=torch.float64).to(DEV) for _ in range(3)]
    empty = torch.zeros(0, device=DEV)
    lhs = sum((a * y).sum() for a, y in zip(rope_split_op(qkv, cos, sin, empty, h), ys))
    rhs = (qkv * rope_merge_op(*ys, cos, sin, empty)).sum()
    assert abs(float(lhs - rhs)) <= 1e-10 * abs(float(lhs))
    x = qkv.clone().requires_grad_(True)
    fn = lambda t: rope_split(t, cos, sin, h)
    assert torch.autograd.gradcheck(fn, (x,), eps=1e-6, atol=1e-8)
    assert torch.autograd.gradgradcheck(fn, (x,), eps=1e-6, atol=1e-8)


QKV_SHAPES = [(2, 9, 9, 8, 64, 512), (1, 30, 30, 8, 64, 512), (3, 10, 10, 2, 128, 256), (1, 3, 4, 4, 64, 128)]


def _qkv_inputs(shape, dtype, seed):
    b, hh, ww, h, d, c = shape
    cos, sin = _tables(hh, ww, d)
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(b, hh * ww, c, generator=g).to(dtype).to(DEV)
    w = (torch.randn(3 * h * d, c, generator=g) * c**-0.5).to(dtype).to(DEV)
    qs = (torch.rand(h, generator=g) + 0.5).to(dtype).float().to(DEV)
    return x, w, cos, sin, qs, h


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", QKV_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("with_scale", [False, True])
def test_qkv_rope_split_is_the_projection_then_the_split(dtype, shape, with_scale):
    """The fused GEMM + split equals the reference's dense split of the correctly rounded projection (x W^T summed
    exactly, rounded once) and the unfused cuBLAS GEMM + split kernel, up to the last bit of a projection value whose
    fp32 sum rounds the other way (rare): a rotated output t c + swap(t) s then moves by at most a few units of
    eps (|t| + |swap(t)|), which near a cancellation is many ulps of the output itself. Row counts that are not a
    multiple of the 128-row tile, D = 128 and a 256-column q / k / v section are included."""
    from ebr_b200.layers import qkv_fusable, qkv_rope_split_op, rope_split_op

    x, w, cos, sin, qs, h = _qkv_inputs(shape, dtype, seed=sum(shape))
    b, n, _ = x.shape
    d = w.shape[0] // (3 * h)
    assert qkv_fusable(x, w, h)
    scale = qs if with_scale else torch.zeros(0, device=DEV)
    got = qkv_rope_split_op(x, w, cos, sin, scale, h)
    exact = (x.double() @ w.double().t()).to(dtype)
    ref = ref_split(exact, cos, sin, h, qs if with_scale else None)
    # cuBLAS summing in fp32 throughout (torch otherwise lets 16-bit GEMMs reduce partial sums in 16 bits).
    m = torch.backends.cuda.matmul
    flags = (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction)
    m.allow_bf16_reduced_precision_reduction = m.allow_fp16_reduced_precision_reduction = False
    try:
        unfused = rope_split_op(F.linear(x, w), cos, sin, scale, h)
    finally:
        m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction = flags
    # Per output element: the magnitude of the rotation's two inputs (v: the element itself) and the bound on their
    # fp32 summation error (K 2^-24 sum |x_i w_i|, which dominates for values near zero), head-major.
    def per_output(t):
        t = t.view(b, n, 3, h, d)
        t = torch.cat([t[:, :, :2] + quarter_swap(t[:, :, :2]), t[:, :, 2:]], dim=2).permute(2, 0, 3, 1, 4)
        if with_scale:
            t[0] = t[0] * qs.double().view(1, h, 1, 1)
        return t

    mag = per_output(exact.double().abs())
    acc = per_output((x.double().abs() @ w.double().abs().t()) * (x.shape[-1] * 2.0**-24))
    eps = torch.finfo(dtype).eps
    for part, (a, r, u) in enumerate(zip(got, ref, unfused)):
        for other in (r, u):
            diff = (a.double() - other.double()).abs()
            bound = 3 * eps * mag[part] + 2 * acc[part]
            assert bool((diff <= bound).all()), float((diff / bound).max())
            assert float((a != other).double().mean()) < 0.01


def test_qkv_rope_split_gradients_match_the_unfused_path_to_second_order():
    """First and second derivatives (create_graph) in x and the weight equal those of F.linear + rope_split, and a
    backward asked for x alone or the weight alone returns that gradient."""
    from ebr_b200.layers import qkv_rope_split, rope_split

    x0, w0, cos, sin, qs, h = _qkv_inputs((2, 9, 9, 8, 64, 512), torch.bfloat16, seed=3)
    g = torch.Generator(device="cpu").manual_seed(4)
    r = torch.randn(x0.shape, generator=g).to(x0.dtype).to(DEV)

    def run(fused):
        x, w = x0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
        q, k, v = qkv_rope_split(x, w, cos, sin, h, qs) if fused else rope_split(F.linear(x, w), cos, sin, h, qs)
        s = (q.float() * k.float()).sum() + (v.float() ** 2).sum()
        gx, gw = torch.autograd.grad(s, (x, w), create_graph=True)
        hw = torch.autograd.grad((gx.float() * r.float()).sum(), w)[0]
        return gx, gw, hw

    for a, b in zip(run(True), run(False)):
        err = float((a.double() - b.double()).abs().max() / b.double().abs().max())
        assert err < 1e-2, err

    # A backward that asks for one input only gets it (the other product is skipped, not its own input's).
    for want in (0, 1):
        got = []
        for fused in (True, False):
            x, w = x0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
            q, k, v = qkv_rope_split(x, w, cos, sin, h, qs) if fused else rope_split(F.linear(x, w), cos, sin, h, qs)
            got.append(torch.autograd.grad((q.float() * k.float()).sum() + (v.float() ** 2).sum(), (x, w)[want])[0])
        if want == 1:
            assert torch.equal(got[0], got[1])
        else:
            # x alone: the merge folded into the GEMM's A operand (ebr_qkv_rope_merge_dx), whose fp32 sums run in
            # another order than cuBLAS's: equal up to last-bit differences.
            err = float((got[0].double() - got[1].double()).abs().max() / got[1].double().abs().max())
            assert err < 1e-2 and float((got[0] != got[1]).double().mean()) < 0.05, err


O_SHAPES = [(2, 8, 81, 64, 512), (1, 8, 900, 64, 512), (3, 2, 100, 128, 256), (2, 4, 300, 64, 256)]


def _o_inputs(shape, dtype, seed, token_major=False):
    b, h, n, d, c = shape
    g = torch.Generator(device="cpu").manual_seed(seed)
    if token_major:  # the layout a [B, N, H, D] buffer viewed head-major gives (strides N H D, D, H D, 1)
        o = (torch.randn(b, n, h, d, generator=g) * 0.5).to(dtype).to(DEV).transpose(1, 2)
    else:
        o = (torch.randn(b, h, n, d, generator=g) * 0.5).to(dtype).to(DEV)
    w = (torch.randn(c, h * d, generator=g) * (h * d) ** -0.5).to(dtype).to(DEV)
    return o, w


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", O_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("token_major", [False, True])
def test_o_proj_is_the_gemm_of_the_transposed_output(dtype, shape, token_major):
    """y = O^T-reshaped times W^T read from the head-major output: within one rounding of the exact product (plus the
    fp32 summation bound for values near zero) and equal to cuBLAS with fp32 reduction but for a last-bit difference
    of a sum taken in another order; token counts that are not a multiple of 128 and both O layouts included."""
    from ebr_b200.layers import o_proj_fusable, o_proj_op

    b, h, n, d, c = shape
    o, w = _o_inputs(shape, dtype, seed=sum(shape), token_major=token_major)
    assert o_proj_fusable(o, w)
    got = o_proj_op(o, w)
    x = o.transpose(1, 2).reshape(b, n, h * d)
    exact = x.double() @ w.double().t()
    ref = exact.to(dtype)
    acc = (x.double().abs() @ w.double().abs().t()) * (h * d * 2.0**-24)
    eps = torch.finfo(dtype).eps
    diff = (got.double() - ref.double()).abs()
    assert bool((diff <= 2 * eps * ref.double().abs() + 2 * acc).all()), float((diff / (ref.double().abs() + acc)).max())
    m = torch.backends.cuda.matmul
    flags = (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction)
    m.allow_bf16_reduced_precision_reduction = m.allow_fp16_reduced_precision_reduction = False
    try:
        unfused = F.linear(x, w)
    finally:
        m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction = flags
    assert float((got != unfused).double().mean()) < 0.01


def test_o_proj_gradients_match_the_unfused_path_to_second_order():
    """First and second derivatives (create_graph) in O and the weight equal those of transpose + F.linear, and a
    backward asked for one input alone returns that gradient."""
    from ebr_b200.layers import o_proj

    o0, w0 = _o_inputs((2, 8, 81, 64, 512), torch.bfloat16, seed=9)
    b, h, n, d = o0.shape
    g = torch.Generator(device="cpu").manual_seed(10)
    r = torch.randn(o0.shape, generator=g).to(o0.dtype).to(DEV)

    def proj(o, w, fused):
        return o_proj(o, w) if fused else F.linear(o.transpose(1, 2).reshape(b, n, h * d), w)

    def run(fused):
        o, w = o0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
        s = (proj(o, w, fused).float() ** 2).sum()
        go, gw = torch.autograd.grad(s, (o, w), create_graph=True)
        hw = torch.autograd.grad((go.float() * r.float()).sum(), w)[0]
        return go, gw, hw

    for a, bb in zip(run(True), run(False)):
        err = float((a.double() - bb.double()).abs().max() / bb.double().abs().max())
        assert err < 1e-2, err
    for want in (0, 1):
        got = []
        for fused in (True, False):
            o, w = o0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
            got.append(torch.autograd.grad((proj(o, w, fused).float() ** 2).sum(), (o, w)[want])[0])
        err = float((got[0].double() - got[1].double()).abs().max() / got[1].double().abs().max())
        assert err < 1e-2, err


MERGE_DX_SHAPES = [(2, 8, 81), (1, 8, 900), (3, 8, 130), (1, 4, 300)]  # (B, H, N) at D = 64, C = 512


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", MERGE_DX_SHAPES, ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("with_scale", [False, True])
def test_qkv_rope_merge_dx_is_the_merge_then_the_gemm(dtype, shape, with_scale):
    """dx = rope_merge(dq, dk, dv) W with the merge done on the GEMM's A tiles in shared memory: within one rounding
    of the exact product of the merged gradient (the merge kernel's own 16-bit output, bit-exact against the
    reference's fixtures) and W, plus the fp32 summation bound, and equal to cuBLAS with fp32 reduction but for a
    last-bit difference of a sum taken in another order. Token counts that are not a multiple of 128 (partial m-tiles
    per sample), a strided dk and the per-head temperature included."""
    from ebr_b200.layers import merge_dx_fusable, qkv_rope_merge_dx_op, rope_merge_op

    b, h, n = shape
    d, c = 64, 512
    g = torch.Generator(device="cpu").manual_seed(b * 1000 + h * 100 + n)
    dq, dv = (torch.randn(b, h, n, d, generator=g).to(dtype).to(DEV) for _ in range(2))
    dk = torch.randn(b, n, h, d, generator=g).to(dtype).to(DEV).transpose(1, 2)  # head-major view, token stride h d
    w = (torch.randn(3 * h * d, c, generator=g) * (3 * h * d) ** -0.5).to(dtype).to(DEV)
    cos, sin = (torch.rand(n, d, generator=g).to(DEV) * 2 - 1 for _ in range(2))
    qs = (torch.rand(h, generator=g) + 0.5).to(DEV) if with_scale else torch.zeros(0, device=DEV)
    assert merge_dx_fusable(dq, w)
    got = qkv_rope_merge_dx_op(dq, dk, dv, w, cos, sin, qs)
    merged = rope_merge_op(dq, dk, dv, cos, sin, qs)
    exact = merged.double() @ w.double()
    ref = exact.to(dtype)
    acc = (merged.double().abs() @ w.double().abs()) * (3 * h * d * 2.0**-24)
    eps = torch.finfo(dtype).eps
    diff = (got.double() - ref.double()).abs()
    assert bool((diff <= 2 * eps * ref.double().abs() + 2 * acc).all()), float((diff / (ref.double().abs() + acc)).max())
    m = torch.backends.cuda.matmul
    flags = (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction)
    m.allow_bf16_reduced_precision_reduction = m.allow_fp16_reduced_precision_reduction = False
    try:
        unfused = merged @ w
    finally:
        m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction = flags
    assert float((got != unfused).double().mean()) < 0.01
    # a residual gradient joined in: exactly the separate 16-bit add of the two
    res = torch.randn(b, n, c, generator=g).to(dtype).to(DEV)
    assert torch.equal(qkv_rope_merge_dx_op(dq, dk, dv, w, cos, sin, qs, res), got + res)


GU_SHAPES = [(2, 81, 512, 1536), (1, 900, 512, 1536), (3, 100, 256, 128), (2, 37, 128, 256)]


def _gu_inputs(shape, dtype, seed):
    b, n, c, i = shape
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(b, n, c, generator=g).to(dtype).to(DEV)
    w = (torch.randn(2 * i, c, generator=g) * c**-0.5).to(dtype).to(DEV)
    return x, w


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", GU_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_gate_up_swiglu_is_the_gemm_then_the_activation(dtype, shape):
    """h equals cuBLAS with fp32 reduction (but for last-bit differences of a sum taken in another order, bounded by
    one rounding plus the fp32 summation error) and act equals the activation kernel applied to that h, bit for bit."""
    from ebr_b200.layers import gate_up_fusable, gate_up_swiglu_op

    b, n, c, i = shape
    x, w = _gu_inputs(shape, dtype, seed=sum(shape))
    assert gate_up_fusable(x, w)
    h, act = gate_up_swiglu_op(x, w)
    exact = x.double() @ w.double().t()
    ref = exact.to(dtype)
    accb = (x.double().abs() @ w.double().abs().t()) * (c * 2.0**-24)
    eps = torch.finfo(dtype).eps
    diff = (h.double() - ref.double()).abs()
    assert bool((diff <= 2 * eps * ref.double().abs() + 2 * accb).all())
    m = torch.backends.cuda.matmul
    flags = (m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction)
    m.allow_bf16_reduced_precision_reduction = m.allow_fp16_reduced_precision_reduction = False
    try:
        unfused = F.linear(x, w)
    finally:
        m.allow_bf16_reduced_precision_reduction, m.allow_fp16_reduced_precision_reduction = flags
    assert float((h != unfused).double().mean()) < 0.01
    from ebr_b200.layers import swiglu_act

    with torch.no_grad():
        assert torch.equal(act, swiglu_act(h))


def test_gate_up_swiglu_gradients_match_the_unfused_path_to_second_order():
    """First and second derivatives (create_graph) in x and the weight equal those of F.linear + swiglu_act, and a
    backward asked for one input alone returns that gradient."""
    from ebr_b200.layers import gate_up_swiglu, swiglu_act

    x0, w0 = _gu_inputs((2, 81, 512, 1536), torch.bfloat16, seed=12)
    g = torch.Generator(device="cpu").manual_seed(13)
    r = torch.randn(x0.shape, generator=g).to(x0.dtype).to(DEV)

    def act(x, w, fused):
        return gate_up_swiglu(x, w) if fused else swiglu_act(F.linear(x, w))

    def run(fused):
        x, w = x0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
        s = (act(x, w, fused).float() ** 2).sum()
        gx, gw = torch.autograd.grad(s, (x, w), create_graph=True)
        hw = torch.autograd.grad((gx.float() * r.float()).sum(), w)[0]
        return gx, gw, hw

    for a, bb in zip(run(True), run(False)):
        err = float((a.double() - bb.double()).abs().max() / bb.double().abs().max())
        assert err < 1e-2, err
    for want in (0, 1):
        got = []
        for fused in (True, False):
            x, w = x0.clone().requires_grad_(True), w0.clone().requires_grad_(True)
            got.append(torch.autograd.grad((act(x, w, fused).float() ** 2).sum(), (x, w)[want])[0])
        err = float((got[0].double() - got[1].double()).abs().max() / got[1].double().abs().max())
        assert err < 1e-2, err


def _check_rounding(a, r):
    """16-bit outputs: at most one ulp apart on under 2% of the elements (a row sum in another order can move a
    rounding); float32: a few ulps (no final rounding hides the sum-order difference)."""
    ulps, frac = _ulp_diff(a, r)
    if a.dtype in (torch.bfloat16, torch.float16):
        assert ulps <= 1.0 and frac < 0.02, (ulps, frac)
    else:
        assert ulps <= 8.0, ulps


def _ulp_diff(a, r):
    """Largest difference in units of the I/O type's last place, and the fraction of unequal elements."""
    eps = torch.finfo(a.dtype).eps
    diff = (a.double() - r.double()).abs()
    scale = r.double().abs().clamp_min(torch.finfo(a.dtype).tiny)
    return float((diff / (scale * eps)).max()), float((a != r).double().mean())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_add_rms_norm_forward_and_backward(dtype):
    from oracle.energy import rms_norm
    from ebr_b200.layers import add_rms_norm

    g = torch.Generator(device="cpu").manual_seed(7)
    x = torch.randn(4, 81, 512, generator=g).to(DEV, dtype)
    a = torch.randn(4, 81, 512, generator=g).to(DEV, dtype)
    gy = torch.randn(4, 81, 512, generator=g).to(DEV, dtype)
    y = add_rms_norm(x, a)
    _check_rounding(y, rms_norm(x + a))
    # first derivative against float64 autograd of the same function on the rounded sum
    xr, ar = x.clone().requires_grad_(True), a.clone().requires_grad_(True)
    (gx, ga) = torch.autograd.grad(add_rms_norm(xr, ar), (xr, ar), gy)
    s64 = (x + a).double().requires_grad_(True)
    (g64,) = torch.autograd.grad(s64 * torch.rsqrt(s64.square().mean(-1, keepdim=True) + 1e-5), s64, gy.double())
    rel = float((gx.double() - g64).abs().max() / g64.abs().max())
    assert rel < 1e-2 and torch.equal(gx, ga), rel


def test_add_rms_norm_second_order_matches_eager():
    """Under create_graph the backward is a kernel whose own backward is the closed-form double backward
    (ebr_rms_norm_bwd2): d<dy/dx gy, u> with respect to x, a and the upstream gradient gy (which depends on the
    parameters downstream in training) equals the eager ops' own; float32 and bf16 (against eager in float64)."""
    from oracle.energy import rms_norm
    from ebr_b200.layers import add_rms_norm

    g = torch.Generator(device="cpu").manual_seed(8)
    x0 = torch.randn(3, 17, 256, generator=g).to(DEV)
    a0 = torch.randn(3, 17, 256, generator=g).to(DEV)
    gy0, u = (torch.randn(3, 17, 256, generator=g).to(DEV) for _ in range(2))

    def hvp(fn, dt):
        x, a = x0.to(dt).clone().requires_grad_(True), a0.to(dt).clone().requires_grad_(True)
        gy = gy0.to(dt).clone().requires_grad_(True)
        (gx,) = torch.autograd.grad(fn(x, a), x, gy, create_graph=True)
        return torch.autograd.grad((gx.to(u.dtype) * u).sum(), (x, a, gy))

    for f, r in zip(hvp(add_rms_norm, torch.float32), hvp(lambda x, a: rms_norm(x + a), torch.float32)):
        assert float((f - r).abs().max() / r.abs().max()) < 1e-4
    for f, r in zip(hvp(add_rms_norm, torch.bfloat16), hvp(lambda x, a: rms_norm(x + a), torch.float64)):
        err = float((f.double() - r).abs().max() / r.abs().max())
        assert err < 2e-2, err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_swiglu_forward_backward_and_second_order(dtype):
    from ebr_b200.layers import swiglu_act

    g = torch.Generator(device="cpu").manual_seed(9)
    h = (torch.randn(5, 81, 2 * 1536, generator=g) * 2).to(DEV, dtype)
    go = torch.randn(5, 81, 1536, generator=g).to(DEV, dtype)
    eager = lambda t: F.silu(t.chunk(2, -1)[0]) * t.chunk(2, -1)[1]
    _check_rounding(swiglu_act(h), eager(h))
    hf, he = h.clone().requires_grad_(True), h.clone().requires_grad_(True)
    (gf,) = torch.autograd.grad(swiglu_act(hf), hf, go)
    (ge,) = torch.autograd.grad(eager(he), he, go)
    assert float((gf.double() - ge.double()).abs().max() / ge.double().abs().max()) < 1e-2
    # create_graph: the second derivatives (closed form, ebr_swiglu_bwd2) with respect to h and to the upstream
    # gradient equal the eager ops'
    u = torch.randn_like(h)
    out = []
    for fn in (swiglu_act, eager):
        t = h.float().clone().requires_grad_(True)
        gof = go.float().clone().requires_grad_(True)
        (gt,) = torch.autograd.grad(fn(t), t, gof, create_graph=True)
        out.append(torch.autograd.grad((gt * u.float()).sum(), (t, gof)))
    for a, b in zip(*out):
        assert float((a - b).abs().max() / b.abs().max()) < 1e-5


def test_descent_point_and_step_match_eager():
    from ebr_b200.layers import noisy_point, step_and_project
    from oracle.energy import rms_norm, sphere

    g = torch.Generator(device="cpu").manual_seed(10)
    z = torch.randn(6, 900, 512, generator=g).to(DEV, torch.bfloat16)
    noise = torch.randn(6, 900, 512, generator=g).to(DEV, torch.bfloat16)
    ulps, frac = _ulp_diff(noisy_point(z, noise, 0.05), rms_norm(z) + noise * 0.05)
    assert ulps <= 1.0 and frac < 0.02, (ulps, frac)
    ulps, frac = _ulp_diff(noisy_point(z, None, 0.0), rms_norm(z))
    assert ulps <= 1.0 and frac < 0.02, (ulps, frac)
    v = rms_norm(z)
    grad = torch.randn(6, 900, 512, generator=g).to(DEV, torch.bfloat16) * 1e-3
    ulps, frac = _ulp_diff(step_and_project(v, grad, 250.0), sphere(v - 250.0 * grad))
    assert ulps <= 1.0 and frac < 0.02, (ulps, frac)


def _network_pair(rows: int, seed: int):
    """The benchmark network on a 9 x 9 board (fused layers, sm_100a attention), its weights under the reference's
    names, and the oracle's eager restatement bound to a given attention."""
    from ebr_b200.energy import LatentEnergyNet, NetShape

    shape = NetShape(board=(9, 9), vocab=10)
    gen = torch.Generator(device=DEV).manual_seed(seed)
    net = LatentEnergyNet(shape).to(DEV)
    net.reset_parameters(gen)
    with torch.no_grad():
        for blk in net.blocks:
            blk.log_temp.copy_(torch.randn(blk.log_temp.shape, generator=gen, device=DEV) * 0.2)
    spec = {"board": (9, 9), "hidden": 512, "heads": 8, "layers": 4, "softplus": False}
    tok = torch.randint(0, 10, (rows, 81), generator=gen, device=DEV)
    return net, net.reference_state(), spec, tok, gen


def _fused_attention(q, k, v):
    from ebr_b200.fused_attn import fused_attention

    return fused_attention(q, k, v)


def test_energy_network_fused_layers_within_noise_floor():
    """dE/dz and one inference microstep of the benchmark network with fused layers vs the oracle's eager layers (same
    sm_100a attention): within 1.25x the deviation that fp32 -> fp64 inside the attention causes, plus 2e-3."""
    from ebr_b200.energy import cell_unit_rms
    from oracle import energy as oe

    net, state, spec, tok, gen = _network_pair(32, 1)
    x = net.embed(tok)
    z = net.fresh_states(32, gen)
    v = cell_unit_rms(z)
    gf = net.energy_and_grad(v, x)[1]
    ge, g32, g64 = (oe.energy_and_grad(state, spec, v, x, att)[1]
                    for att in (_fused_attention, oe.math_attention, oe.math_attention64))  # fmt: skip
    rel = lambda a, r: float((a.float() - r.float()).norm() / r.float().norm())
    floor = rel(g32, g64)
    assert rel(gf, ge) <= 1.25 * floor + 2e-3, (rel(gf, ge), floor)
    zf, _ = net.microstep(z, x, sigma=0.0)
    ze, _ = oe.microstep(state, spec, z, x, attention=_fused_attention)
    z32, _ = oe.microstep(state, spec, z, x, attention=oe.math_attention)
    z64, _ = oe.microstep(state, spec, z, x, attention=oe.math_attention64)
    assert rel(zf, ze) <= 1.25 * rel(z32, z64) + 2e-3, (rel(zf, ze), rel(z32, z64))


def test_training_segment_with_fused_layers():
    """One graded microstep (create_graph, so the double backward runs through the fused layers' graph backwards)
    and the decode loss: the parameter gradients of the fused network against the oracle's eager network with the
    same sm_100a attention, within the network's noise floor (the deviation between fp32 and fp64 math attention in
    the eager network, norm-rel, times 1.25, plus 2e-3), or 2e-2."""
    from ebr_b200.energy import board_unit_rms, cell_unit_rms, stablemax_cross_entropy
    from oracle import energy as oe

    net, state, spec, tok, gen = _network_pair(8, 2)
    labels = torch.randint(0, 10, (8, 81), generator=gen, device=DEV)
    z = net.fresh_states(8, gen)
    names = list(state)

    def eager_grads(attention):
        st = {n: t.clone().requires_grad_(True) for n, t in state.items()}
        x = oe.embed(st, spec, tok, torch.bfloat16)
        v = cell_unit_rms(z).detach().requires_grad_(True)
        _, g = oe.energy_and_grad(st, spec, v, x, attention, create_graph=True)
        z1 = board_unit_rms(v - 250.0 * g)
        logits = torch.nn.functional.linear(z1, st["lm_head.weight"].to(z1.dtype))
        loss = stablemax_cross_entropy(logits, labels).mean()
        return torch.autograd.grad(loss, [st[n] for n in names], allow_unused=True)

    x = net.embed(tok)
    z1, _ = net.microstep(z, x, graded=True, sigma=0.0)
    loss = stablemax_cross_entropy(net.decode(z1), labels).mean()
    own = dict(net.named_parameters())
    inv = {ref: mine for mine, ref in net._name_map().items()}
    ours = torch.autograd.grad(loss, [own[inv[n]] for n in names], allow_unused=True)
    eager, m32, m64 = (eager_grads(a) for a in (_fused_attention, oe.math_attention, oe.math_attention64))

    def rel(ga, gb):
        num = den = 0.0
        for a, b in zip(ga, gb):
            if a is None or b is None:
                assert a is None and b is None
                continue
            assert torch.isfinite(a).all()
            num += float((a.double() - b.double()).square().sum())
            den += float(b.double().square().sum())
        return (num / den) ** 0.5

    got, floor = rel(ours, eager), rel(m32, m64)
    assert got <= max(2e-2, 1.25 * floor + 2e-3), (got, floor)


def test_silu_rounding_is_exact_for_every_bfloat16_gate():
    """Every finite bfloat16 gate value through the three kernels that round silu(g): the activation, its backward (du
    with gout = up = 1) and the gate / up GEMM's epilogue (identity weights, so h reproduces the gates exactly). Each
    must equal round(g / (1 + exp(-g))) taken in fp32 by torch on the same device, bit for bit."""
    from ebr_b200.layers import gate_up_swiglu_op, swiglu_act, swiglu_bwd

    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16)
    g = bits.view(torch.bfloat16).to(DEV)
    g = g[torch.isfinite(g)]
    i = 128
    rows = (g.numel() + i - 1) // i
    g = torch.cat([g, g.new_zeros(rows * i - g.numel())]).view(rows, i)
    g32 = g.float()
    ref = (g32 / (1 + torch.exp(-g32))).to(torch.bfloat16)
    h = torch.cat([g, torch.ones_like(g)], dim=1)
    with torch.no_grad():
        assert torch.equal(swiglu_act(h), ref)
        assert torch.equal(swiglu_bwd(h, torch.ones_like(g))[:, i:], ref)
        x = torch.zeros(rows, 256, device=DEV, dtype=torch.bfloat16)
        x[:, :i] = g
        x[:, i] = 1
        w = torch.zeros(2 * i, 256, device=DEV, dtype=torch.bfloat16)
        w[torch.arange(i), torch.arange(i)] = 1
        w[i:, i] = 1
        hh, act = gate_up_swiglu_op(x, w)
        assert torch.equal(hh, h)
        assert torch.equal(act, ref)
