"""Host-side contract of the fused-attention ops that needs no GPU: schemas, fake kernels, argument checks, and the
absence of any CPU fallback."""

from __future__ import annotations

import pytest
import torch

from ebr_b200 import fused_attn


def test_schemas_match_the_reference():
    # models/fused_attn/ops.py:65-114
    s = {n: str(getattr(torch.ops.ebr_fused, n).default._schema) for n in ("attn_fwd", "attn_bwd", "attn_bwd_bwd")}
    assert s["attn_fwd"] == "ebr_fused::attn_fwd(Tensor q, Tensor k, Tensor v, float scale) -> (Tensor, Tensor)"
    assert s["attn_bwd"] == (
        "ebr_fused::attn_bwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, Tensor do, float scale) "
        "-> (Tensor, Tensor, Tensor)"
    )
    assert s["attn_bwd_bwd"] == (
        "ebr_fused::attn_bwd_bwd(Tensor q, Tensor k, Tensor v, Tensor o, Tensor lse, Tensor do, Tensor dq, "
        "Tensor gq, Tensor gk, Tensor gv, float scale) -> (Tensor, Tensor, Tensor, Tensor)"
    )


def test_fake_kernels_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty(2, 3, 81, 64, dtype=torch.bfloat16).transpose(1, 2).transpose(1, 2)
        o, lse = torch.ops.ebr_fused.attn_fwd(q, q, q, 0.125)
        assert o.shape == q.shape and o.is_contiguous() and lse.shape == (2, 3, 81) and lse.dtype == torch.float32
        dq, dk, dv = torch.ops.ebr_fused.attn_bwd(q, q, q, o, lse, q, 0.125)
        assert dq.shape == q.shape and dv.dtype == torch.bfloat16
        hs = torch.ops.ebr_fused.attn_bwd_bwd(q, q, q, o, lse, q, dq, q, q, q, 0.125)
        assert len(hs) == 4 and all(h.shape == q.shape for h in hs)
        q64 = torch.empty(1, 1, 5, 16, dtype=torch.float64)
        _, lse64 = torch.ops.ebr_fused.attn_fwd(q64, q64, q64, 0.25)
        assert lse64.dtype == torch.float64


def test_shape_and_dtype_checks():
    q = torch.zeros(1, 2, 8, 16)
    with pytest.raises(ValueError):
        fused_attn.attn_fwd(q, q[:, :, :4], q, 0.25)
    with pytest.raises(ValueError):
        fused_attn.attn_fwd(q, q.double(), q, 0.25)
    with pytest.raises(ValueError):
        fused_attn.attn_fwd(q[0], q[0], q[0], 0.25)


def test_no_cpu_fallback():
    q = torch.randn(1, 2, 8, 16)
    with pytest.raises(RuntimeError, match="only on CUDA"):
        fused_attn.fused_attention(q, q, q)
    with pytest.raises(RuntimeError, match="only on CUDA"):
        torch.ops.ebr_fused.attn_bwd(q, q, q, q, q[..., 0], q, 0.25)
    assert fused_attn.implementation("cpu") == "unsupported"
    assert fused_attn.implementation("cuda") == "sm100"


def test_default_scale():
    q = torch.zeros(1, 1, 1, 64)
    assert fused_attn.default_scale(q, None) == 0.125
    assert fused_attn.default_scale(q, 0.3) == 0.3


def test_projection_ops_fake_kernels_and_no_cpu_path():
    """The fused projections' fake kernels give the shapes the CUDA ops return (torch.compile traces through them), the
    ops refuse CPU tensors, and the Python wrappers' kernel checks turn CPU inputs away (no CPU fallback is taken)."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    from ebr_b200 import layers

    with FakeTensorMode():
        x = torch.empty(2, 81, 512, dtype=torch.bfloat16)
        w_qkv = torch.empty(1536, 512, dtype=torch.bfloat16)
        tab = torch.empty(81, 64)
        q, k, v = torch.ops.ebr_fused.qkv_rope_split(x, w_qkv, tab, tab, torch.empty(0), 8)
        assert q.shape == k.shape == v.shape == (2, 8, 81, 64) and q.dtype == torch.bfloat16
        o = torch.empty(2, 8, 81, 64, dtype=torch.bfloat16)
        y = torch.ops.ebr_fused.o_proj(o, torch.empty(512, 512, dtype=torch.bfloat16))
        assert y.shape == (2, 81, 512)
        h, act = torch.ops.ebr_fused.gate_up_swiglu(x, torch.empty(3072, 512, dtype=torch.bfloat16))
        assert h.shape == (2, 81, 3072) and act.shape == (2, 81, 1536)
    x = torch.zeros(1, 4, 512, dtype=torch.bfloat16)
    w = torch.zeros(1536, 512, dtype=torch.bfloat16)
    assert not layers.qkv_fusable(x, w, 8)
    assert not layers.gate_up_fusable(x, torch.zeros(3072, 512, dtype=torch.bfloat16))
    o = torch.zeros(1, 8, 4, 64, dtype=torch.bfloat16)
    assert not layers.o_proj_fusable(o, torch.zeros(512, 512, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="only on CUDA"):
        torch.ops.ebr_fused.qkv_rope_split(x, w, torch.zeros(4, 64), torch.zeros(4, 64), torch.zeros(0), 8)
    with pytest.raises(RuntimeError, match="only on CUDA"):
        torch.ops.ebr_fused.gate_up_swiglu(x, torch.zeros(3072, 512, dtype=torch.bfloat16))
