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
