"""The allocation-free backward entry point, ``ebr_attn_bwd_noalloc``, through the C ABI.

It serves callers that cannot allocate device memory when they call the backward (a host whose GPU memory is planned
up front by another allocator, or a plugin host that gives the plugin only its inputs and outputs). It runs the same
kernels as ``ebr_attn_bwd`` with the row scratch in a built-in device array, so its outputs must match
``ebr_attn_bwd``'s, within the gradient tolerance of the parity tests (1e-2 max-rel), on two calls in a row with
different inputs (the array keeps the previous call's contents). Also checks that a call larger than the built-in
array is refused before any launch.

This file sorts last so that a run stopping at the first failure has run every other test first; it does not depend
on state left by other tests and passes when run alone.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GRAD_TOL = 1e-2


def _maxrel(a: torch.Tensor, r: torch.Tensor) -> float:
    a, r = a.double().cpu(), r.double().cpu()
    return float((a - r).abs().max() / r.abs().max().clamp_min(1e-3))


def _call(lib, fn_name, dtype_code, q, k, v, o, lse, do, scratch=None):
    from ebr_b200 import _native

    B, H, N, D = q.shape
    outs = [torch.empty_like(q) for _ in range(3)]
    op = lambda t: _native.Operand(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))
    ops = [op(t) for t in (q, k, v, do)]
    r = ctypes.byref
    stream = torch.cuda.current_stream().cuda_stream
    common = (dtype_code, B, H, N, D, D**-0.5, r(ops[0]), r(ops[1]), r(ops[2]), o.data_ptr(), lse.data_ptr(),
              r(ops[3]), *[t.data_ptr() for t in outs])  # fmt: skip
    if fn_name == "ebr_attn_bwd":
        st = lib.ebr_attn_bwd(*common, scratch.data_ptr(), scratch.numel(), stream)
    else:
        st = lib.ebr_attn_bwd_noalloc(*common, stream)
    assert st == 0, lib.ebr_attn_last_error()
    return outs


@pytest.mark.parametrize("dtype,shape", [
    (torch.bfloat16, (2, 4, 300, 64)),   # tiled tensor-core backward: row pass writes D_i to the scratch
    (torch.float32, (1, 3, 81, 64)),     # CUDA-core backward: same row-scalar scratch
])  # fmt: skip
def test_noalloc_matches_bwd_on_two_calls(dtype, shape):
    from ebr_b200 import _native
    from ebr_b200.build import build

    build()
    lib = _native.lib()
    code = {torch.bfloat16: _native.BFLOAT16, torch.float32: _native.FLOAT32}[dtype]
    B, H, N, D = shape
    for call in range(2):
        g = torch.Generator().manual_seed(100 + call)
        mk = lambda s: (torch.randn(shape, generator=g) * s).to(dtype).cuda()
        q, k, v, do = mk(0.5), mk(0.5), mk(0.5), mk(1.0)
        o, lse = torch.ops.ebr_fused.attn_fwd(q, k, v, D**-0.5)
        scratch = torch.empty(lib.ebr_attn_bwd_scratch_bytes(code, B, H, N, D), dtype=torch.uint8, device="cuda")
        ref = _call(lib, "ebr_attn_bwd", code, q, k, v, o, lse, do, scratch)
        got = _call(lib, "ebr_attn_bwd_noalloc", code, q, k, v, o, lse, do)
        torch.cuda.synchronize()
        _native.device_status()
        for a, b in zip(got, ref):
            assert torch.isfinite(a.float()).all()
            assert _maxrel(a, b) <= GRAD_TOL


def test_noalloc_refuses_calls_larger_than_its_buffer():
    from ebr_b200 import _native
    from ebr_b200.build import build

    build()
    lib = _native.lib()
    cap = 8 << 20
    B, H, N, D = 1, 8, cap // 4 // 8 + 1, 64  # one row past the float32 limit
    fake = _native.Operand(0x1000, 0, 0, 64)
    r = ctypes.byref
    st = lib.ebr_attn_bwd_noalloc(_native.BFLOAT16, B, H, N, D, 0.125, r(fake), r(fake), r(fake), 0x2000, 0x3000,
                                  r(fake), 0x4000, 0x5000, 0x6000, None)  # fmt: skip
    assert st == _native.ERR_SCRATCH
    assert b"built-in buffer" in lib.ebr_attn_last_error()
    assert np.int64(B * H * (N - 1)) * 4 <= cap
