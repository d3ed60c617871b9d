"""Fused second-order attention on B200: the drop-in for the reference's ``models.fused_attn``.

Same public surface as the reference (``models/fused_attn/ops.py``):

* three ``torch.library`` custom ops with the reference's schemas (``ops.py:65-120``) —
  ``ebr_fused::attn_fwd(q, k, v, scale) -> (o, lse)``,
  ``ebr_fused::attn_bwd(q, k, v, o, lse, do, scale) -> (dq, dk, dv)``,
  ``ebr_fused::attn_bwd_bwd(q, k, v, o, lse, do, dq, gq, gk, gv, scale) -> (hq, hk, hv, hdo)`` —
  each with a fake (meta) kernel so ``torch.compile`` / ``torch.func.grad`` trace them as opaque nodes;
* the two ``autograd.Function`` classes chaining fwd -> bwd -> bwd_bwd with ``setup_context`` (``ops.py:131-175``),
  so ``create_graph=True`` works through both levels;
* ``fused_attention(q, k, v, scale=None)`` on ``[B, H, N, D]`` (``ops.py:188-190``), wrapped with
  ``torch._dynamo.allow_in_graph`` (``ops.py:183-185``).

The ops run the sm_100a kernels of ``libebr_attn.so`` through its C ABI on the current CUDA stream. There is no CPU
or Triton implementation: a non-CUDA tensor is an error.
"""

# No ``from __future__ import annotations``: custom_op schema inference needs real type objects.
import ctypes
from typing import Optional, Tuple

import torch

from ebr_b200 import _native

Tensor = torch.Tensor

_DTYPES = {
    torch.float32: _native.FLOAT32,
    torch.float16: _native.FLOAT16,
    torch.bfloat16: _native.BFLOAT16,
    torch.float64: _native.FLOAT64,
}


def lse_dtype_for(x: Tensor) -> torch.dtype:
    """``lse`` is float32, float64 for float64 inputs (the reference's ``reference.lse_dtype_for``)."""
    return torch.float64 if x.dtype == torch.float64 else torch.float32


def default_scale(q: Tensor, scale: Optional[float]) -> float:
    return float(q.shape[-1] ** -0.5) if scale is None else float(scale)


def implementation(device="cuda") -> str:
    """What the ops run on ``device``: ``"sm100"`` on CUDA; anything else is unsupported (the ops raise)."""
    return "sm100" if torch.device(device).type == "cuda" else "unsupported"


def _check(q: Tensor, k: Tensor, v: Tensor) -> None:
    """Same-shape [B, H, N, D] and one dtype, else ValueError (the reference's ``_check``, ops.py:51-57)."""
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(
            f"fused attention expects q, k, v of identical shape [B, H, N, D]; got {q.shape}, {k.shape}, {v.shape}"
        )
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError(f"fused attention expects one dtype; got {q.dtype}, {k.dtype}, {v.dtype}")


def _require_cuda(q: Tensor) -> None:
    if not q.is_cuda:
        raise RuntimeError(
            f"ebr_b200 fused attention runs only on CUDA (sm_100a) tensors, got device {q.device}; there is no CPU path"
        )
    if q.dtype not in _DTYPES:
        raise TypeError(f"fused attention: unsupported dtype {q.dtype}")


def _d1(t: Tensor) -> Tensor:
    """Any batch / head / token strides are taken as they are; only the head dim must be unit-stride."""
    return t if (t.stride(-1) == 1 or t.shape[-1] == 1) else t.contiguous()


def _operand(t: Optional[Tensor]) -> Optional[_native.Operand]:
    if t is None:
        return None
    return _native.Operand(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _ref(op: Optional[_native.Operand]):
    return None if op is None else ctypes.byref(op)


def _stream(t: Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


class KernelTimer:
    """CUDA-event timing of every native attention call made while it is active (``with kernel_timer() as t``).

    Events are recorded on the stream each call launches on, around the C ABI call, so one record covers all the
    kernels of that op (the tiled backward is two launches). ``summary()`` synchronizes and returns, per op, the call
    count and total milliseconds.
    """

    def __init__(self) -> None:
        self.records: list[tuple[str, tuple, torch.cuda.Event, torch.cuda.Event]] = []

    def summary(self) -> dict:
        torch.cuda.synchronize()
        out: dict = {}
        for name, shape, a, b in self.records:
            d = out.setdefault(name, {"calls": 0, "ms": 0.0, "shape": shape})
            d["calls"] += 1
            d["ms"] += a.elapsed_time(b)
        return out


_TIMER: Optional[KernelTimer] = None


class kernel_timer:
    def __enter__(self) -> KernelTimer:
        global _TIMER
        self.prev, _TIMER = _TIMER, KernelTimer()
        return _TIMER

    def __exit__(self, *exc) -> None:
        global _TIMER
        _TIMER = self.prev


class _Timed:
    def __init__(self, name: str, q: Tensor) -> None:
        self.name, self.q = name, q

    def __enter__(self):
        if _TIMER is not None:
            self.a = torch.cuda.Event(enable_timing=True)
            self.b = torch.cuda.Event(enable_timing=True)
            self.a.record()

    def __exit__(self, *exc):
        if _TIMER is not None:
            self.b.record()
            _TIMER.records.append((self.name, tuple(self.q.shape), self.a, self.b))


class _OnDevice:
    """Make ``t``'s device current for the native call (the C ABI launches on the current device)."""

    def __init__(self, t: Tensor) -> None:
        self.index = t.device.index
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if self.index is not None and cur != self.index:
            self.prev = cur
            torch.cuda.set_device(self.index)

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)


# ----------------------------------------------------------------------------------------------------------------------
# Ops
# ----------------------------------------------------------------------------------------------------------------------


@torch.library.custom_op("ebr_fused::attn_fwd", mutates_args=())
def attn_fwd(q: Tensor, k: Tensor, v: Tensor, scale: float) -> Tuple[Tensor, Tensor]:
    _check(q, k, v)
    _require_cuda(q)
    q, k, v = _d1(q), _d1(k), _d1(v)
    B, H, N, D = q.shape
    o = torch.empty((B, H, N, D), device=q.device, dtype=q.dtype)
    lse = torch.empty((B, H, N), device=q.device, dtype=lse_dtype_for(q))
    oq, ok, ov = _operand(q), _operand(k), _operand(v)
    with _OnDevice(q), _Timed("attn_fwd", q):
        _native.check(
            _native.lib().ebr_attn_fwd(
                _DTYPES[q.dtype], B, H, N, D, float(scale), _ref(oq), _ref(ok), _ref(ov),
                o.data_ptr(), lse.data_ptr(), _stream(q),
            ),
            "ebr_attn_fwd",
        )  # fmt: skip
    return o, lse


@attn_fwd.register_fake
def _(q: Tensor, k: Tensor, v: Tensor, scale: float) -> Tuple[Tensor, Tensor]:
    o = torch.empty_like(q, memory_format=torch.contiguous_format)
    lse = q.new_empty(q.shape[:-1], dtype=lse_dtype_for(q))
    return o, lse


@torch.library.custom_op("ebr_fused::attn_bwd", mutates_args=())
def attn_bwd(
    q: Tensor, k: Tensor, v: Tensor, o: Tensor, lse: Tensor, do: Tensor, scale: float
) -> Tuple[Tensor, Tensor, Tensor]:
    _check(q, k, v)
    _require_cuda(q)
    do = _d1(do.to(q.dtype))
    q, k, v = _d1(q), _d1(k), _d1(v)
    o, lse = o.contiguous(), lse.contiguous()
    B, H, N, D = q.shape
    dq, dk, dv = (torch.empty((B, H, N, D), device=q.device, dtype=q.dtype) for _ in range(3))
    dt = _DTYPES[q.dtype]
    lib = _native.lib()
    nbytes = lib.ebr_attn_bwd_scratch_bytes(dt, B, H, N, D)
    scratch = torch.empty((max(nbytes, 1),), device=q.device, dtype=torch.uint8)
    oq, ok, ov, odo = _operand(q), _operand(k), _operand(v), _operand(do)
    with _OnDevice(q), _Timed("attn_bwd", q):
        _native.check(
            lib.ebr_attn_bwd(
                dt, B, H, N, D, float(scale), _ref(oq), _ref(ok), _ref(ov), o.data_ptr(), lse.data_ptr(), _ref(odo),
                dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), scratch.data_ptr(), nbytes, _stream(q),
            ),
            "ebr_attn_bwd",
        )  # fmt: skip
    return dq, dk, dv


@attn_bwd.register_fake
def _(
    q: Tensor, k: Tensor, v: Tensor, o: Tensor, lse: Tensor, do: Tensor, scale: float
) -> Tuple[Tensor, Tensor, Tensor]:
    f = lambda x: torch.empty_like(x, memory_format=torch.contiguous_format)
    return f(q), f(k), f(v)


@torch.library.custom_op("ebr_fused::attn_bwd_bwd", mutates_args=())
def attn_bwd_bwd(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    o: Tensor,
    lse: Tensor,
    do: Tensor,
    dq: Tensor,
    gq: Tensor,
    gk: Tensor,
    gv: Tensor,
    scale: float,
) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    _check(q, k, v)
    _require_cuda(q)
    q, k, v, do = _d1(q), _d1(k), _d1(v), _d1(do.to(q.dtype))
    gq, gk, gv = (_d1(g.to(q.dtype)) for g in (gq, gk, gv))
    o, lse = o.contiguous(), lse.contiguous()
    B, H, N, D = q.shape
    hq, hk, hv, hdo = (torch.empty((B, H, N, D), device=q.device, dtype=q.dtype) for _ in range(4))
    dt = _DTYPES[q.dtype]
    lib = _native.lib()
    nbytes = lib.ebr_attn_bwd_bwd_scratch_bytes(dt, B, H, N, D)
    scratch = torch.empty((max(nbytes, 1),), device=q.device, dtype=torch.uint8)
    ops = [_operand(t) for t in (q, k, v, do, gq, gk, gv)]
    with _OnDevice(q), _Timed("attn_bwd_bwd", q):
        _native.check(
            lib.ebr_attn_bwd_bwd(
                dt, B, H, N, D, float(scale), _ref(ops[0]), _ref(ops[1]), _ref(ops[2]), o.data_ptr(), lse.data_ptr(),
                _ref(ops[3]), dq.data_ptr(), _ref(ops[4]), _ref(ops[5]), _ref(ops[6]),
                hq.data_ptr(), hk.data_ptr(), hv.data_ptr(), hdo.data_ptr(), scratch.data_ptr(), nbytes, _stream(q),
            ),
            "ebr_attn_bwd_bwd",
        )  # fmt: skip
    return hq, hk, hv, hdo


@attn_bwd_bwd.register_fake
def _(q, k, v, o, lse, do, dq, gq, gk, gv, scale):
    f = lambda x: torch.empty_like(x, memory_format=torch.contiguous_format)
    return f(q), f(k), f(v), f(do)


# ----------------------------------------------------------------------------------------------------------------------
# Autograd: fwd -> bwd -> bwd_bwd
# ----------------------------------------------------------------------------------------------------------------------
#
# autograd.Functions with setup_context (torch.func.grad, used by the compiled dE/dz, needs them); the raw ops carry no
# autograd formula, so only fused_attention is differentiable (the reference's design, ops.py:123-128).


class _FusedAttnBwd(torch.autograd.Function):
    """(q, k, v, o, lse, do) -> (dq, dk, dv); its backward is attn_bwd_bwd, the total derivative through O."""

    @staticmethod
    def forward(q, k, v, o, lse, do, scale):
        return torch.ops.ebr_fused.attn_bwd(q, k, v, o, lse, do, scale)

    @staticmethod
    def setup_context(ctx, inputs, output):
        q, k, v, o, lse, do, scale = inputs
        ctx.save_for_backward(q, k, v, o, lse, do, output[0])
        ctx.scale = scale

    @staticmethod
    def backward(ctx, gq, gk, gv):
        q, k, v, o, lse, do, dq = ctx.saved_tensors
        gq = torch.zeros_like(q) if gq is None else gq.to(q.dtype)
        gk = torch.zeros_like(k) if gk is None else gk.to(k.dtype)
        gv = torch.zeros_like(v) if gv is None else gv.to(v.dtype)
        hq, hk, hv, hdo = torch.ops.ebr_fused.attn_bwd_bwd(q, k, v, o, lse, do, dq, gq, gk, gv, ctx.scale)
        return hq, hk, hv, None, None, hdo, None


class _FusedAttn(torch.autograd.Function):
    """(q, k, v) -> o; its backward is _FusedAttnBwd, itself differentiable."""

    @staticmethod
    def forward(q, k, v, scale):
        o, lse = torch.ops.ebr_fused.attn_fwd(q, k, v, scale)
        return o, lse

    @staticmethod
    def setup_context(ctx, inputs, output):
        q, k, v, scale = inputs
        o, lse = output
        ctx.mark_non_differentiable(lse)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale = scale

    @staticmethod
    def backward(ctx, do, dlse):
        del dlse  # lse is non-differentiable
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = _FusedAttnBwd.apply(q, k, v, o, lse, do, ctx.scale)
        return dq, dk, dv, None


def _fused_attention_apply(q: Tensor, k: Tensor, v: Tensor, scale: float) -> Tensor:
    o, _ = _FusedAttn.apply(q, k, v, scale)
    return o


# One opaque node for dynamo; AOTAutograd then traces the Functions above into the three custom ops.
_fused_attention_apply = torch._dynamo.allow_in_graph(_fused_attention_apply)


def fused_attention(q: Tensor, k: Tensor, v: Tensor, scale: Optional[float] = None) -> Tensor:
    """Non-causal softmax attention, ``[B, H, N, D]`` in and out, differentiable to second order."""
    return _fused_attention_apply(q, k, v, default_scale(q, scale))


def uses_tensor_cores(q: Tensor, k: Tensor, v: Tensor) -> bool:
    """Whether calls with these operands take the tcgen05 kernels (16-bit, D in {64, 128}, TMA-compatible strides)."""
    ops = [_operand(_d1(t)) for t in (q, k, v)]
    return bool(_native.lib().ebr_attn_uses_tensor_cores(_DTYPES[q.dtype], q.shape[-1], *map(_ref, ops)))


__all__ = [
    "KernelTimer",
    "kernel_timer",
    "attn_bwd",
    "attn_bwd_bwd",
    "attn_fwd",
    "default_scale",
    "fused_attention",
    "implementation",
    "lse_dtype_for",
    "uses_tensor_cores",
]
