"""Fused kernels on either side of the attention in the energy network (``include/ebr_layers.h``).

* 2D-RoPE split / merge: the reference's ``rope_impl: fused`` path (``models/fused_attn/rope_split.py``): custom ops
  ``ebr_fused::rope_split(qkv, cos, sin, qscale, heads) -> (q, k, v)`` and
  ``ebr_fused::rope_merge(dq, dk, dv, cos, sin, qscale) -> dqkv`` with the reference's schemas and fake kernels
  (``rope_split.py:75-103``), the two autograd Functions that are each other's adjoint, so every derivative order is
  exact (``:110-150``), and ``rope_split(qkv, cos, sin, heads, qscale=None)`` (``:161-178``). ``rotary_tables`` builds
  the ``[H * W, D]`` cos / sign-folded sin tables of ``RotaryTable2D`` (``models/layers.py:143-172``).
* ``add_rms_norm(x, a)``: rms_norm(x + a) of the post-norm block (``models/layers.py:37-42``), one kernel forward and
  one backward.
* ``swiglu_act(h)``: ``silu(gate) * up`` of ``SwiGLU`` (``models/layers.py:82-84``), one kernel each way.
* ``noisy_point`` / ``step_and_project``: the pointwise ops of an inference microstep, ``v = rms_norm(z) + noise``
  and ``z' = sphere(v - alpha g)`` (``models/energy.py:219-241``), one and two kernels.

The row kernels' backwards run the fused kernel when no higher-order graph is being built; under ``create_graph``
(graded microsteps) they evaluate the same formula with differentiable torch ops, so the double backward of training
differentiates through them. Every op is CUDA-only: a CPU tensor is an error (the CPU model uses the eager layers).
"""

# No ``from __future__ import annotations``: custom_op schema inference needs real type objects.
import ctypes
from typing import Optional, Tuple

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable
from torch.autograd.graph import get_gradient_edge

from ebr_b200 import _native

Tensor = torch.Tensor

_DTYPES = {
    torch.float32: _native.FLOAT32,
    torch.float16: _native.FLOAT16,
    torch.bfloat16: _native.BFLOAT16,
    torch.float64: _native.FLOAT64,
}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(t: Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what} runs only on CUDA (sm_100a) tensors, got device {t.device}; there is no CPU path")
    if t.dtype not in _DTYPES:
        raise TypeError(f"{what}: unsupported dtype {t.dtype}")


def _ptr(t: Optional[Tensor]):
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------------------------------------------- 2D RoPE


def quarter_swap(x: Tensor) -> Tensor:
    """``(a, b, c, d) -> (b, a, d, c)`` over the quarters of the last dim (rotate_half of each half, without sign)."""
    shape = x.shape
    return x.reshape(*shape[:-1], 2, 2, shape[-1] // 4).flip(-2).reshape(shape)


def rotary_tables(cos_h: Tensor, sin_h: Tensor, cos_w: Tensor, sin_w: Tensor) -> Tuple[Tensor, Tensor]:
    """``[H * W, D]`` float32 tables from the per-row / per-column ``[H, D/2]`` / ``[W, D/2]`` RoPE tables: cell
    ``i * W + j`` has row ``i``'s angles in the first half of D and column ``j``'s in the second, and the sign of
    rotate_half is folded into sin, so ``t' = t * cos + quarter_swap(t) * sin`` (``models/layers.py:143-172``)."""
    height, width, half = cos_h.shape[0], cos_w.shape[0], cos_h.shape[1]
    dim = 2 * half
    rows = torch.arange(height, device=cos_h.device).repeat_interleave(width)
    cols = torch.arange(width, device=cos_h.device).repeat(height)
    cos = torch.cat((cos_h[rows], cos_w[cols]), dim=-1)
    sin = torch.cat((sin_h[rows], sin_w[cols]), dim=-1)
    sign = torch.ones(dim, device=cos_h.device)
    sign[: dim // 4] = -1.0
    sign[dim // 2 : dim // 2 + dim // 4] = -1.0
    return cos.to(torch.float32).contiguous(), (sin * sign).to(torch.float32).contiguous()


def _qscale_arg(qscale: Tensor):
    if qscale is None or qscale.numel() == 0:
        return None, None
    qs = qscale.detach().to(torch.float32).contiguous()
    return qs, qs.data_ptr()


def _table(t: Tensor, dev) -> Tensor:
    return t.to(device=dev, dtype=torch.float32).contiguous()


@torch.library.custom_op("ebr_fused::rope_split", mutates_args=())
def rope_split_op(qkv: Tensor, cos: Tensor, sin: Tensor, qscale: Tensor, heads: int) -> Tuple[Tensor, Tensor, Tensor]:
    _require_cuda(qkv, "rope_split")
    b, n, c3 = qkv.shape
    d = c3 // (3 * heads)
    if qkv.stride(-1) != 1:
        qkv = qkv.contiguous()
    q, k, v = (torch.empty((b, heads, n, d), device=qkv.device, dtype=qkv.dtype) for _ in range(3))
    cos, sin = _table(cos, qkv.device), _table(sin, qkv.device)
    qs, qs_ptr = _qscale_arg(qscale)
    _native.check(
        _native.lib().ebr_rope_split(_DTYPES[qkv.dtype], b, n, heads, d, qkv.data_ptr(), qkv.stride(0), qkv.stride(1),
                                     cos.data_ptr(), sin.data_ptr(), qs_ptr, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                     _stream()),  # fmt: skip
        "rope_split",
    )
    return q, k, v


@rope_split_op.register_fake
def _(qkv, cos, sin, qscale, heads):
    b, n, c3 = qkv.shape
    d = c3 // (3 * heads)
    return tuple(qkv.new_empty((b, heads, n, d)) for _ in range(3))


@torch.library.custom_op("ebr_fused::rope_merge", mutates_args=())
def rope_merge_op(dq: Tensor, dk: Tensor, dv: Tensor, cos: Tensor, sin: Tensor, qscale: Tensor) -> Tensor:
    _require_cuda(dq, "rope_merge")
    dk, dv = dk.to(dq.dtype), dv.to(dq.dtype)
    dq, dk, dv = (t if t.stride(-1) == 1 else t.contiguous() for t in (dq, dk, dv))
    b, h, n, d = dq.shape
    out = torch.empty((b, n, 3 * h * d), device=dq.device, dtype=dq.dtype)
    cos, sin = _table(cos, dq.device), _table(sin, dq.device)
    qs, qs_ptr = _qscale_arg(qscale)
    ops = [_native.Operand(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2)) for t in (dq, dk, dv)]
    r = ctypes.byref
    _native.check(
        _native.lib().ebr_rope_merge(_DTYPES[dq.dtype], b, n, h, d, r(ops[0]), r(ops[1]), r(ops[2]), cos.data_ptr(),
                                     sin.data_ptr(), qs_ptr, out.data_ptr(), _stream()),  # fmt: skip
        "rope_merge",
    )
    return out


@rope_merge_op.register_fake
def _(dq, dk, dv, cos, sin, qscale):
    b, h, n, d = dq.shape
    return dq.new_empty((b, n, 3 * h * d))


class _Split(torch.autograd.Function):
    """Forward: the split; backward: the merge (its exact adjoint). ``rope_split.py:110-131``."""

    @staticmethod
    def forward(qkv, cos, sin, qscale, heads):
        return torch.ops.ebr_fused.rope_split(qkv, cos, sin, qscale, heads)

    @staticmethod
    def setup_context(ctx, inputs, output):
        qkv, cos, sin, qscale, heads = inputs
        ctx.save_for_backward(cos, sin, qscale)
        ctx.heads = heads
        ctx.shape = tuple(output[0].shape)

    @staticmethod
    def backward(ctx, gq, gk, gv):
        cos, sin, qscale = ctx.saved_tensors
        ref = next(g for g in (gq, gk, gv) if g is not None)
        z = None
        if gq is None or gk is None or gv is None:
            z = torch.zeros(ctx.shape, dtype=ref.dtype, device=ref.device)
        gq, gk, gv = (z if g is None else g for g in (gq, gk, gv))
        return _Merge.apply(gq, gk, gv, cos, sin, qscale), None, None, None, None


class _Merge(torch.autograd.Function):
    """Forward: the merge; backward: the split. ``rope_split.py:134-150``."""

    @staticmethod
    def forward(dq, dk, dv, cos, sin, qscale):
        return torch.ops.ebr_fused.rope_merge(dq, dk, dv, cos, sin, qscale)

    @staticmethod
    def setup_context(ctx, inputs, output):
        dq, dk, dv, cos, sin, qscale = inputs
        ctx.save_for_backward(cos, sin, qscale)
        ctx.heads = int(dq.shape[1])

    @staticmethod
    def backward(ctx, g):
        cos, sin, qscale = ctx.saved_tensors
        gq, gk, gv = _Split.apply(g, cos, sin, qscale, ctx.heads)
        return gq, gk, gv, None, None, None


def _split(qkv: Tensor, cos: Tensor, sin: Tensor, qscale: Tensor, heads: int):
    return _Split.apply(qkv, cos, sin, qscale, heads)


_split = torch._dynamo.allow_in_graph(_split)


def rope_split(qkv: Tensor, cos: Tensor, sin: Tensor, heads: int,
               qscale: Optional[Tensor] = None) -> Tuple[Tensor, Tensor, Tensor]:  # fmt: skip
    """``[B, N, 3*H*D]`` -> rotated ``q``, ``k`` and ``v``, each ``[B, H, N, D]``; differentiable to every order.

    ``qscale`` (optional, ``[H]``, no gradient): per-head temperature already rounded to the I/O type, folded into q as
    ``round(round(R q) * t)``; the adjoint scales first (``rope_split.py:161-178``)."""
    if qkv.dim() != 3 or qkv.shape[-1] % (3 * heads):
        raise ValueError(f"rope_split expects [B, N, 3*H*D], got {tuple(qkv.shape)} for {heads} heads")
    d = qkv.shape[-1] // (3 * heads)
    if d % 4 or tuple(cos.shape) != (qkv.shape[1], d) or tuple(sin.shape) != (qkv.shape[1], d):
        raise ValueError(f"rope_split: tables must be [N, D] with D % 4 == 0, got {tuple(cos.shape)} (D={d})")
    if qscale is None:
        qscale = qkv.new_zeros((0,), dtype=torch.float32)
    return _split(qkv, cos, sin, qscale.detach(), heads)


# ---------------------------------------------------------------------------------------------------- qkv projection


@torch.library.custom_op("ebr_fused::qkv_rope_split", mutates_args=())
def qkv_rope_split_op(x: Tensor, weight: Tensor, cos: Tensor, sin: Tensor, qscale: Tensor,
                      heads: int) -> Tuple[Tensor, Tensor, Tensor]:  # fmt: skip
    _require_cuda(x, "qkv_rope_split")
    b, n, c = x.shape
    d = weight.shape[0] // (3 * heads)
    x = x.contiguous()
    weight = weight.to(x.dtype).contiguous()
    q, k, v = (torch.empty((b, heads, n, d), device=x.device, dtype=x.dtype) for _ in range(3))
    cos, sin = _table(cos, x.device), _table(sin, x.device)
    qs, qs_ptr = _qscale_arg(qscale)
    _native.check(
        _native.lib().ebr_qkv_rope_split(_DTYPES[x.dtype], b, n, heads, d, c, x.data_ptr(), c, weight.data_ptr(),
                                         cos.data_ptr(), sin.data_ptr(), qs_ptr, q.data_ptr(), k.data_ptr(),
                                         v.data_ptr(), _stream()),  # fmt: skip
        "qkv_rope_split",
    )
    return q, k, v


@qkv_rope_split_op.register_fake
def _(x, weight, cos, sin, qscale, heads):
    b, n, _ = x.shape
    d = weight.shape[0] // (3 * heads)
    return tuple(x.new_empty((b, heads, n, d)) for _ in range(3))


def _engine_needs(node) -> bool:
    """Whether the running backward will execute ``node`` (None: the input needs no gradient). The engine cannot
    answer for a leaf's accumulator under autograd.grad; such an input is assumed needed."""
    if node is None:
        return False
    try:
        return bool(torch._C._will_engine_execute_node(node))
    except RuntimeError:
        return True


@torch.library.custom_op("ebr_fused::qkv_rope_merge_dx", mutates_args=())
def qkv_rope_merge_dx_op(dq: Tensor, dk: Tensor, dv: Tensor, weight: Tensor, cos: Tensor, sin: Tensor,
                         qscale: Tensor, addend: Optional[Tensor] = None) -> Tensor:  # fmt: skip
    """``rope_merge(dq, dk, dv, cos, sin, qscale) @ weight`` (``+ addend``, rounded as a separate add would) as one
    tensor-core GEMM whose A operand is merged in shared memory (``ebr_qkv_rope_merge_dx``): the input gradient of the
    qkv projection, with a residual gradient joined in when given. Shapes ``merge_dx_fusable`` takes."""
    _require_cuda(dq, "qkv_rope_merge_dx")
    dk, dv = dk.to(dq.dtype), dv.to(dq.dtype)
    dq, dk, dv = (t if t.stride(-1) == 1 else t.contiguous() for t in (dq, dk, dv))
    b, h, n, d = dq.shape
    w = weight.to(dq.dtype).contiguous()
    out = torch.empty((b, n, w.shape[1]), device=dq.device, dtype=dq.dtype)
    cos, sin = _table(cos, dq.device), _table(sin, dq.device)
    qs, qs_ptr = _qscale_arg(qscale)
    ops = [_native.Operand(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2)) for t in (dq, dk, dv)]
    add = None if addend is None else addend.to(dq.dtype).reshape(out.shape).contiguous()
    r = ctypes.byref
    _native.check(
        _native.lib().ebr_qkv_rope_merge_dx(_DTYPES[dq.dtype], b, n, h, d, w.shape[1], r(ops[0]), r(ops[1]),
                                            r(ops[2]), w.data_ptr(), cos.data_ptr(), sin.data_ptr(), qs_ptr,
                                            _ptr(add), out.data_ptr(), _stream()),  # fmt: skip
        "qkv_rope_merge_dx",
    )
    return out


@qkv_rope_merge_dx_op.register_fake
def _(dq, dk, dv, weight, cos, sin, qscale, addend=None):
    b, h, n, d = dq.shape
    return dq.new_empty((b, n, weight.shape[1]))


def merge_dx_fusable(g: Tensor, weight: Tensor) -> bool:
    """Whether ``ebr_qkv_rope_merge_dx`` serves a qkv projection's input gradient: 16-bit CUDA head-major gradients
    [B, H, N, 64] and a [3 H 64, 512] weight."""
    if g.dim() != 4 or not g.is_cuda or g.dtype not in (torch.bfloat16, torch.float16):
        return False
    h, d = g.shape[1], g.shape[3]
    return d == 64 and weight.dim() == 2 and tuple(weight.shape) == (3 * h * d, 512)


class _QkvSplit(torch.autograd.Function):
    """Forward: the projection with the split as its epilogue. Backward: the merge (the split's exact adjoint), then
    the projection's two products, all differentiable ops, so every higher order follows."""

    @staticmethod
    def forward(x, weight, cos, sin, qscale, heads):
        return torch.ops.ebr_fused.qkv_rope_split(x, weight, cos, sin, qscale, heads)

    @staticmethod
    def setup_context(ctx, inputs, output):
        x, weight, cos, sin, qscale, heads = inputs
        ctx.save_for_backward(x, weight, cos, sin, qscale)
        ctx.shape = tuple(output[0].shape)
        # The autograd nodes of x and weight: a backward that does not reach one of them (dE/dz in the descent never
        # needs the weight's gradient) skips its product, as the engine skips it for a plain F.linear.
        ctx.nodes = tuple(get_gradient_edge(t).node if t.requires_grad else None for t in (x, weight))

    @staticmethod
    def backward(ctx, gq, gk, gv):
        x, weight, cos, sin, qscale = ctx.saved_tensors
        ref = next(g for g in (gq, gk, gv) if g is not None)
        z = None
        if gq is None or gk is None or gv is None:
            z = torch.zeros(ctx.shape, dtype=ref.dtype, device=ref.device)
        gq, gk, gv = (z if g is None else g for g in (gq, gk, gv))
        need_x, need_w = (_engine_needs(n) for n in ctx.nodes)
        if need_x and not need_w and not torch.is_grad_enabled() and merge_dx_fusable(gq, weight):
            # dE/dz only, no higher-order graph: the merge folded into the GEMM's A operand.
            return qkv_rope_merge_dx_op(gq, gk, gv, weight, cos, sin, qscale), None, None, None, None, None
        gqkv = _Merge.apply(gq, gk, gv, cos, sin, qscale)
        gx = gqkv @ weight.to(gqkv.dtype) if need_x else None
        gw = gqkv.flatten(0, 1).t() @ x.flatten(0, 1) if need_w else None
        return gx, gw, None, None, None, None


def _qkv_split(x: Tensor, weight: Tensor, cos: Tensor, sin: Tensor, qscale: Tensor, heads: int):
    return _QkvSplit.apply(x, weight, cos, sin, qscale, heads)


_qkv_split = torch._dynamo.allow_in_graph(_qkv_split)


def qkv_fusable(x: Tensor, weight: Tensor, heads: int) -> bool:
    """Whether ``ebr_qkv_rope_split`` serves this projection: 16-bit CUDA ``x`` [B, N, C] and ``weight`` [3 H D, C] of
    one dtype, D = 64 or 128, H D a multiple of 256, C a multiple of 64."""
    if x.dim() != 3 or not x.is_cuda or x.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != x.dtype:
        return False
    c = x.shape[-1]
    if weight.dim() != 2 or weight.shape[1] != c or weight.shape[0] % (3 * heads):
        return False
    d = weight.shape[0] // (3 * heads)
    return d in (64, 128) and (heads * d) % 256 == 0 and c % 64 == 0


def qkv_rope_split(x: Tensor, weight: Tensor, cos: Tensor, sin: Tensor, heads: int,
                   qscale: Optional[Tensor] = None) -> Tuple[Tensor, Tensor, Tensor]:  # fmt: skip
    """``rope_split(F.linear(x, weight), cos, sin, heads, qscale)`` as one tensor-core GEMM whose epilogue rotates and
    lays out q, k, v (``ebr_qkv_rope_split``); shapes the kernel does not take run the GEMM and the split kernel.
    ``x`` [B, N, C], ``weight`` [3 H D, C] (no bias); differentiable to every order in x and weight."""
    if qscale is None:
        qscale = x.new_zeros((0,), dtype=torch.float32)
    if not qkv_fusable(x, weight, heads):
        return rope_split(F.linear(x, weight.to(x.dtype)), cos, sin, heads, qscale if qscale.numel() else None)
    d = weight.shape[0] // (3 * heads)
    if tuple(cos.shape) != (x.shape[1], d) or tuple(sin.shape) != (x.shape[1], d):
        raise ValueError(f"qkv_rope_split: tables must be [N, D], got {tuple(cos.shape)} (N={x.shape[1]}, D={d})")
    return _qkv_split(x, weight, cos, sin, qscale.detach(), heads)


# ---------------------------------------------------------------------------------------------------- o projection


@torch.library.custom_op("ebr_fused::o_proj", mutates_args=())
def o_proj_op(o: Tensor, weight: Tensor) -> Tensor:
    _require_cuda(o, "o_proj")
    b, h, n, d = o.shape
    if o.stride(-1) != 1:
        o = o.contiguous()
    weight = weight.to(o.dtype).contiguous()
    y = torch.empty((b, n, weight.shape[0]), device=o.device, dtype=o.dtype)
    op = _native.Operand(o.data_ptr(), o.stride(0), o.stride(1), o.stride(2))
    _native.check(
        _native.lib().ebr_o_proj(_DTYPES[o.dtype], b, h, n, d, weight.shape[0], ctypes.byref(op), weight.data_ptr(),
                                 y.data_ptr(), _stream()),  # fmt: skip
        "o_proj",
    )
    return y


@o_proj_op.register_fake
def _(o, weight):
    b, _, n, _ = o.shape
    return o.new_empty((b, n, weight.shape[0]))


class _OProj(torch.autograd.Function):
    """Forward: the projection read from the head-major attention output. Backward: the two products, as
    differentiable ops, each only when the running backward reaches its input; the gradient of O is returned as a
    head-major view of [B, N, H D] (the attention's backward reads strided dO), so no transpose is made."""

    @staticmethod
    def forward(o, weight):
        return torch.ops.ebr_fused.o_proj(o, weight)

    @staticmethod
    def setup_context(ctx, inputs, output):
        o, weight = inputs
        ctx.save_for_backward(o, weight)
        ctx.nodes = tuple(get_gradient_edge(t).node if t.requires_grad else None for t in (o, weight))

    @staticmethod
    def backward(ctx, gy):
        o, weight = ctx.saved_tensors
        b, h, n, d = o.shape
        need_o, need_w = (_engine_needs(nd) for nd in ctx.nodes)
        go = (gy @ weight.to(gy.dtype)).view(b, n, h, d).transpose(1, 2) if need_o else None
        gw = gy.flatten(0, 1).t() @ o.transpose(1, 2).reshape(b * n, h * d) if need_w else None
        return go, gw


def _o_proj(o: Tensor, weight: Tensor) -> Tensor:
    return _OProj.apply(o, weight)


_o_proj = torch._dynamo.allow_in_graph(_o_proj)


def o_proj_fusable(o: Tensor, weight: Tensor) -> bool:
    """Whether ``ebr_o_proj`` serves this projection: 16-bit CUDA ``o`` [B, H, N, D] with unit head-dim stride and
    16-byte-multiple strides, ``weight`` [C_out, H D] of the same dtype, D = 64 or 128, C_out a multiple of 256."""
    if o.dim() != 4 or not o.is_cuda or o.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != o.dtype:
        return False
    b, h, n, d = o.shape
    if d not in (64, 128) or weight.dim() != 2 or weight.shape[1] != h * d or weight.shape[0] % 256:
        return False
    return o.stride(-1) == 1 and all(s % 8 == 0 for s in o.stride()[:3]) and o.data_ptr() % 16 == 0


def o_proj(o: Tensor, weight: Tensor) -> Tensor:
    """``F.linear(o.transpose(1, 2).reshape(B, N, H * D), weight)`` without the transpose copy (``ebr_o_proj``); shapes
    the kernel does not take run the copy and the GEMM. ``o`` [B, H, N, D], ``weight`` [C_out, H D] (no bias);
    differentiable to every order in o and weight."""
    if not o_proj_fusable(o, weight):
        b, h, n, d = o.shape
        return F.linear(o.transpose(1, 2).reshape(b, n, h * d), weight.to(o.dtype))
    return _o_proj(o, weight)


# ---------------------------------------------------------------------------------------------------- rms_norm


def _rows(x: Tensor) -> Tuple[int, int]:
    c = x.shape[-1]
    return x.numel() // c if c else 0, c


def _rms_norm_bwd_kernel(s: Tensor, rstd: Tensor, gy: Tensor) -> Tensor:
    gy = gy.to(s.dtype).contiguous()
    rows, c = _rows(s)
    gs = torch.empty_like(s)
    _native.check(
        _native.lib().ebr_rms_norm_bwd(_DTYPES[s.dtype], rows, c, s.data_ptr(), rstd.data_ptr(), gy.data_ptr(),
                                       gs.data_ptr(), _stream()),  # fmt: skip
        "rms_norm_bwd",
    )
    return gs


class _RmsNormBwd(torch.autograd.Function):
    """The rms_norm backward gs = r (gy - xh mean(gy xh)) as one kernel, differentiable once more by the closed-form
    double backward (``ebr_rms_norm_bwd2``): the graph a second-order training step builds through it. ``x`` / ``a``
    only carry the graph (s = x + a was formed by the forward kernel); ds is the gradient of both."""

    @staticmethod
    def forward(ctx, x: Tensor, a: Optional[Tensor], s: Tensor, rstd: Tensor, gy: Tensor) -> Tensor:
        gy = gy.to(s.dtype).contiguous()
        ctx.save_for_backward(s, rstd, gy)
        ctx.has_a = a is not None
        return _rms_norm_bwd_kernel(s, rstd, gy)

    @staticmethod
    @once_differentiable
    def backward(ctx, u: Tensor):
        s, rstd, gy = ctx.saved_tensors
        u = u.to(s.dtype).contiguous()
        rows, c = _rows(s)
        ds, dgy = torch.empty_like(s), torch.empty_like(s)
        _native.check(
            _native.lib().ebr_rms_norm_bwd2(_DTYPES[s.dtype], rows, c, s.data_ptr(), rstd.data_ptr(), gy.data_ptr(),
                                            u.data_ptr(), ds.data_ptr(), dgy.data_ptr(), _stream()),  # fmt: skip
            "rms_norm_bwd2",
        )
        return ds, (ds if ctx.has_a else None), None, None, dgy


def add_rms_norm_fwd(x: Tensor, a: Optional[Tensor] = None, eps: float = 1e-5) -> Tuple[Tensor, Tensor, Tensor]:
    """``rms_norm(x + a)`` without autograd, returning (y, s = round(x + a) (x itself when a is None), rstd [rows]
    float32): what the backward needs, for callers that run it explicitly."""
    _require_cuda(x, "add_rms_norm")
    x = x.contiguous()
    a = None if a is None else a.to(x.dtype).contiguous()
    rows, c = _rows(x)
    y = torch.empty_like(x)
    s = torch.empty_like(x) if a is not None else None
    rstd = torch.empty(rows, device=x.device, dtype=torch.float32)
    _native.check(
        _native.lib().ebr_add_rms_norm(_DTYPES[x.dtype], rows, c, eps, x.data_ptr(), _ptr(a), _ptr(s),
                                       y.data_ptr(), rstd.data_ptr(), None, 0.0, _stream()),  # fmt: skip
        "add_rms_norm",
    )
    return y, (x if s is None else s), rstd


def rms_norm_bwd(s: Tensor, rstd: Tensor, gy: Tensor) -> Tensor:
    """The gradient of ``rms_norm(s)`` (both x and a of ``add_rms_norm``) from the forward's s and rstd, one kernel."""
    return _rms_norm_bwd_kernel(s, rstd, gy)


def swiglu_bwd(h: Tensor, gout: Tensor) -> Tensor:
    """The gradient of the SwiGLU activation with respect to h = [gate, up], one kernel (no higher-order graph)."""
    return _swiglu_bwd_kernel(h.contiguous(), gout)


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, a: Optional[Tensor], eps: float) -> Tensor:
        y, s, rstd = add_rms_norm_fwd(x, a, eps)
        ctx.save_for_backward(x.contiguous(), None if a is None else a.to(x.dtype), s, rstd)
        ctx.eps = eps
        ctx.has_a = a is not None
        return y

    @staticmethod
    def backward(ctx, gy: Tensor):
        x, a, s, rstd = ctx.saved_tensors
        if torch.is_grad_enabled():
            gs = _RmsNormBwd.apply(x, a, s, rstd, gy)  # a graph for the double backward
        else:
            gs = _rms_norm_bwd_kernel(s, rstd, gy)
        return gs, (gs if ctx.has_a else None), None


def add_rms_norm(x: Tensor, a: Optional[Tensor] = None, eps: float = 1e-5) -> Tensor:
    """``rms_norm(x + a)`` (``a`` optional): the residual add rounded to the I/O type, then the row norm in float32
    (``models/layers.py:37-42``). Differentiable to second order: the backward and its own backward are fused
    kernels."""
    return _AddRMSNorm.apply(x, a, float(eps))


# ---------------------------------------------------------------------------------------------------- SwiGLU


class _SwiGLUAct(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h: Tensor) -> Tensor:
        _require_cuda(h, "swiglu")
        h = h.contiguous()
        rows, c2 = _rows(h)
        inter = c2 // 2
        out = torch.empty((*h.shape[:-1], inter), device=h.device, dtype=h.dtype)
        _native.check(
            _native.lib().ebr_swiglu_fwd(_DTYPES[h.dtype], rows, inter, h.data_ptr(), out.data_ptr(), _stream()),
            "swiglu_fwd",
        )
        ctx.save_for_backward(h)
        return out

    @staticmethod
    def backward(ctx, gout: Tensor):
        (h,) = ctx.saved_tensors
        return _swiglu_grad(h, gout)


def _swiglu_bwd_kernel(h: Tensor, gout: Tensor) -> Tensor:
    gout = gout.to(h.dtype).contiguous()
    rows, c2 = _rows(h)
    gh = torch.empty_like(h)
    _native.check(
        _native.lib().ebr_swiglu_bwd(_DTYPES[h.dtype], rows, c2 // 2, h.data_ptr(), gout.data_ptr(), gh.data_ptr(),
                                     _stream()),  # fmt: skip
        "swiglu_bwd",
    )
    return gh


class _SwigluBwd(torch.autograd.Function):
    """d act / d h applied to gout as one kernel, differentiable once more by the closed-form double backward
    (``ebr_swiglu_bwd2``): the graph a second-order training step builds through it."""

    @staticmethod
    def forward(ctx, h: Tensor, gout: Tensor) -> Tensor:
        h = h.contiguous()
        gout = gout.to(h.dtype).contiguous()
        ctx.save_for_backward(h, gout)
        return _swiglu_bwd_kernel(h, gout)

    @staticmethod
    @once_differentiable
    def backward(ctx, u: Tensor):
        h, gout = ctx.saved_tensors
        u = u.to(h.dtype).contiguous()
        rows, c2 = _rows(h)
        dh, dgout = torch.empty_like(h), torch.empty_like(gout)
        _native.check(
            _native.lib().ebr_swiglu_bwd2(_DTYPES[h.dtype], rows, c2 // 2, h.data_ptr(), gout.data_ptr(), u.data_ptr(),
                                          dh.data_ptr(), dgout.data_ptr(), _stream()),  # fmt: skip
            "swiglu_bwd2",
        )
        return dh, dgout


def _swiglu_grad(h: Tensor, gout: Tensor) -> Tensor:
    """d act / d h applied to gout: the fused kernel, differentiable once more when a higher-order graph is built."""
    if torch.is_grad_enabled():
        return _SwigluBwd.apply(h, gout)
    return _swiglu_bwd_kernel(h.contiguous(), gout)


@torch.library.custom_op("ebr_fused::gate_up_swiglu", mutates_args=())
def gate_up_swiglu_op(x: Tensor, weight: Tensor) -> Tuple[Tensor, Tensor]:
    _require_cuda(x, "gate_up_swiglu")
    x = x.contiguous()
    weight = weight.to(x.dtype).contiguous()
    rows, c = _rows(x)
    i2 = weight.shape[0]
    h = torch.empty((*x.shape[:-1], i2), device=x.device, dtype=x.dtype)
    act = torch.empty((*x.shape[:-1], i2 // 2), device=x.device, dtype=x.dtype)
    _native.check(
        _native.lib().ebr_gate_up_swiglu(_DTYPES[x.dtype], rows, c, i2 // 2, x.data_ptr(), c, weight.data_ptr(),
                                         h.data_ptr(), act.data_ptr(), _stream()),  # fmt: skip
        "gate_up_swiglu",
    )
    return h, act


@gate_up_swiglu_op.register_fake
def _(x, weight):
    i2 = weight.shape[0]
    return x.new_empty((*x.shape[:-1], i2)), x.new_empty((*x.shape[:-1], i2 // 2))


class _GateUpAct(torch.autograd.Function):
    """Forward: the gate / up GEMM with the SwiGLU activation as its epilogue (h is kept for the backward). Backward:
    the activation's gradient from the stored h, then the projection's two products, each only when the running
    backward reaches its input; building a higher-order graph it recomputes h = x W^T with differentiable ops, so the
    double backward differentiates through the projection too."""

    @staticmethod
    def forward(ctx, x, weight):
        h, act = torch.ops.ebr_fused.gate_up_swiglu(x, weight)
        ctx.save_for_backward(x, weight, h)
        ctx.nodes = tuple(get_gradient_edge(t).node if t.requires_grad else None for t in (x, weight))
        return act

    @staticmethod
    def backward(ctx, gact):
        x, weight, h = ctx.saved_tensors
        need_x, need_w = (_engine_needs(nd) for nd in ctx.nodes)
        if torch.is_grad_enabled():
            h = F.linear(x, weight.to(x.dtype))
        gh = _swiglu_grad(h, gact)
        gx = gh @ weight.to(gh.dtype) if need_x else None
        gw = gh.flatten(0, -2).t() @ x.flatten(0, -2) if need_w else None
        return gx, gw


def _gate_up(x: Tensor, weight: Tensor) -> Tensor:
    return _GateUpAct.apply(x, weight)


_gate_up = torch._dynamo.allow_in_graph(_gate_up)


def gate_up_fusable(x: Tensor, weight: Tensor) -> bool:
    """Whether ``ebr_gate_up_swiglu`` serves this projection: 16-bit CUDA ``x`` [..., C] and ``weight`` [2 I, C] of
    one dtype, C a multiple of 64, I a multiple of 128."""
    if not x.is_cuda or x.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != x.dtype:
        return False
    c = x.shape[-1]
    return weight.dim() == 2 and weight.shape[1] == c and c % 64 == 0 and weight.shape[0] % 256 == 0


def gate_up_swiglu(x: Tensor, weight: Tensor) -> Tensor:
    """``swiglu_act(F.linear(x, weight))`` as one GEMM with the activation in its epilogue (``ebr_gate_up_swiglu``);
    shapes it does not take run the GEMM and the activation kernel. Differentiable to every order in x and weight."""
    if not gate_up_fusable(x, weight):
        return swiglu_act(F.linear(x, weight.to(x.dtype)))
    return _gate_up(x, weight)


def swiglu_act(h: Tensor) -> Tensor:
    """``silu(gate) * up`` for ``gate, up = h.chunk(2, -1)`` (``models/layers.py:82-84``)."""
    if h.shape[-1] % 2:
        raise ValueError(f"swiglu_act expects an even last dim, got {h.shape[-1]}")
    return _SwiGLUAct.apply(h)


# ---------------------------------------------------------------------------------------------------- descent step


@torch.no_grad()
def noisy_point(z: Tensor, noise: Optional[Tensor] = None, sigma: float = 1.0, eps: float = 1e-5) -> Tensor:
    """``v = rms_norm(z) + round(noise * sigma)`` in one kernel (no autograd: inference microsteps). With ``noise``
    None, ``v = rms_norm(z)`` (``models/energy.py:226-232``, ``:322-341``)."""
    _require_cuda(z, "noisy_point")
    z = z.contiguous()
    rows, c = _rows(z)
    v = torch.empty_like(z)
    noise = None if noise is None else noise.to(z.dtype).contiguous()
    _native.check(
        _native.lib().ebr_add_rms_norm(_DTYPES[z.dtype], rows, c, eps, z.data_ptr(), None, None, v.data_ptr(), None,
                                       _ptr(noise), float(sigma), _stream()),  # fmt: skip
        "noisy_point",
    )
    return v


@torch.no_grad()
def step_and_project(v: Tensor, g: Tensor, alpha: float, eps: float = 1e-5) -> Tensor:
    """``z' = sphere(v - alpha * g)``: each row (board) of ``v`` rescaled to unit RMS in float32 after the step, in
    two kernels (``models/energy.py:219-241``; no autograd: inference microsteps)."""
    _require_cuda(v, "step_and_project")
    v, g = v.contiguous(), g.to(v.dtype).contiguous()
    rows = v.shape[0]
    row_elems = v.numel() // rows if rows else 0
    z = torch.empty_like(v)
    lib = _native.lib()
    nfl = lib.ebr_descent_step_scratch_floats(rows, row_elems)
    partial = torch.empty(max(int(nfl), 1), device=v.device, dtype=torch.float32)
    _native.check(
        lib.ebr_descent_step(_DTYPES[v.dtype], rows, row_elems, float(alpha), float(eps), v.data_ptr(), g.data_ptr(),
                             z.data_ptr(), partial.data_ptr(), partial.numel(), _stream()),  # fmt: skip
        "descent_step",
    )
    return z


__all__ = [
    "add_rms_norm",
    "gate_up_fusable",
    "gate_up_swiglu",
    "gate_up_swiglu_op",
    "noisy_point",
    "o_proj",
    "o_proj_fusable",
    "o_proj_op",
    "qkv_fusable",
    "qkv_rope_split",
    "qkv_rope_split_op",
    "quarter_swap",
    "rope_merge_op",
    "rope_split",
    "rope_split_op",
    "rotary_tables",
    "step_and_project",
    "swiglu_act",
]
