"""Latent-descent energy network on the sm_100a kernels: the caller that drives the attention hot path.

The network computes the reference's scalar energy E(z; x) and its descent microstep (``models/energy.py``
``ScalarEnergy`` :190-216, ``EnergyDescent.forward`` :285-319; blocks of ``models/attention.py`` :181-266), but is
built as a pipeline of this package's fused CUDA ops rather than as a tree of layer modules:

    h = v + x
    per block:  q, k, v = qkv_rope_split(h W_qkv^T)        (one tcgen05 GEMM; 2D RoPE + head-major layout epilogue)
                y = fused_attention(q * temperature, k, v)  (the sm_100a forward / backward / double backward)
                h = add_rms_norm(h, o_proj(y))              (projection read from the head-major output)
                h = add_rms_norm(h, gate_up_swiglu(h) W_down^T)
    E = sum over cells of  w2 . silu(W1 h + b1)   (softplus per cell when the head is non-negative)

Parameters live in one flat module (``LatentEnergyNet``) in float32 and are cast to the compute dtype at use, as the
reference's casted layers do; ``load_reference_state`` / ``reference_state`` translate to and from the reference's
state-dict names, so weights move between the two and the golden tests pin this network to the reference's outputs.
Every op runs on CUDA; there is no CPU path (the CPU restatement used as a yardstick lives in the test oracle).

Graded microsteps (those differentiated again by training) apply the per-head temperature as a differentiable
product; elsewhere it is folded into the projection's epilogue, as the reference does (``models/attention.py``
:228-240).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from ebr_b200 import layers as fl
from ebr_b200.fused_attn import fused_attention

AttentionFn = Callable[[Tensor, Tensor, Tensor], Tensor]


@dataclass(frozen=True)
class NetShape:
    """Architecture and descent settings. Defaults: the benchmark network (4 layers, hidden 512, 8 heads x 64, SwiGLU
    4x, bf16) with the reference's eval descent (step 250, noise 0.05, config/arch/ebr.yaml)."""

    board: tuple[int, int] = (9, 9)
    vocab: int = 10
    hidden: int = 512
    heads: int = 8
    layers: int = 4
    expansion: float = 4.0
    cell_softplus: bool = False
    dtype: torch.dtype = torch.bfloat16
    eps: float = 1e-5
    rope_base: float = 10000.0
    step_size: float = 250.0
    noise_scale: float = 0.05
    init_std: float = 1.0

    @property
    def seq_len(self) -> int:
        return self.board[0] * self.board[1]

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def mlp_width(self) -> int:
        """2/3 of ``expansion * hidden`` rounded up to a multiple of 256 (the reference's SwiGLU width rule,
        ``models/layers.py:74-80``)."""
        width = round(self.expansion * self.hidden * 2 / 3)
        return (width + 255) // 256 * 256


def rope_tables(shape: NetShape, device=None) -> tuple[Tensor, Tensor]:
    """``[H * W, D]`` cos / sign-folded sin tables of the 2D rotation: the first half of each head's channels turns
    with the cell's row, the second with its column, at frequencies ``1 / base^(2i / (D / 2))`` (the angles of the
    reference's ``RotaryEmbedding2D``, ``models/layers.py:98-117``, evaluated in the same form so that the tables
    agree to the last bit)."""
    half = shape.head_dim // 2
    freq = 1.0 / (shape.rope_base ** (torch.arange(0, half, 2, dtype=torch.float32, device=device) / half))
    ang_h = torch.outer(torch.arange(shape.board[0], dtype=torch.float32, device=device), freq).repeat(1, 2)
    ang_w = torch.outer(torch.arange(shape.board[1], dtype=torch.float32, device=device), freq).repeat(1, 2)
    return fl.rotary_tables(ang_h.cos(), ang_h.sin(), ang_w.cos(), ang_w.sin())


class _BlockWeights(nn.Module):
    def __init__(self, shape: NetShape) -> None:
        super().__init__()
        c, w = shape.hidden, shape.mlp_width
        self.w_qkv = nn.Parameter(torch.empty(3 * c, c))
        self.w_out = nn.Parameter(torch.empty(c, c))
        self.log_temp = nn.Parameter(torch.zeros(shape.heads))
        self.w_gate_up = nn.Parameter(torch.empty(2 * w, c))
        self.w_down = nn.Parameter(torch.empty(c, w))


# this module's parameter name -> the reference's state-dict name ({i}: block index)
_BLOCK_NAMES = {
    "log_temp": "level.energy.layers.{i}.self_attn.log_logit_scale",
    "w_qkv": "level.energy.layers.{i}.self_attn.qkv_proj.weight",
    "w_out": "level.energy.layers.{i}.self_attn.o_proj.weight",
    "w_gate_up": "level.energy.layers.{i}.mlp.gate_up_proj.weight",
    "w_down": "level.energy.layers.{i}.mlp.down_proj.weight",
}
_TOP_NAMES = {
    "embedding": "embed_tokens.embedding_weight",
    "readout": "lm_head.weight",
    "cell_w1": "level.energy.energy_head.hidden.weight",
    "cell_b1": "level.energy.energy_head.hidden.bias",
    "cell_w2": "level.energy.energy_head.output.weight",
}


class LatentEnergyNet(nn.Module):
    """Token embedding, the energy E(z; x), dE/dz, the descent microstep and the readout, on CUDA.

    ``attention`` replaces the sm_100a attention by another callable with the same ``(q, k, v) -> o`` contract on
    ``[B, H, N, D]`` tensors; the tests use it to measure the kernels against softmax attention inside the same
    network. There is no registry and no fallback: the default is ``fused_attention``."""

    def __init__(self, shape: NetShape, attention: Optional[AttentionFn] = None,
                 generator: Optional[torch.Generator] = None) -> None:  # fmt: skip
        super().__init__()
        self.shape = shape
        c, v = shape.hidden, shape.vocab
        self.embedding = nn.Parameter(torch.empty(v, c))
        self.readout = nn.Parameter(torch.empty(v, c))
        self.blocks = nn.ModuleList(_BlockWeights(shape) for _ in range(shape.layers))
        self.cell_w1 = nn.Parameter(torch.empty(c, c))
        self.cell_b1 = nn.Parameter(torch.zeros(c))
        self.cell_w2 = nn.Parameter(torch.empty(1, c))
        cos, sin = rope_tables(shape)
        self.register_buffer("rope_cos", cos, persistent=False)
        self.register_buffer("rope_sin", sin, persistent=False)
        self._attention = attention
        self.reset_parameters(generator)

    # -- parameters -------------------------------------------------------------------------------------------------

    @torch.no_grad()
    def reset_parameters(self, generator: Optional[torch.Generator] = None) -> None:
        """Truncated normals (two standard deviations) with fan-in scaling; the embedding at 1/sqrt(hidden); zero
        temperatures and bias."""

        def fill(t: Tensor, std: float) -> None:
            t.copy_(torch.randn(t.shape, generator=generator, device=t.device).clamp_(-2.0, 2.0) * std)

        fill(self.embedding, self.shape.hidden**-0.5)
        fill(self.readout, self.shape.hidden**-0.5)
        for blk in self.blocks:
            for w in (blk.w_qkv, blk.w_out, blk.w_gate_up, blk.w_down):
                fill(w, w.shape[1] ** -0.5)
            blk.log_temp.zero_()
        fill(self.cell_w1, self.shape.hidden**-0.5)
        self.cell_b1.zero_()
        fill(self.cell_w2, self.shape.hidden**-0.5)

    def _name_map(self) -> dict[str, str]:
        out = dict(_TOP_NAMES)
        for i in range(len(self.blocks)):
            for mine, ref in _BLOCK_NAMES.items():
                out[f"blocks.{i}.{mine}"] = ref.format(i=i)
        return out

    @torch.no_grad()
    def load_reference_state(self, state: dict[str, Tensor]) -> None:
        """Copy weights from a state dict in the reference's names (``InnerNetwork.state_dict()``); every parameter
        of this network must be present."""
        own = dict(self.named_parameters())
        for mine, ref in self._name_map().items():
            if ref not in state:
                raise KeyError(f"reference state lacks {ref!r}")
            own[mine].copy_(state[ref].to(own[mine].device, torch.float32))

    @torch.no_grad()
    def reference_state(self) -> dict[str, Tensor]:
        """This network's weights under the reference's state-dict names."""
        own = dict(self.named_parameters())
        return {ref: own[mine].detach().clone() for mine, ref in self._name_map().items()}

    # -- energy -----------------------------------------------------------------------------------------------------

    def embed(self, tokens: Tensor) -> Tensor:
        """x = sqrt(hidden) * embedding[tokens] in the compute dtype, ``[B, L, hidden]``."""
        dt = self.shape.dtype
        return F.embedding(tokens.to(torch.int32), self.embedding.to(dt)) * math.sqrt(self.shape.hidden)

    def fresh_states(self, rows: int, generator: Optional[torch.Generator] = None) -> Tensor:
        """Initial latents ``[rows, L, hidden]``: a normal truncated at two standard deviations, times init_std."""
        s = self.shape
        z = torch.randn((rows, s.seq_len, s.hidden), generator=generator, device=self.embedding.device)
        return (z.clamp_(-2.0, 2.0) * s.init_std).to(s.dtype)

    def _attend(self, q: Tensor, k: Tensor, v: Tensor) -> Tensor:
        if self._attention is not None:
            return self._attention(q, k, v)
        return fused_attention(q, k, v, scale=q.shape[-1] ** -0.5)

    def _block(self, blk: _BlockWeights, h: Tensor, graded: bool) -> Tensor:
        s, dt = self.shape, h.dtype
        folded = None if graded else blk.log_temp.detach().exp().to(dt)
        q, k, v = fl.qkv_rope_split(h, blk.w_qkv.to(dt), self.rope_cos, self.rope_sin, s.heads, folded)
        if graded:
            q = q * blk.log_temp.exp().to(dt).view(1, -1, 1, 1)
        h = fl.add_rms_norm(h, fl.o_proj(self._attend(q, k, v), blk.w_out.to(dt)), s.eps)
        mlp = F.linear(fl.gate_up_swiglu(h, blk.w_gate_up.to(dt)), blk.w_down.to(dt))
        return fl.add_rms_norm(h, mlp, s.eps)

    def energy(self, v: Tensor, x: Tensor, graded: bool = False) -> Tensor:
        """E(v; x) per row, ``[B]`` float32. ``graded``: the call's dE/dv will be differentiated again."""
        dt = v.dtype
        h = v + x
        for blk in self.blocks:
            h = self._block(blk, h, graded)
        cell = F.linear(F.silu(F.linear(h, self.cell_w1.to(dt), self.cell_b1.to(dt))), self.cell_w2.to(dt))
        if self.shape.cell_softplus:
            cell = F.softplus(cell.float())
        return cell.float().squeeze(-1).sum(dim=1)

    def energy_and_grad(self, v: Tensor, x: Tensor, create_graph: bool = False) -> tuple[Tensor, Tensor]:
        """(E per row, dE/dv); with ``create_graph`` the gradient is itself differentiable (double backward). Without
        it, on the shapes every fused kernel takes, the blocks' backward runs explicitly (``_energy_and_grad_dz``)."""
        if not create_graph and self._dz_fusable(v):
            return self._energy_and_grad_dz(v, x)
        with torch.enable_grad():
            if not v.requires_grad:
                v = v.detach().requires_grad_(True)
            e = self.energy(v, x, graded=create_graph)
            (g,) = torch.autograd.grad(e.sum(), v, create_graph=create_graph)
        return (e if create_graph else e.detach()), g

    def _dz_fusable(self, v: Tensor) -> bool:
        """Whether the explicit dE/dv path serves this call: the default attention, 16-bit CUDA activations, head dim 64
        or 128 and hidden 512 (the shapes the fused projections take; the merge GEMM serves head dim 64, and 128 takes
        the RoPE-merge kernel and a cuBLAS product)."""
        s = self.shape
        return (self._attention is None and v.is_cuda and v.dtype in (torch.bfloat16, torch.float16)
                and s.head_dim in (64, 128) and s.hidden == 512 and (2 * s.mlp_width) % 256 == 0)  # fmt: skip

    def _energy_and_grad_dz(self, v: Tensor, x: Tensor) -> tuple[Tensor, Tensor]:
        """(E, dE/dv) with the blocks' backward run explicitly, not through autograd. Each block's forward runs the same
        fused ops as ``_block`` and keeps what its backward needs; the backward then runs the fused kernels in reverse.
        A block input's residual gradient joins its branch gradient inside a product instead of a separate add:
        through the merge GEMM's addend at the attention input (rounded as the add would be; at head dim 128, cuBLAS's
        beta = 1 accumulate after the RoPE-merge kernel) and cuBLAS's beta = 1 accumulate at the MLP input (one
        rounding instead of two). Only dE/dv: no parameter gradients."""
        s, dt = self.shape, v.dtype
        b, n, c = v.shape
        hh, d = s.heads, s.head_dim
        scale = d**-0.5
        saved = []
        with torch.no_grad():
            h = v + x
            for blk in self.blocks:
                folded = blk.log_temp.detach().exp().to(dt)
                w_qkv, w_out, w_gu, w_down = (w.detach().to(dt) for w in (blk.w_qkv, blk.w_out, blk.w_gate_up,
                                                                              blk.w_down))  # fmt: skip
                q, k, vv = fl.qkv_rope_split_op(h, w_qkv, self.rope_cos, self.rope_sin, folded, hh)
                o, lse = torch.ops.ebr_fused.attn_fwd(q, k, vv, scale)
                h1, s1, r1 = fl.add_rms_norm_fwd(h, fl.o_proj_op(o, w_out), s.eps)
                gu, act = fl.gate_up_swiglu_op(h1, w_gu)
                h, s2, r2 = fl.add_rms_norm_fwd(h1, F.linear(act, w_down), s.eps)
                saved.append((q, k, vv, o, lse, s1, r1, gu, s2, r2, w_qkv, w_out, w_gu, w_down, folded))
        with torch.enable_grad():  # the energy head (small): autograd
            hd = h.detach().requires_grad_(True)
            cell = F.linear(F.silu(F.linear(hd, self.cell_w1.to(dt), self.cell_b1.to(dt))), self.cell_w2.to(dt))
            if s.cell_softplus:
                cell = F.softplus(cell.float())
            e = cell.float().squeeze(-1).sum(dim=1)
            (g,) = torch.autograd.grad(e.sum(), hd)
        with torch.no_grad():
            for q, k, vv, o, lse, s1, r1, gu, s2, r2, w_qkv, w_out, w_gu, w_down, folded in reversed(saved):
                ds2 = fl.rms_norm_bwd(s2, r2, g)
                d_gu = fl.swiglu_bwd(gu, ds2 @ w_down)
                g1 = torch.addmm(ds2.reshape(-1, c), d_gu.reshape(-1, d_gu.shape[-1]), w_gu).view(b, n, c)
                ds1 = fl.rms_norm_bwd(s1, r1, g1)
                d_o = (ds1 @ w_out).view(b, n, hh, d).transpose(1, 2)
                dq, dk, dv = torch.ops.ebr_fused.attn_bwd(q, k, vv, o, lse, d_o, scale)
                if fl.merge_dx_fusable(dq, w_qkv):
                    g = fl.qkv_rope_merge_dx_op(dq, dk, dv, w_qkv, self.rope_cos, self.rope_sin, folded, ds1)
                else:  # head dim 128: the merged gradient [B N, 3 H D] times W, the residual gradient accumulated
                    merged = fl.rope_merge_op(dq, dk, dv, self.rope_cos, self.rope_sin, folded)
                    g = torch.addmm(ds1.reshape(-1, c), merged.reshape(-1, merged.shape[-1]), w_qkv).view(b, n, c)
        return e.detach(), g

    # -- descent ----------------------------------------------------------------------------------------------------

    def microstep(self, z: Tensor, x: Tensor, *, graded: bool = False, noise: Optional[Tensor] = None,
                  sigma: Optional[float] = None, alpha=None) -> tuple[Tensor, Tensor]:  # fmt: skip
        """One descent step ``z' = sphere(rms_norm(z) + noise - alpha dE/dv)``; returns (z', E per row).

        ``noise``: replayed noise, added as is; otherwise ``sigma`` (default noise_scale) times a fresh normal draw.
        ``alpha``: a float or a per-row ``[B, 1, 1]`` tensor (default step_size). ``graded``: build the graph through
        dE/dv (training); otherwise the step runs as fused kernels and returns detached tensors."""
        s = self.shape
        sigma = s.noise_scale if sigma is None else sigma
        alpha = s.step_size if alpha is None else alpha
        if not graded and not torch.is_tensor(alpha):
            if noise is not None:
                v = fl.noisy_point(z, noise, 1.0, s.eps)
            else:
                v = fl.noisy_point(z, torch.randn_like(z) if sigma else None, float(sigma), s.eps)
            e, g = self.energy_and_grad(v, x)
            return fl.step_and_project(v, g, float(alpha), s.eps), e.detach()
        v = fl.add_rms_norm(z, None, s.eps)  # cell_unit_rms as one kernel, differentiable to second order
        if noise is not None:
            v = v + noise.to(v.dtype)
        elif sigma:
            v = v + torch.randn_like(v) * sigma
        e, g = self.energy_and_grad(v, x, create_graph=graded)
        step = alpha.to(v.dtype) if torch.is_tensor(alpha) else alpha
        z_next = board_unit_rms(v - step * g, s.eps)
        return (z_next, e) if graded else (z_next.detach(), e.detach())

    def decode(self, z: Tensor) -> Tensor:
        """Per-cell token logits ``[B, L, vocab]``."""
        return F.linear(z, self.readout.to(z.dtype))


def cell_unit_rms(z: Tensor, eps: float = 1e-5) -> Tensor:
    """Each cell's vector scaled to unit RMS over the hidden dim, in float32 (rms_norm, ``models/layers.py:37-42``);
    differentiable."""
    zf = z.float()
    return (zf * torch.rsqrt(zf.square().mean(-1, keepdim=True) + eps)).to(z.dtype)


def board_unit_rms(z: Tensor, eps: float = 1e-5) -> Tensor:
    """Each row (whole board) scaled to unit RMS, in float32 (sphere, ``models/energy.py:219-222``); differentiable."""
    zf = z.float()
    rms = zf.square().mean(dim=(1, 2), keepdim=True).sqrt().clamp_min(eps)
    return (zf / rms).to(z.dtype)


def descend(net: LatentEnergyNet, z: Tensor, x: Tensor, steps: int, *, sigma: Optional[float] = None,
            noises: Optional[list[Tensor]] = None) -> tuple[Tensor, Tensor]:  # fmt: skip
    """``steps`` inference microsteps (forward + first-order dE/dz each). Returns (z, energies of the last)."""
    e = None
    for t in range(steps):
        z, e = net.microstep(z, x, sigma=sigma, noise=None if noises is None else noises[t])
    return z, e


@torch.no_grad()
def lowest_energy_pick(energy: Tensor, samples: int) -> Tensor:
    """``energy`` [inputs * samples] (each input's samples contiguous) -> index of each input's lowest-energy sample
    (the evaluation protocol's pick, ``evaluators/protocol.py:10-12``)."""
    return energy.view(-1, samples).argmin(dim=1)


def stablemax_cross_entropy(logits: Tensor, labels: Tensor) -> Tensor:
    """Per-cell cross entropy under stablemax (exp(x) replaced by x + 1 for x >= 0 and 1 / (1 - x) below), in
    float64 (the reference's training loss, ``models/losses.py:29-44``). ``logits`` [..., V], ``labels`` [...]."""
    x = logits.double()
    s = torch.where(x < 0, 1.0 / (1.0 - x + 1e-30), x + 1.0)
    logp = torch.log(s / s.sum(-1, keepdim=True))
    return -logp.gather(-1, labels.long().unsqueeze(-1)).squeeze(-1)


class MicrostepGraph:
    """One no-graph descent microstep of a fixed batch shape, captured once as a CUDA graph and then replayed.

    Training rollouts -- a segment's ungraded prefix, forward SXM's candidate trajectories -- run a few hundred rows
    of 81-100 tokens: every microstep is a few hundred kernels of a few microseconds each, and launched one by one from
    Python their host cost exceeds their GPU time. A replay issues the whole microstep (forward, dE/dv, step) as one
    graph launch. The graph reads the parameters in place (the optimizer updates them in place), so one capture serves
    every training step. ``step`` copies its inputs into the graph's buffers and returns the graph's output tensor,
    which the next replay overwrites. Noise is an input (drawn by the caller), so the graph consumes no random
    numbers."""

    def __init__(self, net: LatentEnergyNet, z: Tensor, x: Tensor, alpha) -> None:
        self.net = net
        self.z, self.x = z.detach().clone(), x.detach().clone()
        self.noise = torch.zeros_like(self.z)
        self.alpha = alpha.detach().clone() if torch.is_tensor(alpha) else alpha
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(2):  # first launches outside the capture (kernel attributes, the allocator's pool)
                self._run()
        torch.cuda.current_stream().wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        # thread_local: CUDA calls of other threads (NCCL's, under torchrun) do not invalidate this capture
        with torch.no_grad(), torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            self.out = self._run()

    def _run(self) -> Tensor:
        z_next, _ = self.net.microstep(self.z, self.x, noise=self.noise, sigma=0.0, alpha=self.alpha)
        return z_next

    def step(self, z: Tensor, x: Tensor, noise: Tensor, alpha=None) -> Tensor:
        self.z.copy_(z)
        self.x.copy_(x)
        self.noise.copy_(noise)
        if torch.is_tensor(self.alpha):
            self.alpha.copy_(alpha)
        self.graph.replay()
        return self.out


def graphed_microstep(net: LatentEnergyNet, z: Tensor, x: Tensor, noise: Tensor, alpha=None) -> Tensor:
    """``net.microstep(z, x, noise=noise, sigma=0, alpha=alpha)[0]`` without a graph, through the net's cached
    ``MicrostepGraph`` for this shape (captured on first use). The result is the graph's buffer: clone it to keep it
    past the next graphed microstep of the same shape."""
    alpha = net.shape.step_size if alpha is None else alpha
    key = (tuple(z.shape), z.dtype, tuple(x.shape), tuple(alpha.shape) if torch.is_tensor(alpha) else float(alpha))
    cache = net.__dict__.setdefault("_microstep_graphs", {})
    graph = cache.get(key)
    if graph is None:
        graph = cache[key] = MicrostepGraph(net, z, x, alpha)
    return graph.step(z, x, noise, alpha)


def train_segment_loss(net: LatentEnergyNet, z: Tensor, x: Tensor, labels: Tensor, prefix: int, graded: int,
                       alpha=None) -> Tensor:  # fmt: skip
    """A training segment: ``prefix`` microsteps without a graph, then ``graded`` with ``create_graph=True`` (so the
    backward runs the attention's double backward), and the mean stablemax cross entropy of the decoded endpoint
    against ``labels`` (``models/energy.py:582-636`` rollout, ``models/losses.py`` loss)."""
    sigma = net.shape.noise_scale
    with torch.no_grad():
        for _ in range(prefix):
            noise = torch.randn_like(z) * sigma if sigma else torch.zeros_like(z)
            z = graphed_microstep(net, z, x, noise, alpha)
        z = z.clone()
    for _ in range(graded):
        z, _ = net.microstep(z, x, graded=True, alpha=alpha)
    return stablemax_cross_entropy(net.decode(z), labels).mean()


def sxm_explore_loss(net: LatentEnergyNet, z: Tensor, challengers: Tensor, x: Tensor, labels: Tensor, prefix: int,
                     graded: int, alpha=None, sigma: Optional[float] = None) -> tuple[Tensor, Tensor, Tensor]:  # fmt: skip
    """Forward SXM for one training segment (the algorithm of the reference's ``InnerNetwork.explore``,
    ``models/energy.py:669-733``): K candidate trajectories per input -- the input's own state ``z`` [B, L, C] and
    ``challengers`` [K - 1, B, L, C] -- run the whole segment as one batch without a graph, with noise drawn once per
    microstep; each input keeps the candidate whose decoded endpoint has the lowest stablemax cross entropy against
    ``labels``; the winner's graded window is run again from its state at the window's start with the same noise and
    ``create_graph=True`` (so only one trajectory per input is differentiated twice).

    Returns (loss of the recomputed winners, their endpoints, the K - 1 losers' endpoints as the next challengers
    [K - 1, B, L, C], best first). An input's candidates stay together in the batch, so the batch shards over ranks
    by input."""
    k, b = challengers.shape[0] + 1, z.shape[0]
    sigma = net.shape.noise_scale if sigma is None else sigma
    steps = prefix + graded
    cand = torch.cat([z.detach(), challengers.reshape(-1, *z.shape[1:]).to(z.dtype)])
    xk, lk = x.repeat(k, 1, 1), labels.repeat(k, 1)
    noise = [torch.randn_like(cand) * sigma for _ in range(steps)] if sigma else None
    with torch.no_grad():
        zc, start = cand, cand
        for t in range(steps):
            if t == prefix:
                start = zc.clone()
            zc = graphed_microstep(net, zc, xk, torch.zeros_like(cand) if noise is None else noise[t], alpha)
        zc = zc.clone()
        per_row = stablemax_cross_entropy(net.decode(zc), lk).mean(-1).view(k, b)
        order = per_row.argsort(dim=0)  # best candidate first, per input
    rows = torch.arange(b, device=z.device)
    pick = lambda t: t.view(k, b, *t.shape[1:])[order[0], rows]  # noqa: E731
    zw = pick(start)
    for t in range(prefix, steps):
        zw, _ = net.microstep(zw, x, graded=True, noise=None if noise is None else pick(noise[t]), sigma=0.0,
                              alpha=alpha)  # fmt: skip
    loss = stablemax_cross_entropy(net.decode(zw), labels).mean()
    losers = zc.view(k, b, *z.shape[1:])[order[1:], rows.unsqueeze(0)]
    return loss, zw.detach(), losers


__all__ = [
    "LatentEnergyNet",
    "NetShape",
    "board_unit_rms",
    "cell_unit_rms",
    "descend",
    "graphed_microstep",
    "lowest_energy_pick",
    "rope_tables",
    "stablemax_cross_entropy",
    "sxm_explore_loss",
    "train_segment_loss",
]
