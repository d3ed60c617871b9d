"""Data-parallel plumbing over ``torch.distributed`` (NCCL on GPU, gloo on CPU).

The reference (``utils/runtime.py:95-139``) broadcasts the weights at start, all-reduces every parameter's gradient
separately after the whole backward, and all-gathers a parameter checksum at checkpoints. This module keeps the same
collectives and results, with two B200-side changes to the gradient reduction:

* ``allreduce_gradients``: all gradients as ONE flat fp32 bucket (one NCCL call per step instead of one per tensor);
* ``GradientBuckets``: the gradients in a few buckets of ~16 MB, each all-reduced asynchronously as soon as the outer
  backward has produced all of its gradients (post-accumulate hooks), so the transfers over NVLink overlap the rest of
  the backward; ``finish()`` waits for them after the backward.

Either way a parameter that no rank produced a gradient for keeps ``grad = None`` (the reference skips such tensors,
``utils/runtime.py:122``, so the optimizer skips them too); a parameter some ranks left without one receives the sum.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def init_distributed(timeout_s: float = 120.0) -> tuple[int, int, int]:
    """(rank, world, local_rank) from the torchrun environment; (0, 1, 0) when not launched by torchrun."""
    if "RANK" not in os.environ or int(os.environ.get("WORLD_SIZE", "1")) <= 1:
        return 0, 1, 0
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
        backend = "nccl"
    else:
        backend = "gloo"
    if not dist.is_initialized():
        kw = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(**kw)
    return rank, world, local


def world() -> int:
    return dist.get_world_size() if dist.is_initialized() else 1


@torch.no_grad()
def broadcast_model(model: torch.nn.Module, src: int = 0) -> None:
    """Every parameter and buffer from rank ``src`` (``utils/runtime.py:109-115``)."""
    if world() == 1:
        return
    for t in list(model.parameters()) + list(model.buffers()):
        dist.broadcast(t.data, src)


def _presence(ps: list[torch.Tensor], dev) -> torch.Tensor:
    return torch.tensor([p.grad is not None for p in ps], dtype=torch.float32, device=dev)


@torch.no_grad()
def allreduce_gradients(params: list[torch.Tensor], average: bool = False) -> int:
    """Sum every parameter gradient over ranks in one flat fp32 bucket. Returns the bucket's element count.

    Same result as the reference's per-tensor ``all_reduce(SUM)`` (``utils/runtime.py:118-124``): a parameter without
    a gradient contributes zeros; it receives the sum when any rank has one and stays ``None`` when no rank has.
    """
    ps = [p for p in params if p.requires_grad]
    if not ps:
        return 0
    dev = ps[0].device
    present = _presence(ps, dev)
    if world() == 1:
        return int(sum(p.numel() for p in ps))
    flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1).to(torch.float32)
                      for p in ps] + [present])  # fmt: skip
    dist.all_reduce(flat, op=dist.ReduceOp.SUM)
    if average:
        flat[: flat.numel() - len(ps)] /= world()
    _scatter_back(ps, flat, flat[flat.numel() - len(ps) :])
    return int(flat.numel() - len(ps))


def _scatter_back(ps: list[torch.Tensor], flat: torch.Tensor, present: torch.Tensor) -> None:
    off = 0
    keep = present.gt(0).tolist()
    for p, k in zip(ps, keep):
        n = p.numel()
        if not k:
            p.grad = None
        else:
            g = flat[off : off + n].view_as(p).to(p.dtype)
            if p.grad is None:
                p.grad = g.clone()
            else:
                p.grad.copy_(g)
        off += n


class GradientBuckets:
    """Bucketed gradient all-reduce overlapped with the outer backward.

    ``params`` are split, in reverse registration order (the backward reaches the last layers first), into buckets of
    about ``bucket_mb`` MB of fp32. A post-accumulate-grad hook copies each finished gradient into its bucket; once
    a bucket and every bucket before it are complete, it is all-reduced with ``async_op=True`` on the collective's
    own stream while the backward goes on (in index order on every rank, as collectives must be). Use per step::

        buckets.start()          # before the backward
        loss.backward()
        buckets.finish()         # launches what is left, waits, writes the sums back into .grad

    No other collective may be issued between ``start()`` and ``finish()``: buckets already in flight on one rank
    would then meet it out of order on another.

    With one process it only applies the ``None`` rule above. The presence of each gradient is summed alongside, in
    the last bucket's call.
    """

    def __init__(self, params: list[torch.Tensor], bucket_mb: float = 16.0, average: bool = False) -> None:
        self.params = [p for p in params if p.requires_grad]
        self.average = average
        self.world = world()
        cap = max(1, int(bucket_mb * (1 << 20) / 4))
        self.buckets: list[list[int]] = []  # parameter indices per bucket
        cur, size = [], 0
        for i in reversed(range(len(self.params))):
            n = self.params[i].numel()
            if cur and size + n > cap:
                self.buckets.append(cur)
                cur, size = [], 0
            cur.append(i)
            size += n
        if cur:
            self.buckets.append(cur)
        self.where: dict[int, tuple[int, int]] = {}  # param index -> (bucket, offset)
        self.sizes = []
        for b, idx in enumerate(self.buckets):
            off = 0
            for i in idx:
                self.where[i] = (b, off)
                off += self.params[i].numel()
            self.sizes.append(off)
        dev = self.params[0].device if self.params else torch.device("cpu")
        self.flat = [torch.zeros(n, dtype=torch.float32, device=dev) for n in self.sizes]
        self.present = torch.zeros(len(self.params), dtype=torch.float32, device=dev)
        self.index = {id(p): i for i, p in enumerate(self.params)}
        self.pending = [0] * len(self.buckets)
        self.handles: list = [None] * len(self.buckets)
        self.active = False
        self.next_launch = 0
        self.launched_early = 0
        for p in self.params:
            p.register_post_accumulate_grad_hook(self._hook)

    def start(self) -> None:
        for f in self.flat:
            f.zero_()
        self.present.zero_()
        self.pending = [len(idx) for idx in self.buckets]
        self.handles = [None] * len(self.buckets)
        self.next_launch = 0
        self.launched_early = 0
        self.active = True

    @torch.no_grad()
    def _hook(self, p: torch.Tensor) -> None:
        if not self.active:
            return
        i = self.index[id(p)]
        b, off = self.where[i]
        self.flat[b][off : off + p.numel()].copy_(p.grad.reshape(-1))
        self.present[i] = 1.0
        self.pending[b] -= 1
        # Launch complete buckets strictly in index order, so every rank issues the same collectives in the same
        # order even when a parameter has no gradient on some rank (its bucket then waits for finish() everywhere
        # after it). The last bucket always waits for finish(): it carries the presence flags.
        while self.world > 1 and self.next_launch < len(self.buckets) - 1 and self.pending[self.next_launch] == 0:
            b0 = self.next_launch
            self.handles[b0] = dist.all_reduce(self.flat[b0], op=dist.ReduceOp.SUM, async_op=True)
            self.next_launch += 1
            self.launched_early += 1

    @torch.no_grad()
    def finish(self) -> None:
        """Launch the buckets still waiting (some gradient missing on this rank: it contributes zeros), wait for
        every bucket, and write the sums back (``None`` where no rank had a gradient)."""
        self.active = False
        last = len(self.buckets) - 1
        if self.world > 1:
            for b in range(self.next_launch, len(self.buckets)):
                if self.handles[b] is None:
                    if b == last:
                        # the presence flags ride along in the last bucket's call
                        buf = torch.cat([self.flat[b], self.present])
                        dist.all_reduce(buf, op=dist.ReduceOp.SUM)
                        self.flat[b].copy_(buf[: self.sizes[b]])
                        self.present.copy_(buf[self.sizes[b] :])
                    else:
                        self.handles[b] = dist.all_reduce(self.flat[b], op=dist.ReduceOp.SUM, async_op=True)
            for h in self.handles:
                if h is not None:
                    h.wait()
        keep = self.present.gt(0).tolist()
        for b, idx in enumerate(self.buckets):
            flat = self.flat[b]
            if self.average and self.world > 1:
                flat /= self.world
            for i in idx:
                p = self.params[i]
                _, off = self.where[i]
                if not keep[i]:
                    p.grad = None
                elif p.grad is None:
                    p.grad = flat[off : off + p.numel()].view_as(p).to(p.dtype).clone()
                else:
                    p.grad.copy_(flat[off : off + p.numel()].view_as(p))


@torch.no_grad()
def param_checksum(model: torch.nn.Module) -> float:
    return float(sum(p.detach().double().sum().item() for p in model.parameters()))


@torch.no_grad()
def check_param_sync(model: torch.nn.Module, rtol: float = 0.0) -> list[float]:
    """All-gather one float64 parameter checksum per rank and raise if they differ (``utils/runtime.py:127-139``)."""
    local = torch.tensor([param_checksum(model)], dtype=torch.float64)
    if world() == 1:
        return [local.item()]
    if dist.get_backend() == "nccl":
        local = local.cuda()
    outs = [torch.zeros_like(local) for _ in range(world())]
    dist.all_gather(outs, local)
    vals = [o.item() for o in outs]
    ref = vals[0]
    if any(abs(v - ref) > rtol * max(abs(ref), 1.0) for v in vals):
        raise RuntimeError(f"parameters diverged across ranks: checksums {vals}")
    return vals


@torch.no_grad()
def max_over_ranks(value: float) -> float:
    """The maximum of a host float over ranks (device timing is reported as the slowest rank)."""
    if world() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64)
    if dist.get_backend() == "nccl":
        t = t.cuda()
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
