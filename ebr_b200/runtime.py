"""Data-parallel plumbing over ``torch.distributed`` (NCCL on GPU, gloo on CPU).

The reference (``utils/runtime.py:95-139``) broadcasts the weights at start, all-reduces every parameter's gradient
separately after the backward, and all-gathers a parameter checksum at checkpoints. The B200 build keeps the same
collectives but reduces all gradients as ONE flat fp32 bucket (one NCCL call per step instead of one per tensor),
which over NVLink 5 / NVSwitch makes the reduction a fixed ~55 MB transfer per step for the benchmark model.
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


@torch.no_grad()
def allreduce_gradients(params: list[torch.Tensor], average: bool = False) -> int:
    """Sum every parameter gradient over ranks in one flat fp32 bucket. Returns the bucket's element count.

    Same result as the reference's per-tensor ``all_reduce(SUM)`` (``utils/runtime.py:118-124``); a parameter without
    a gradient contributes zeros and receives the sum (as a fresh gradient) when any rank has one.
    """
    ps = [p for p in params if p.requires_grad]
    if not ps:
        return 0
    dev = ps[0].device
    flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1).to(torch.float32)
                      for p in ps]).to(dev)  # fmt: skip
    if world() > 1:
        dist.all_reduce(flat, op=dist.ReduceOp.SUM)
        if average:
            flat /= world()
    off = 0
    for p in ps:
        n = p.numel()
        g = flat[off : off + n].view_as(p).to(p.dtype)
        if p.grad is None:
            p.grad = g.clone()
        else:
            p.grad.copy_(g)
        off += n
    return int(flat.numel())


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
